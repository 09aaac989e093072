// Fold a user LoRA into the rank-128 LoRA slots of a MOSS q8 weight set (the SVD fold of the reference's
// moss/mossrun/lorafold.cpp:200-284 `fold` + `fold_block`), on the loaded device weights.
//
// A LoRA-carrying MOSS matrix holds its current ("turbo") rank-128 LoRA as two parts: the B side as 128
// extra K columns of the base matrix W[N][K_base + 128] (already multiplied by its scale), and the A side
// as 128 rows of a LoRA-A matrix A[128][K_base] (export_moss.py:14-27). The LoRA adds B^T-side x A to
// the projection. Folding a user LoRA (B_u [N][r], A_u [r][K_base], scale s) means: stack
//     BT = [turbo B^T ; s B_u^T]   (R x N),   AM = [turbo A ; A_u]   (R x K_base),   R = 128 + r,
// whose product BT^T AM is the combined delta, and replace the slots by its best rank-128
// approximation (Eckart-Young), computed without forming the N x K_base product:
//   1. Gram matrices Gb = BT BT^T and Ga = AM AM^T (R x R, float64, on the GPU);
//   2. their eigendecompositions Gb = Vb diag(lb) Vb^T, Ga = Va diag(la) Va^T (host, cyclic Jacobi),
//      so BT^T = Ub Sb Vb^T and AM = Va Sa Ua^T with Sb = sqrt(lb), Sa = sqrt(la) and Ub, Ua orthonormal;
//   3. the R x R core C = Sb Vb^T Va Sa, so BT^T AM = Ub C Ua^T; its SVD C = U S W^T from the
//      eigendecomposition of C^T C (host, cyclic Jacobi; U = C W S^-1);
//   4. keep the 128 largest singular values: B'^T = Ub U_k S_k, A' = W_k^T Ua^T, i.e.
//      B' = Tb^T BT with Tb = Vb Sb^-1 U_k S_k  (R x 128)  and  A' = Ta AM with Ta = W_k^T Sa^-1 Va^T;
//      the singular values go to the B side, as in the reference;
//   5. requantise B' into the 128 LoRA K columns of W and A' into the LoRA-A rows, per K-group with
//      the pack rule (lorafold.cpp:138-156: a = fp16(v), s = fp16(max|a| / 127) floored at 6.2e-5,
//      q = rint(a / s) clipped to +-127).
// Eigenvalues below 1e-12 of the largest are treated as zero (rank-deficient slots, e.g. unused turbo
// rows). The eigen/SVD solvers differ from the reference's one-sided Jacobi, so the folded factors
// match it up to rounding and the sign / rotation freedom of equal singular values, not bit for bit.
#include <algorithm>
#include <cmath>
#include <numeric>
#include <vector>

#include "hx_internal.h"

namespace hx {

namespace {

constexpr int KEEP = 128;  // rank of the LoRA slots
constexpr int GT = 16;     // Gram tile

// BT[r][n] (rows padded to Rp with zeros): r < 128 the dequantised LoRA K column k_base + r of W,
// r < R the scaled user B (logical row of device row n), else 0
__global__ void gather_b_kernel(float* __restrict__ BT, int Rp, int R, int N, const uint8_t* __restrict__ w,
                                const __half* __restrict__ wsc, int K, int group, int k_base,
                                const float* __restrict__ Bu, int rank, float scale, int row_mode, int F) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x, r = blockIdx.y;
  if (n >= N || r >= Rp) return;
  float v = 0.f;
  if (r < KEEP) {
    const int k = k_base + r;
    v = static_cast<float>(static_cast<int>(w[static_cast<size_t>(n) * K + k]) - 128) *
        __half2float(wsc[static_cast<size_t>(k / group) * N + n]);
  } else if (r < R) {
    int ln = n;
    if (row_mode == 1) {  // up_gate: device rows per 256 are [128 up, 128 gate] of the same outputs
      const int t = n / 256, l = n % 256, o = t * 128 + (l & 127);
      ln = l < 128 ? o : F + o;
    }
    v = scale * Bu[static_cast<size_t>(ln) * rank + (r - KEEP)];
  }
  BT[static_cast<size_t>(r) * N + n] = v;
}

// AM[r][i]: r < 128 the dequantised LoRA-A row a_row0 + r, r < R the user A row r - 128, else 0
__global__ void gather_a_kernel(float* __restrict__ AM, int Rp, int R, int I, const uint8_t* __restrict__ a,
                                const __half* __restrict__ asc, int NA, int group, int a_row0,
                                const float* __restrict__ Au) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x, r = blockIdx.y;
  if (i >= I || r >= Rp) return;
  float v = 0.f;
  if (r < KEEP) {
    const int row = a_row0 + r;
    v = static_cast<float>(static_cast<int>(a[static_cast<size_t>(row) * I + i]) - 128) *
        __half2float(asc[static_cast<size_t>(i / group) * NA + row]);
  } else if (r < R) {
    v = Au[static_cast<size_t>(r - KEEP) * I + i];
  }
  AM[static_cast<size_t>(r) * I + i] = v;
}

// G = X X^T for X [Rp][n] (Rp a multiple of 16), float64 sums of float32 products; one 16x16 tile of G
// per block, X staged 64 columns at a time
__global__ void __launch_bounds__(GT * GT) gram_kernel(const float* __restrict__ X, int Rp, int n,
                                                       double* __restrict__ G) {
  __shared__ float sa[GT][65], sb[GT][65];
  const int i0 = blockIdx.y * GT, j0 = blockIdx.x * GT;
  if (j0 < i0) return;  // upper triangle of tiles; mirrored below
  const int tx = threadIdx.x % GT, ty = threadIdx.x / GT;
  double acc = 0.0;
  for (int c0 = 0; c0 < n; c0 += 64) {
    for (int e = threadIdx.x; e < GT * 64; e += GT * GT) {
      const int r = e / 64, c = e % 64;
      sa[r][c] = c0 + c < n ? X[static_cast<size_t>(i0 + r) * n + c0 + c] : 0.f;
      sb[r][c] = c0 + c < n ? X[static_cast<size_t>(j0 + r) * n + c0 + c] : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int c = 0; c < 64; ++c) acc += static_cast<double>(sa[ty][c]) * static_cast<double>(sb[tx][c]);
    __syncthreads();
  }
  G[static_cast<size_t>(i0 + ty) * Rp + j0 + tx] = acc;
  G[static_cast<size_t>(j0 + tx) * Rp + i0 + ty] = acc;
}

// Y[k][c] = sum_r coef[r][k] * X[r][c] for k < 128 (coef [Rp][128]); fp32 sums in order of r
__global__ void project_kernel(const float* __restrict__ coef, const float* __restrict__ X, int Rp, int n,
                               float* __restrict__ Y) {
  __shared__ float sc[256][8];
  const int c = blockIdx.x * blockDim.x + threadIdx.x, k0 = blockIdx.y * 8;
  for (int e = threadIdx.x; e < Rp * 8; e += blockDim.x) sc[e / 8][e % 8] = coef[static_cast<size_t>(e / 8) * KEEP + k0 + e % 8];
  __syncthreads();
  if (c >= n) return;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int r = 0; r < Rp; ++r) {
    const float x = X[static_cast<size_t>(r) * n + c];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = fmaf(sc[r][j], x, acc[j]);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) Y[static_cast<size_t>(k0 + j) * n + c] = acc[j];
}

__device__ __forceinline__ void quant_group(const float* v, int g, uint8_t* q, int qstride, __half* s) {
  float m = 0.f;
  for (int j = 0; j < g; ++j) m = fmaxf(m, fabsf(__half2float(__float2half_rn(v[j]))));
  float sf = m / 127.0f;
  if (sf < 6.2e-5f) sf = 6.2e-5f;
  const __half s16 = __float2half_rn(sf);
  const float sd = __half2float(s16);
  for (int j = 0; j < g; ++j) {
    const float a = __half2float(__float2half_rn(v[j]));
    const float qq = fminf(127.f, fmaxf(-127.f, rintf(a / sd)));
    q[static_cast<size_t>(j) * qstride] = static_cast<uint8_t>(static_cast<int>(qq) + 128);
  }
  *s = s16;
}

// B' [128][N] into W[n][k_base + k]: one thread per (n, K-group of the 128 LoRA columns)
__global__ void requant_b_kernel(const float* __restrict__ Bo, int N, uint8_t* __restrict__ w, __half* __restrict__ wsc,
                                 int K, int group, int k_base) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x, gi = blockIdx.y;
  if (n >= N) return;
  float v[64];
  for (int j = 0; j < group; ++j) v[j] = Bo[static_cast<size_t>(gi * group + j) * N + n];
  const int k = k_base + gi * group;
  quant_group(v, group, w + static_cast<size_t>(n) * K + k, 1, wsc + static_cast<size_t>(k / group) * N + n);
}

// A' [128][I] into the LoRA-A rows a_row0 + k: one thread per (row, K-group)
__global__ void requant_a_kernel(const float* __restrict__ Ao, int I, uint8_t* __restrict__ a, __half* __restrict__ asc,
                                 int NA, int group, int a_row0) {
  const int gi = blockIdx.x * blockDim.x + threadIdx.x, k = blockIdx.y;
  if (gi >= I / group) return;
  float v[64];
  for (int j = 0; j < group; ++j) v[j] = Ao[static_cast<size_t>(k) * I + gi * group + j];
  const int row = a_row0 + k;
  quant_group(v, group, a + static_cast<size_t>(row) * I + gi * group, 1,
              asc + static_cast<size_t>(gi) * NA + row);
}

// Symmetric eigendecomposition by the cyclic Jacobi method (Jacobi 1846; Rutishauser's rotation
// formulas): A [n][n] is destroyed; V columns are the eigenvectors (V[t * n + i] = component t of
// vector i), w the eigenvalues.
void jacobi_eig(std::vector<double>& A, int n, std::vector<double>& V, std::vector<double>& w) {
  V.assign(static_cast<size_t>(n) * n, 0.0);
  for (int i = 0; i < n; ++i) V[static_cast<size_t>(i) * n + i] = 1.0;
  auto at = [&](int r, int c) -> double& { return A[static_cast<size_t>(r) * n + c]; };
  for (int sweep = 0; sweep < 60; ++sweep) {
    double off = 0.0, diag = 0.0;
    for (int p = 0; p < n; ++p) {
      diag += at(p, p) * at(p, p);
      for (int q = p + 1; q < n; ++q) off += at(p, q) * at(p, q);
    }
    if (off <= 1e-30 * diag || off == 0.0) break;
    for (int p = 0; p < n - 1; ++p) {
      for (int q = p + 1; q < n; ++q) {
        const double apq = at(p, q);
        if (apq == 0.0) continue;
        const double theta = (at(q, q) - at(p, p)) / (2.0 * apq);
        const double t = (theta >= 0.0 ? 1.0 : -1.0) / (std::fabs(theta) + std::sqrt(theta * theta + 1.0));
        const double c = 1.0 / std::sqrt(t * t + 1.0), s = t * c, tau = s / (1.0 + c);
        at(p, p) -= t * apq;
        at(q, q) += t * apq;
        at(p, q) = at(q, p) = 0.0;
        for (int r = 0; r < n; ++r) {
          if (r != p && r != q) {
            const double arp = at(r, p), arq = at(r, q);
            at(r, p) = at(p, r) = arp - s * (arq + tau * arp);
            at(r, q) = at(q, r) = arq + s * (arp - tau * arq);
          }
          const double vrp = V[static_cast<size_t>(r) * n + p], vrq = V[static_cast<size_t>(r) * n + q];
          V[static_cast<size_t>(r) * n + p] = vrp - s * (vrq + tau * vrp);
          V[static_cast<size_t>(r) * n + q] = vrq + s * (vrp - tau * vrq);
        }
      }
    }
  }
  w.resize(n);
  for (int i = 0; i < n; ++i) w[i] = at(i, i);
}

}  // namespace

// Host part of the fold: from the two Gram matrices g2 = [Gb ; Ga] (each n x n, row-major) to the
// coefficients [Tb (n x 128) ; Ta^T (n x 128)] (float32, row-major) that turn BT into B' and AM into A'.
std::vector<float> slot_fold_coefs(const std::vector<double>& g2, int n) {
  std::vector<double> Gb(g2.begin(), g2.begin() + static_cast<size_t>(n) * n), Ga(g2.begin() + static_cast<size_t>(n) * n, g2.end());
  std::vector<double> Vb, lb, Va, la;
  jacobi_eig(Gb, n, Vb, lb);
  jacobi_eig(Ga, n, Va, la);
  auto roots = [&](const std::vector<double>& l, std::vector<double>& sq, std::vector<double>& inv) {
    const double mx = *std::max_element(l.begin(), l.end());
    sq.assign(n, 0.0);
    inv.assign(n, 0.0);
    for (int i = 0; i < n; ++i)
      if (mx > 0.0 && l[i] > mx * 1e-12) {
        sq[i] = std::sqrt(l[i]);
        inv[i] = 1.0 / sq[i];
      }
  };
  std::vector<double> sb, ib, sa, ia;
  roots(lb, sb, ib);
  roots(la, sa, ia);
  std::vector<double> C(static_cast<size_t>(n) * n, 0.0);  // C = Sb Vb^T Va Sa
  for (int i = 0; i < n; ++i) {
    if (sb[i] == 0.0) continue;
    for (int j = 0; j < n; ++j) {
      if (sa[j] == 0.0) continue;
      double d = 0.0;
      for (int t = 0; t < n; ++t) d += Vb[static_cast<size_t>(t) * n + i] * Va[static_cast<size_t>(t) * n + j];
      C[static_cast<size_t>(i) * n + j] = sb[i] * d * sa[j];
    }
  }
  std::vector<double> CtC(static_cast<size_t>(n) * n, 0.0);
  for (int i = 0; i < n; ++i)
    for (int j = i; j < n; ++j) {
      double d = 0.0;
      for (int t = 0; t < n; ++t) d += C[static_cast<size_t>(t) * n + i] * C[static_cast<size_t>(t) * n + j];
      CtC[static_cast<size_t>(i) * n + j] = CtC[static_cast<size_t>(j) * n + i] = d;
    }
  std::vector<double> Wv, sv2;
  jacobi_eig(CtC, n, Wv, sv2);
  std::vector<int> ord(n);
  std::iota(ord.begin(), ord.end(), 0);
  std::stable_sort(ord.begin(), ord.end(), [&](int x, int y) { return sv2[x] > sv2[y]; });
  const double smax = std::sqrt(std::max(sv2[ord[0]], 0.0));
  std::vector<float> hcoef(static_cast<size_t>(2) * n * KEEP, 0.f);  // Tb [n][128], then Ta^T [n][128]
  std::vector<double> u(n), wcol(n);
  for (int c = 0; c < KEEP && c < n; ++c) {
    const int j = ord[c];
    const double sj = std::sqrt(std::max(sv2[j], 0.0));
    if (!(sj > smax * 1e-12)) continue;
    for (int i = 0; i < n; ++i) wcol[i] = Wv[static_cast<size_t>(i) * n + j];
    for (int i = 0; i < n; ++i) {  // u = C w / s
      double d = 0.0;
      for (int t = 0; t < n; ++t) d += C[static_cast<size_t>(i) * n + t] * wcol[t];
      u[i] = d / sj;
    }
    for (int t = 0; t < n; ++t) {
      double xb = 0.0, xa = 0.0;
      for (int i = 0; i < n; ++i) {
        xb += Vb[static_cast<size_t>(t) * n + i] * ib[i] * u[i];
        xa += Va[static_cast<size_t>(t) * n + i] * ia[i] * wcol[i];
      }
      hcoef[static_cast<size_t>(t) * KEEP + c] = static_cast<float>(xb * sj);
      hcoef[static_cast<size_t>(n) * KEEP + static_cast<size_t>(t) * KEEP + c] = static_cast<float>(xa);
    }
  }
  return hcoef;
}

// W: the LoRA-carrying matrix (q8, K = k_base + 128); A: the LoRA-A matrix (q8, K = k_base) whose rows
// a_row0 .. a_row0 + 127 are this projection's slots. Bu [N][rank] in the matrix's logical row order
// (row_mode 1: MOSS up_gate), Au [rank][k_base], both fp32 on the device.
cudaError_t lora_fold_slots(const DevMat& W, int k_base, int row_mode, const DevMat& A, int a_row0, const float* Bu,
                            const float* Au, int rank, float scale, cudaStream_t s) {
  if (W.fmt != WF_Q8 || A.fmt != WF_Q8 || !Bu || !Au || rank < 1 || rank > 128) return cudaErrorInvalidValue;
  if (W.K != k_base + KEEP || A.K != k_base || a_row0 < 0 || a_row0 + KEEP > A.N) return cudaErrorInvalidValue;
  if ((W.group != 32 && W.group != 64) || (A.group != 32 && A.group != 64) || k_base % 64) return cudaErrorInvalidValue;
  if (row_mode == 1 && W.N % 256) return cudaErrorInvalidValue;
  const int N = W.N, I = k_base, R = KEEP + rank, Rp = (R + GT - 1) / GT * GT;
  float *BT = nullptr, *AM = nullptr, *coef = nullptr, *Y = nullptr;
  double* G = nullptr;
  cudaError_t e = cudaSuccess;
  auto fail = [&](cudaError_t x) {
    cudaStreamSynchronize(s);
    cudaFree(BT);
    cudaFree(AM);
    cudaFree(coef);
    cudaFree(Y);
    cudaFree(G);
    return x;
  };
  if ((e = cudaMalloc(&BT, sizeof(float) * Rp * N)) != cudaSuccess) return fail(e);
  if ((e = cudaMalloc(&AM, sizeof(float) * Rp * I)) != cudaSuccess) return fail(e);
  if ((e = cudaMalloc(&coef, sizeof(float) * 2 * Rp * KEEP)) != cudaSuccess) return fail(e);
  if ((e = cudaMalloc(&Y, sizeof(float) * KEEP * std::max(N, I))) != cudaSuccess) return fail(e);
  if ((e = cudaMalloc(&G, sizeof(double) * 2 * Rp * Rp)) != cudaSuccess) return fail(e);

  gather_b_kernel<<<dim3((N + 255) / 256, Rp), 256, 0, s>>>(BT, Rp, R, N, static_cast<const uint8_t*>(W.w), W.scale,
                                                             W.K, W.group, k_base, Bu, rank, scale, row_mode, N / 2);
  gather_a_kernel<<<dim3((I + 255) / 256, Rp), 256, 0, s>>>(AM, Rp, R, I, static_cast<const uint8_t*>(A.w), A.scale,
                                                             A.N, A.group, a_row0, Au);
  gram_kernel<<<dim3(Rp / GT, Rp / GT), GT * GT, 0, s>>>(BT, Rp, N, G);
  gram_kernel<<<dim3(Rp / GT, Rp / GT), GT * GT, 0, s>>>(AM, Rp, I, G + static_cast<size_t>(Rp) * Rp);
  std::vector<double> hg(static_cast<size_t>(2) * Rp * Rp);
  if ((e = cudaMemcpyAsync(hg.data(), G, sizeof(double) * hg.size(), cudaMemcpyDeviceToHost, s)) != cudaSuccess ||
      (e = cudaStreamSynchronize(s)) != cudaSuccess)
    return fail(e);

  const int n = Rp;
  const std::vector<float> hcoef = slot_fold_coefs(hg, n);
  if ((e = cudaMemcpyAsync(coef, hcoef.data(), sizeof(float) * hcoef.size(), cudaMemcpyHostToDevice, s)) != cudaSuccess)
    return fail(e);

  // B' = Tb^T BT -> LoRA K columns of W; A' = Ta AM -> LoRA-A rows
  project_kernel<<<dim3((N + 255) / 256, KEEP / 8), 256, 0, s>>>(coef, BT, Rp, N, Y);
  requant_b_kernel<<<dim3((N + 127) / 128, KEEP / W.group), 128, 0, s>>>(Y, N, static_cast<uint8_t*>(W.w), W.scale, W.K,
                                                                          W.group, k_base);
  project_kernel<<<dim3((I + 255) / 256, KEEP / 8), 256, 0, s>>>(coef + static_cast<size_t>(n) * KEEP, AM, Rp, I, Y);
  requant_a_kernel<<<dim3((I / A.group + 127) / 128, KEEP), 128, 0, s>>>(Y, I, static_cast<uint8_t*>(A.w), A.scale, A.N,
                                                                          A.group, a_row0);
  e = cudaGetLastError();
  const cudaError_t e2 = cudaStreamSynchronize(s);
  return fail(e != cudaSuccess ? e : e2);
}

}  // namespace hx

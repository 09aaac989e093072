// Weight-only LoRA fold into q8 weights, on the device.
//
// W'[n][k] = q[n][k] * s[g][n] + scale * sum_r B[n][r] * A[r][k]   for k < k_base, then every K-group
// of W' is requantised with the q8 pack rule of the reference's fold tool (lorafold.cpp:138-156
// `quant`, the same rule as export_all_q8.py:10-18): a = fp16(W'), s' = fp16(max|a| / 127) with the
// model's floor (MOSS: < 6.2e-5 -> 6.2e-5; Anima: 0 -> 1.0), q' = clip(rint(a / s'), -127, 127).
// The reference folds a user LoRA into the rank-128 LoRA slots by SVD (lorafold.cpp:200-284); this
// is the variant that adds a rank <= 128 delta into the base tiles themselves.
//
// The arithmetic is fixed so that a CPU restatement reproduces the bytes exactly: the rank sum runs
// in order r = 0 .. rank-1 with separately rounded products and sums (no FMA contraction), then
// one rounded multiply by `scale` and one rounded add to the dequantised weight; the divisions are
// IEEE divisions.
//
// Device layout (gemm.cu): u8 W[N][K] offset binary (u = q + 128), fp16 scale[K/group][N]. Columns
// [k_base, K) (the appended LoRA K rows of MOSS packs) are left untouched. B rows are given in the
// matrix's logical order; row_mode 1 is the MOSS up_gate regrouping of repack.cu (device rows per
// 256: [0,128) up, [128,256) gate of the same 128 outputs; logical rows [0,F) up, [F,2F) gate).
#include "hx_internal.h"

namespace hx {

namespace {

constexpr int FOLD_ROWS = 16;   // rows per CTA: 8 warps x 2
constexpr int FOLD_K = 128;     // columns per CTA: 32 lanes x 4
constexpr int FOLD_RC = 32;     // rank chunk staged in shared memory

__device__ __forceinline__ int logical_row(int r, int row_mode, int F) {
  if (row_mode == 1) {
    const int t = r / 256, l = r % 256, o = t * 128 + (l & 127);
    return l < 128 ? o : F + o;
  }
  return r;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__global__ void __launch_bounds__(256) lora_fold_kernel(uint8_t* __restrict__ u, __half* __restrict__ scale, int N,
                                                        int K, int k_base, int group, const float* __restrict__ B,
                                                        const float* __restrict__ A, int rank, float lscale,
                                                        int row_mode, int F, int floor_mode) {
  __shared__ float sB[FOLD_ROWS][FOLD_RC];
  __shared__ float sA[FOLD_RC][FOLD_K];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k0 = blockIdx.x * FOLD_K, n0 = blockIdx.y * FOLD_ROWS;
  float acc[2][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int rc = 0; rc < rank; rc += FOLD_RC) {
    const int nr = min(FOLD_RC, rank - rc);
    __syncthreads();  // previous chunk consumed
    for (int i = threadIdx.x; i < FOLD_ROWS * FOLD_RC; i += blockDim.x) {
      const int row = i / FOLD_RC, rr = i % FOLD_RC;
      sB[row][rr] = rr < nr ? B[static_cast<size_t>(logical_row(n0 + row, row_mode, F)) * rank + rc + rr] : 0.f;
    }
    for (int i = threadIdx.x; i < FOLD_RC * FOLD_K; i += blockDim.x) {
      const int rr = i / FOLD_K, kk = i % FOLD_K;
      sA[rr][kk] = rr < nr ? A[static_cast<size_t>(rc + rr) * k_base + k0 + kk] : 0.f;
    }
    __syncthreads();
    for (int rr = 0; rr < nr; ++rr) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float b = sB[2 * warp + i][rr];
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(b, sA[rr][lane + 32 * j]));
      }
    }
  }

  // requantise: lanes of one j cover 32 consecutive k of one row; groups of 64 / 128 pair up j's
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int n = n0 + 2 * warp + i;
    float a[4], m[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = k0 + lane + 32 * j;
      const float q = static_cast<float>(static_cast<int>(u[static_cast<size_t>(n) * K + k]) - 128);
      const float s = __half2float(scale[static_cast<size_t>(k / group) * N + n]);
      const float v = __fadd_rn(q * s, __fmul_rn(lscale, acc[i][j]));  // q * s is exact in fp32
      a[j] = __half2float(__float2half_rn(v));
      m[j] = warp_max(fabsf(a[j]));
    }
    __syncwarp();  // every lane has read the old scales before lane 0 overwrites them
    const int gj = group / 32;  // j's per group: 1, 2 or 4
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float mg = m[j];
      const int j0 = (j / gj) * gj;
      for (int t = j0; t < j0 + gj; ++t) mg = fmaxf(mg, m[t]);
      float s = mg / 127.0f;
      if (floor_mode == 0) {
        if (s < 6.2e-5f) s = 6.2e-5f;
      } else if (s == 0.f) {
        s = 1.0f;
      }
      const __half s16 = __float2half_rn(s);
      const float sf = __half2float(s16);
      const float q = fminf(127.f, fmaxf(-127.f, rintf(a[j] / sf)));
      const int k = k0 + lane + 32 * j;
      u[static_cast<size_t>(n) * K + k] = static_cast<uint8_t>(static_cast<int>(q) + 128);
      if (lane == 0 && j == j0) scale[static_cast<size_t>(k / group) * N + n] = s16;
    }
  }
}

}  // namespace

cudaError_t lora_fold_launch(const DevMat& W, int k_base, const float* B, const float* A, int rank, float lscale,
                             int row_mode, int floor_mode, cudaStream_t s) {
  if (W.fmt != WF_Q8 || !W.w || !W.scale || !B || !A) return cudaErrorInvalidValue;
  if (rank < 1 || rank > 128 || k_base <= 0 || k_base > W.K || k_base % FOLD_K || W.N % FOLD_ROWS) return cudaErrorInvalidValue;
  if (W.group != 32 && W.group != 64 && W.group != 128) return cudaErrorInvalidValue;
  if (row_mode == 1 && W.N % 256) return cudaErrorInvalidValue;
  dim3 grid(k_base / FOLD_K, W.N / FOLD_ROWS);
  lora_fold_kernel<<<grid, 256, 0, s>>>(static_cast<uint8_t*>(W.w), W.scale, W.N, W.K, k_base, W.group, B, A, rank,
                                        lscale, row_mode, W.N / 2, floor_mode);
  return cudaGetLastError();
}

}  // namespace hx

// Per-step glue of the Anima sampler on the GPU (phone/animad.cpp:423-492): timestep embedding,
// t_embedder mat-vecs, patchify, final-layer modulation, unpatchify and the Euler update.
// MOSS sampler glue (moss/sample_ref.py:14-20, moss_ref.py:96-120, mossrun.cpp:306-333): the time
// embedding of the step codes, the latent mix z + Q x0 feeding video_embedder, and x0 = z - v.
// The GEMMs of the glue (x_embedder 68->D, final linear D->64) run on gemm.cu with an fp32-store
// epilogue; the final LayerNorm modulation reuses elem.cu's lnmod.
#include "hx_internal.h"
#include "hx_ptx.cuh"

namespace hx {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// animad.cpp:424-427: tp[i] = cos(t * exp(-ln(1e4) i / (D/2))), tp[i + D/2] = sin(...);
// emb = tp * rsqrt(mean(tp^2) + 1e-6) * w_norm. One block per step.
__global__ void temb_kernel(Sigmas sig, int D, const __half* __restrict__ w_norm, float* __restrict__ tp,
                            float* __restrict__ emb) {
  const int s = blockIdx.x;
  const float t = sig.s[s];
  float* tps = tp + static_cast<size_t>(s) * D;
  float* es = emb + static_cast<size_t>(s) * D;
  const int half = D / 2;
  float ss = 0.f;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float a = t * expf(-logf(10000.f) * static_cast<float>(i) / static_cast<float>(half));
    const float c = cosf(a), sn = sinf(a);
    tps[i] = c;
    tps[i + half] = sn;
    ss += c * c + sn * sn;
  }
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float k = 1.0f / sqrtf(red[0] / static_cast<float>(D) + 1e-6f);
  for (int i = threadIdx.x; i < D; i += blockDim.x) es[i] = tps[i] * k * __half2float(w_norm[i]);
}

// Y[s][o] = add[s][o] + sum_k W[o][k] * f(X[s][k]) for S <= 8 vectors; f = identity or silu.
// One warp per output row; the row of W is read once for all S vectors.
template <int S>
__global__ void gemv_rows_kernel(const __half* __restrict__ W, const float* __restrict__ X, float* __restrict__ Y,
                                 int K, int O, int silu_in, const float* __restrict__ add, int add_ld, int y_ld) {
  const int lane = threadIdx.x & 31;
  const int o = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (o >= O) return;
  const __half* row = W + static_cast<size_t>(o) * K;
  float acc[S];
#pragma unroll
  for (int s = 0; s < S; ++s) acc[s] = 0.f;
  for (int k = lane * 8; k < K; k += 256) {
    const uint4 wv = *reinterpret_cast<const uint4*>(row + k);
    const __half2* w2 = reinterpret_cast<const __half2*>(&wv);
    float wf[8];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 f = __half22float2(w2[t]);
      wf[2 * t] = f.x;
      wf[2 * t + 1] = f.y;
    }
#pragma unroll
    for (int s = 0; s < S; ++s) {
      const float* xs = X + static_cast<size_t>(s) * K + k;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float xv = xs[e];
        if (silu_in) xv = xv / (1.f + expf(-xv));
        acc[s] = fmaf(wf[e], xv, acc[s]);
      }
    }
  }
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const float v = warp_sum(acc[s]);
    if (lane == 0) Y[static_cast<size_t>(s) * y_ld + o] = v + (add ? add[static_cast<size_t>(s) * add_ld + o] : 0.f);
  }
}

// latent [B][C][H][W] -> tokens [B*T][kpad] fp16; feature (c, a, b) -> c*4 + a*2 + b (animad.cpp:447-449),
// features >= C*4 (the zero 17th channel and the K padding) are 0.
__global__ void patchify_kernel(const float* __restrict__ lat, __half* __restrict__ P, int B, int C, int H, int W,
                                int kpad) {
  const int gh = H / 2, gw = W / 2, T = gh * gw;
  const long total = static_cast<long>(B) * T * kpad;
  const long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int f = static_cast<int>(i % kpad);
  const long tok = i / kpad;
  const int b = static_cast<int>(tok / T), t = static_cast<int>(tok % T);
  float v = 0.f;
  if (f < C * 4) {
    const int c = f >> 2, a = (f >> 1) & 1, bb = f & 1;
    const int y = (t / gw) * 2 + a, x = (t % gw) * 2 + bb;
    v = lat[((static_cast<size_t>(b) * C + c) * H + y) * W + x];
  }
  P[i] = __float2half_rn(v);
}

// latent[b][c][gy*2+a][gx*2+bb] += dt * y[b*T + gy*gw + gx][(a*2+bb)*C + c]   (animad.cpp:490-492 layout)
__global__ void unpatch_euler_kernel(const float* __restrict__ y, float* __restrict__ lat, int B, int C, int H,
                                     int W, int ldy, float dt) {
  const long total = static_cast<long>(B) * C * H * W;
  const long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int x = static_cast<int>(i % W);
  const int yy = static_cast<int>((i / W) % H);
  const int c = static_cast<int>((i / (static_cast<long>(W) * H)) % C);
  const int b = static_cast<int>(i / (static_cast<long>(W) * H * C));
  const int gw = W / 2, T = (H / 2) * gw;
  const int tok = (yy / 2) * gw + x / 2;
  const int f = ((yy & 1) * 2 + (x & 1)) * C + c;
  lat[i] += dt * y[(static_cast<size_t>(b) * T + tok) * ldy + f];
}

// dst[r][c] = src[r][c] for c < cols, 0 for cols <= c < ld_dst
__global__ void pad_cols_kernel(const __half* __restrict__ src, __half* __restrict__ dst, int rows, int cols,
                                int ld) {
  const long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long>(rows) * ld) return;
  const int r = static_cast<int>(i / ld), c = static_cast<int>(i % ld);
  dst[i] = c < cols ? src[static_cast<size_t>(r) * cols + c] : __float2half_rn(0.f);
}

}  // namespace

// MOSS time embedding (moss_ref.py:97-100): e[s] = [cos(c_s f_i), sin(c_s f_i)], f_i = 10000^(-i/128),
// computed in float64 and rounded once to float32 like the reference.
__global__ void moss_temb_kernel(Sigmas codes, float* __restrict__ e) {
  const int s = blockIdx.x, i = threadIdx.x;  // 256 threads
  const int j = i & 127;
  const double ph = static_cast<double>(codes.s[s]) * pow(10000.0, -static_cast<double>(j) / 128.0);
  e[s * 256 + i] = static_cast<float>(i < 128 ? cos(ph) : sin(ph));
}

// xin[b][t][:] (fp16, row pitch kp) for the video_embedder GEMM: for image tokens t < Ni the mixed latent
// z[b][o][t] + sum_c Q[o][c] x0[b][c][t] (sample_ref.py:16) in columns 0..127 and 1.0 in column 128 (the
// embedder bias rides in the weight's column 128); text and padding rows t >= Ni are all zero.
// One CTA per (32 tokens, image), thread o = output channel; Q^T and the x0 tile staged in shared memory.
__global__ void __launch_bounds__(128) moss_mix_kernel(const float* __restrict__ z, const float* __restrict__ x0,
                                                       const float* __restrict__ Q, __half* __restrict__ xin,
                                                       int Ni, int ntok, int kp) {
  extern __shared__ float sm[];
  float* qt = sm;               // [128 c][128 o]
  float* xs = sm + 128 * 128;   // [128 c][33]
  const int b = blockIdx.y, t0 = blockIdx.x * 32, o = threadIdx.x;
  for (int i = threadIdx.x; i < 128 * 128; i += blockDim.x) qt[(i % 128) * 128 + i / 128] = Q[i];
  for (int i = threadIdx.x; i < 128 * 32; i += blockDim.x) {
    const int c = i / 32, tt = i % 32;
    xs[c * 33 + tt] = t0 + tt < Ni ? x0[(static_cast<size_t>(b) * 128 + c) * Ni + t0 + tt] : 0.f;
  }
  __syncthreads();
  for (int tt = 0; tt < 32; ++tt) {
    const int t = t0 + tt;
    if (t >= ntok) break;
    __half* row = xin + (static_cast<size_t>(b) * ntok + t) * kp;
    if (t < Ni) {
      float acc = 0.f;
#pragma unroll 8
      for (int c = 0; c < 128; ++c) acc = fmaf(qt[c * 128 + o], xs[c * 33 + tt], acc);
      row[o] = __float2half_rn(z[(static_cast<size_t>(b) * 128 + o) * Ni + t] + acc);
      for (int c = 128 + o; c < kp; c += 128) row[c] = __float2half_rn(c == 128 ? 1.f : 0.f);
    } else {
      for (int c = o; c < kp; c += 128) row[c] = __float2half_rn(0.f);
    }
  }
}

// x0[b][c][t] = z[b][c][t] - v[b*ntok + t][c]   (sample_ref.py:19), t < Ni
__global__ void moss_x0_kernel(const float* __restrict__ z, const float* __restrict__ v, float* __restrict__ x0,
                               int B, int Ni, int ntok, int ldv) {
  const long total = static_cast<long>(B) * 128 * Ni;
  const long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int t = static_cast<int>(i % Ni), c = static_cast<int>((i / Ni) % 128), b = static_cast<int>(i / (128L * Ni));
  x0[i] = z[i] - v[(static_cast<size_t>(b) * ntok + t) * ldv + c];
}

// video_embedder W [D][128] fp16 + bias [D] fp32 -> [D][kp] fp16 with the bias in column 128
__global__ void moss_emb_pad_kernel(const __half* __restrict__ W, const float* __restrict__ bias,
                                    __half* __restrict__ Wp, int D, int kp) {
  const long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long>(D) * kp) return;
  const int r = static_cast<int>(i / kp), c = static_cast<int>(i % kp);
  Wp[i] = c < 128 ? W[static_cast<size_t>(r) * 128 + c] : __float2half_rn(c == 128 ? bias[r] : 0.f);
}

cudaError_t pad_cols_launch(const __half* src, __half* dst, int rows, int cols, int ld_dst, cudaStream_t s) {
  const long total = static_cast<long>(rows) * ld_dst;
  pad_cols_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(src, dst, rows, cols, ld_dst);
  return cudaGetLastError();
}

cudaError_t temb_launch(Sigmas sig, int S, int D, const __half* w_norm, float* tp, float* emb, cudaStream_t s) {
  if (S <= 0 || S > 8 || D % 2) return cudaErrorInvalidValue;
  temb_kernel<<<S, 256, 0, s>>>(sig, D, w_norm, tp, emb);
  return cudaGetLastError();
}

cudaError_t gemv_rows_launch(const __half* W, const float* X, float* Y, int S, int K, int O, int silu_in,
                             const float* add, int add_ld, int y_ld, cudaStream_t s) {
  if (K % 256 || S <= 0 || S > 8) return cudaErrorInvalidValue;
  const int t = 256, grid = (O + t / 32 - 1) / (t / 32);
  switch (S) {
#define HX_GEMV(N) \
  case N: gemv_rows_kernel<N><<<grid, t, 0, s>>>(W, X, Y, K, O, silu_in, add, add_ld, y_ld); break;
    HX_GEMV(1) HX_GEMV(2) HX_GEMV(3) HX_GEMV(4) HX_GEMV(5) HX_GEMV(6) HX_GEMV(7) HX_GEMV(8)
#undef HX_GEMV
  }
  return cudaGetLastError();
}

cudaError_t patchify_launch(const float* lat, __half* P, int B, int C, int H, int W, int kpad, cudaStream_t s) {
  if (H % 2 || W % 2 || kpad < 4 * C) return cudaErrorInvalidValue;
  const long total = static_cast<long>(B) * (H / 2) * (W / 2) * kpad;
  patchify_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(lat, P, B, C, H, W, kpad);
  return cudaGetLastError();
}

cudaError_t unpatch_euler_launch(const float* y, float* lat, int B, int C, int H, int W, int ldy, float dt,
                                 cudaStream_t s) {
  const long total = static_cast<long>(B) * C * H * W;
  unpatch_euler_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(y, lat, B, C, H, W, ldy, dt);
  return cudaGetLastError();
}

cudaError_t moss_temb_launch(Sigmas codes, int S, float* e, cudaStream_t s) {
  if (S <= 0 || S > 8) return cudaErrorInvalidValue;
  moss_temb_kernel<<<S, 256, 0, s>>>(codes, e);
  return cudaGetLastError();
}

cudaError_t moss_mix_launch(const float* z, const float* x0, const float* Q, __half* xin, int B, int Ni, int ntok,
                            int kp, cudaStream_t s) {
  if (B <= 0 || Ni <= 0 || ntok < Ni || kp < 129 || kp % 8) return cudaErrorInvalidValue;
  constexpr int smem = (128 * 128 + 128 * 33) * 4;
  static uint64_t attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set >> dev & 1)) {
    cudaError_t e = cudaFuncSetAttribute(moss_mix_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_set |= 1ull << dev;
  }
  dim3 grid((ntok + 31) / 32, B);
  moss_mix_kernel<<<grid, 128, smem, s>>>(z, x0, Q, xin, Ni, ntok, kp);
  return cudaGetLastError();
}

cudaError_t moss_x0_launch(const float* z, const float* v, float* x0, int B, int Ni, int ntok, int ldv,
                           cudaStream_t s) {
  const long total = static_cast<long>(B) * 128 * Ni;
  moss_x0_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(z, v, x0, B, Ni, ntok, ldv);
  return cudaGetLastError();
}

cudaError_t moss_emb_pad_launch(const __half* W, const float* bias, __half* Wp, int D, int kp, cudaStream_t s) {
  const long total = static_cast<long>(D) * kp;
  moss_emb_pad_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(W, bias, Wp, D, kp);
  return cudaGetLastError();
}

}  // namespace hx

// Memory-bound kernels of the block: AdaLN LayerNorm / RMSNorm modulation (fp32 residual in,
// fp16 operand out), the per-block modulation mat-vecs and small conversions.
//
//  lnmod  : k_ln_prep + k_lnmod_s (hexagon/mega/kern.c:31-65): y = (x-mu)*rstd*(1+scale)+shift,
//           var = E[x^2]-mu^2, no affine, eps 1e-6.
//  rmsmod : k_rms_prep + k_rmsmod_s (moss/hexagon/mega/kern.c:345-375): y = x*rsqrt(E[x^2]+eps)*w*(1+scale)+shift.
//  modulation: the helper-thread mat-vecs of megarun (hexagon/mega/megarun.cpp:158-171):
//           per site h = A[256][D] silu(emb); mod = B[6144][256] h + lora.
// One warp per row, the row held in registers (D/32 floats per lane), 16-byte loads and stores.
#include <mutex>

#include "../../include/hxdit.h"
#include "hx_internal.h"
#include "hx_ptx.cuh"

namespace hx {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// NV = number of float4 per lane (D = 128 * NV)
template <int NV, bool RMS>
__global__ void __launch_bounds__(256) norm_mod_kernel(const float* __restrict__ x, __half* __restrict__ h, int rows,
                                                       const float* __restrict__ w, const float* __restrict__ shift,
                                                       const float* __restrict__ scale, long vec_bstride,
                                                       int rows_per_img, float eps) {
  constexpr int D = 128 * NV;
  grid_dep_wait();  // x is complete
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(row) * D);
  float4 v[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) v[i] = __ldcs(xr + lane + 32 * i);
  float s = 0.f, q = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    q = fmaf(v[i].x, v[i].x, q);
    q = fmaf(v[i].y, v[i].y, q);
    q = fmaf(v[i].z, v[i].z, q);
    q = fmaf(v[i].w, v[i].w, q);
  }
  s = warp_sum(s);
  q = warp_sum(q);
  const float inv_d = 1.0f / static_cast<float>(D);
  float mu = 0.f, rstd;
  if (RMS) {
    rstd = rsqrtf(q * inv_d + eps);
  } else {
    mu = s * inv_d;
    rstd = rsqrtf(fmaxf(q * inv_d - mu * mu, 0.f) + eps);
  }
  const long voff = static_cast<long>(row / rows_per_img) * vec_bstride;
  const float4* sh4 = reinterpret_cast<const float4*>(shift + voff);
  const float4* sc4 = reinterpret_cast<const float4*>(scale + voff);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  uint2* hr = reinterpret_cast<uint2*>(h + static_cast<size_t>(row) * D);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + 32 * i;
    const float4 sh = __ldg(sh4 + c), sc = __ldg(sc4 + c);
    float4 m = make_float4(1.f + sc.x, 1.f + sc.y, 1.f + sc.z, 1.f + sc.w);
    if (RMS) {
      const float4 ww = __ldg(w4 + c);
      m.x *= ww.x;
      m.y *= ww.y;
      m.z *= ww.z;
      m.w *= ww.w;
    }
    const float y0 = fmaf((v[i].x - mu) * rstd, m.x, sh.x), y1 = fmaf((v[i].y - mu) * rstd, m.y, sh.y);
    const float y2 = fmaf((v[i].z - mu) * rstd, m.z, sh.z), y3 = fmaf((v[i].w - mu) * rstd, m.w, sh.w);
    hr[c] = make_uint2(pack_half2(y0, y1), pack_half2(y2, y3));
  }
}

template <bool RMS>
cudaError_t norm_dispatch(const float* x, __half* h, int rows, int D, const float* w, const float* shift,
                          const float* scale, long vec_bstride, int rows_per_img, float eps, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  // a warp per row with the row in registers: from D = 3072 up a thread holds 96+ floats (136 registers
  // at D = 3072), so a 256-thread CTA leaves room for one CTA per SM (8 warps in flight); 2-warp CTAs let
  // the register file hold 14 warps (MOSS RMS-mod, 4608 x 3072: 23.7 us at 3.6 TB/s with 8-warp CTAs)
  const int threads = D >= 3072 ? 64 : 256, rpb = threads / 32;
  const int grid = (rows + rpb - 1) / rpb;
  if (rows_per_img <= 0) rows_per_img = 1 << 30;
  cudaError_t e = cudaSuccess;
#define HX_NORM_CASE(NV)                                                                                   \
  case 128 * NV:                                                                                            \
    e = launch_pdl(norm_mod_kernel<NV, RMS>, dim3(grid), dim3(threads), 0, s, x, h, rows, w, shift, scale, vec_bstride, \
                   rows_per_img, eps);                                                                     \
    break;
  switch (D) {
    HX_NORM_CASE(1) HX_NORM_CASE(2) HX_NORM_CASE(3) HX_NORM_CASE(4) HX_NORM_CASE(6) HX_NORM_CASE(8)
    HX_NORM_CASE(12) HX_NORM_CASE(16) HX_NORM_CASE(24) HX_NORM_CASE(32)
    default: return cudaErrorInvalidValue;
  }
#undef HX_NORM_CASE
  return e != cudaSuccess ? e : cudaGetLastError();
}

// ---------------------------------------------------------------- modulation mat-vecs
// stage 1: hid[site][j] = sum_i A[site][j][i] * silu(emb[i]); one warp per (site, j)
__global__ void mod_stage1(const __half* __restrict__ A, const float* __restrict__ emb, float* __restrict__ hid,
                           int nsite, int D, int R) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= nsite * R) return;
  const __half* row = A + static_cast<size_t>(gw) * D;
  float acc = 0.f;
  for (int i = lane * 8; i < D; i += 256) {
    const uint4 wv = *reinterpret_cast<const uint4*>(row + i);
    const __half2* w2 = reinterpret_cast<const __half2*>(&wv);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 wf = __half22float2(w2[t]);
      const float e0 = emb[i + 2 * t], e1 = emb[i + 2 * t + 1];
      acc = fmaf(wf.x, e0 / (1.f + expf(-e0)), acc);
      acc = fmaf(wf.y, e1 / (1.f + expf(-e1)), acc);
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) hid[gw] = acc;
}
// stage 2: out[site][o] = lora[o] + sum_j B[site][o][j] * hid[site][j]; one warp per (site, o)
__global__ void mod_stage2(const __half* __restrict__ Bw, const float* __restrict__ hid, const float* __restrict__ lora,
                           float* __restrict__ out, int nsite, int R, int O) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= nsite * O) return;
  const int site = gw / O, o = gw % O;
  const __half* row = Bw + static_cast<size_t>(gw) * R;
  const float* hs = hid + static_cast<size_t>(site) * R;
  float acc = 0.f;
  for (int j = lane * 8; j < R; j += 256) {
    const uint4 wv = *reinterpret_cast<const uint4*>(row + j);
    const __half2* w2 = reinterpret_cast<const __half2*>(&wv);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 wf = __half22float2(w2[t]);
      acc = fmaf(wf.x, hs[j + 2 * t], acc);
      acc = fmaf(wf.y, hs[j + 2 * t + 1], acc);
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) out[gw] = acc + (lora ? lora[o] : 0.f);
}

// The same two stages for every block of a chain at once (blockIdx.y = block), weights from per-block
// pointer tables, silu(emb) computed once (silu_kernel) instead of in every warp; out for block b at
// out + b * out_stride: [nsite][O] outputs, then [nsite][R] hidden.
__global__ void silu_kernel(const float* __restrict__ e, float* __restrict__ y, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = e[i] / (1.f + expf(-e[i]));
}
__global__ void mod_batch_stage1(const __half* const* __restrict__ Atab, const float* __restrict__ se,
                                 float* __restrict__ out, size_t out_stride, int nsite, int D, int R, int O) {
  const int lane = threadIdx.x & 31, b = blockIdx.y;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= nsite * R) return;
  const __half* row = Atab[b] + static_cast<size_t>(gw) * D;
  float acc = 0.f;
  for (int i = lane * 8; i < D; i += 256) {
    const uint4 wv = *reinterpret_cast<const uint4*>(row + i);
    const __half2* w2 = reinterpret_cast<const __half2*>(&wv);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 wf = __half22float2(w2[t]);
      acc = fmaf(wf.x, se[i + 2 * t], acc);
      acc = fmaf(wf.y, se[i + 2 * t + 1], acc);
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) out[b * out_stride + static_cast<size_t>(nsite) * O + gw] = acc;
}
__global__ void mod_batch_stage2(const __half* const* __restrict__ Btab, const float* __restrict__ lora,
                                 float* __restrict__ out, size_t out_stride, int nsite, int R, int O) {
  const int lane = threadIdx.x & 31, b = blockIdx.y;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= nsite * O) return;
  const int site = gw / O, o = gw % O;
  float* ob = out + b * out_stride;
  const __half* row = Btab[b] + static_cast<size_t>(gw) * R;
  const float* hs = ob + static_cast<size_t>(nsite) * O + static_cast<size_t>(site) * R;
  float acc = 0.f;
  for (int j = lane * 8; j < R; j += 256) {
    const uint4 wv = *reinterpret_cast<const uint4*>(row + j);
    const __half2* w2 = reinterpret_cast<const __half2*>(&wv);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 wf = __half22float2(w2[t]);
      acc = fmaf(wf.x, hs[j + 2 * t], acc);
      acc = fmaf(wf.y, hs[j + 2 * t + 1], acc);
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) ob[gw] = acc + (lora ? lora[o] : 0.f);
}

__global__ void f32_to_f16_kernel(const float* __restrict__ s, __half* __restrict__ d, size_t n) {
  const size_t i = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (i + 3 < n) {
    const float4 v = *reinterpret_cast<const float4*>(s + i);
    *reinterpret_cast<uint2*>(d + i) = make_uint2(pack_half2(v.x, v.y), pack_half2(v.z, v.w));
  } else {
    for (size_t k = i; k < n; ++k) d[k] = __float2half_rn(s[k]);
  }
}

// Self-test of the bounded wait (the runtime's analogue of the reference's HMX self-test, which returns
// rc -77 when its check fails, moss/hexagon/mega/blk.c:112-118,149-155): thread 0 waits on a shared
// mbarrier of arrival count 1 with a run-time limit; thread 32 arrives on it only when `arrive` is set.
// Nothing else is in flight, so an expired wait leaves no copy or MMA behind.
__global__ void wait_selftest_kernel(int* status, unsigned long long limit_ns, int arrive) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (arrive && threadIdx.x == 32) mbar_arrive(&bar);
  if (threadIdx.x == 0) mbar_wait_limit(&bar, 0, status, 901, limit_ns);
}

}  // namespace

cudaError_t wait_selftest_launch(int* status, unsigned long long limit_ns, int arrive, cudaStream_t s) {
  wait_selftest_kernel<<<1, 64, 0, s>>>(status, limit_ns, arrive);
  return cudaGetLastError();
}

cudaError_t lnmod_launch(const float* x, __half* h, int rows, int D, const float* shift, const float* scale,
                         long vec_bstride, int rows_per_img, float eps, cudaStream_t s) {
  return norm_dispatch<false>(x, h, rows, D, nullptr, shift, scale, vec_bstride, rows_per_img, eps, s);
}

cudaError_t rmsmod_launch(const float* x, __half* h, int rows, int D, const float* w, const float* shift,
                          const float* scale, long vec_bstride, int rows_per_img, float eps, cudaStream_t s) {
  if (!w) return cudaErrorInvalidValue;
  return norm_dispatch<true>(x, h, rows, D, w, shift, scale, vec_bstride, rows_per_img, eps, s);
}

// every block of a chain: Atab / Btab device tables of nblk weight pointers, se a device scratch of D floats
cudaError_t modulation_batch_launch(const __half* const* Atab, const __half* const* Btab, int nblk, const float* emb,
                                    const float* lora, float* out, size_t out_stride, float* se, int nsite, int D,
                                    int R, int O, cudaStream_t s) {
  if (D % 256 || R % 256 || nblk < 1 || nblk > 65535 || out_stride < static_cast<size_t>(nsite) * (O + R))
    return cudaErrorInvalidValue;
  const int t = 256, wpb = t / 32;
  silu_kernel<<<(D + 255) / 256, 256, 0, s>>>(emb, se, D);
  mod_batch_stage1<<<dim3((nsite * R + wpb - 1) / wpb, nblk), t, 0, s>>>(Atab, se, out, out_stride, nsite, D, R, O);
  mod_batch_stage2<<<dim3((nsite * O + wpb - 1) / wpb, nblk), t, 0, s>>>(Btab, lora, out, out_stride, nsite, R, O);
  return cudaGetLastError();
}

// hid scratch lives right after the nsite*O outputs: out must hold nsite*(O+R) floats
cudaError_t modulation_launch(const __half* Aw, const __half* Bw, const float* emb, const float* lora, float* out,
                              int nsite, int D, int R, int O, cudaStream_t s) {
  if (D % 256 || R % 256) return cudaErrorInvalidValue;
  float* hid = out + static_cast<size_t>(nsite) * O;
  const int t = 256, wpb = t / 32;
  mod_stage1<<<(nsite * R + wpb - 1) / wpb, t, 0, s>>>(Aw, emb, hid, nsite, D, R);
  mod_stage2<<<(nsite * O + wpb - 1) / wpb, t, 0, s>>>(Bw, hid, lora, out, nsite, R, O);
  return cudaGetLastError();
}

cudaError_t f32_to_f16_launch(const float* src, __half* dst, size_t n, cudaStream_t s) {
  if (!n) return cudaSuccess;
  const size_t threads = 256, per = threads * 4;
  f32_to_f16_kernel<<<static_cast<unsigned>((n + per - 1) / per), threads, 0, s>>>(src, dst, n);
  return cudaGetLastError();
}

}  // namespace hx

// ---------------------------------------------------------------- allocation-free modulation
// Scratch of hx_modulation_noalloc: the per-site 256-wide hidden vectors (stage 1 output, stage 2
// input). Fixed at 4096 floats; every GPU that loads the library holds it until the process exits.
#define HX_NOALLOC_MOD_HID_FLOATS 4096
static __device__ __align__(256) float g_noalloc_mod_hid[HX_NOALLOC_MOD_HID_FLOATS];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_hid_ptr[64];  // device address of g_noalloc_mod_hid per device, looked up once
}  // namespace

extern "C" HX_API int hx_modulation_noalloc(const void* modA, const void* modB, const float* emb_dev,
                                            const float* lora_dev, float* mod_dev, int nsite, int D, void* stream) {
  if (!modA || !modB || !emb_dev || !mod_dev || nsite <= 0 || D <= 0 || D % 256) return HX_E_ARG;
  // the stage kernels read modA / modB rows 16 bytes at a time
  if ((reinterpret_cast<uintptr_t>(modA) | reinterpret_cast<uintptr_t>(modB)) & 15) return HX_E_ARG;
  if (static_cast<long>(nsite) * 256 > HX_NOALLOC_MOD_HID_FLOATS) return HX_E_SCRATCH;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return HX_E_CUDA;
  void* hid = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_hid_ptr[dev]) {
      // In host code g_noalloc_mod_hid only stands for the symbol: its device address comes from here.
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_noalloc_mod_hid) != cudaSuccess || !p) return HX_E_CUDA;
      g_noalloc_hid_ptr[dev] = p;
    }
    hid = g_noalloc_hid_ptr[dev];
  }
  // Stage 1 writes every hid element stage 2 reads, so nothing needs clearing between calls.
  // cudaLaunchKernel reports the error of its own launch, not one left queued by an earlier call.
  int R = 256, O = 3 * D;
  const int t = 256, wpb = t / 32;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const __half* A = static_cast<const __half*>(modA);
  const __half* Bw = static_cast<const __half*>(modB);
  float* hidf = static_cast<float*>(hid);
  const float* hidc = hidf;
  void* a1[] = {&A, &emb_dev, &hidf, &nsite, &D, &R};
  if (cudaLaunchKernel(reinterpret_cast<const void*>(&hx::mod_stage1), dim3((nsite * R + wpb - 1) / wpb), dim3(t), a1,
                       0, s) != cudaSuccess)
    return HX_E_CUDA;
  void* a2[] = {&Bw, &hidc, &lora_dev, &mod_dev, &nsite, &R, &O};
  if (cudaLaunchKernel(reinterpret_cast<const void*>(&hx::mod_stage2), dim3((nsite * O + wpb - 1) / wpb), dim3(t), a2,
                       0, s) != cudaSuccess)
    return HX_E_CUDA;
  return HX_OK;
}

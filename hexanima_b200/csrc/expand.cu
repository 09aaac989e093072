// Weight expansion: a quantised matrix dequantised to fp16 W[N][K] in a scratch buffer just before
// its GEMM, so that the GEMM streams fp16 weights by TMA instead of dequantising in its main loop.
//
// The reference dequantises every weight tile on each use as well, on the DSP while the tile is copied
// from DDR into VTCM (hexagon/mega/gemm2.c:20-35 `dq_tile`, moss/hexagon/mega/gemm2.c:39-56 `dq4_tile`);
// here the copy goes to HBM / L2 instead of VTCM and runs as its own memory-bound pass. One matrix
// expands to 2 bytes per weight (the largest Anima matrix, mlp.layer1, to 33.5 MB: it stays in the
// 126 MB L2 for the GEMM that follows). The values are bit-identical to the in-kernel dequantisers of
// gemm.cu (the same operations in the same order), so the GEMM's result does not depend on the path.
#include <algorithm>

#include <cuda_fp16.h>

#include "hx_internal.h"
#include "hx_ptx.cuh"

namespace hx {

namespace {

// Work unit: 8 consecutive k of one row (8 bytes of q8 or 4 of q4 in, one 16-byte fp16 store out). Unit i
// covers elements 8i .. 8i + 7 of the row-major matrix, so a warp's 32 units read 256 (q8) or 128 (q4)
// contiguous bytes and write 512; each thread keeps UNROLL units' loads in flight before converting.
constexpr int EXP_THREADS = 256, UNROLL = 4;

__device__ __forceinline__ uint4 q8x8(uint2 v, __half s) {
  // bytes as fp16 0x64uu = 1024 + u exactly; minus 1152 = q exactly; one rounded multiply by s
  const __half2 off = __half2half2(__ushort_as_half(0x6480));  // 1152.0
  const __half2 s2 = __half2half2(s);
  const uint32_t wd[2] = {v.x, v.y};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    uint32_t lo = __byte_perm(wd[j], 0x64646464u, 0x4140);
    uint32_t hi = __byte_perm(wd[j], 0x64646464u, 0x4342);
    __half2 a = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&lo), off), s2);
    __half2 b = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&hi), off), s2);
    o[2 * j] = *reinterpret_cast<uint32_t*>(&a);
    o[2 * j + 1] = *reinterpret_cast<uint32_t*>(&b);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// q4 word: 8 consecutive k, k at nibble (k & 7) / 2 + 4 (k & 1): nibbles t and t + 4 are k = 2t, 2t + 1
__device__ __forceinline__ uint4 q4x8(uint32_t wd, __half s) {  // fp16((nib - 8) * s)
  const __half2 off = __half2half2(__ushort_as_half(0x6408));  // 1032.0: 1024 + nib exact, minus 1032 exact
  const __half2 s2 = __half2half2(s);
  uint32_t o[4];
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    uint32_t e = ((wd >> (4 * t)) & 0x000F000Fu) | 0x64006400u;
    __half2 a = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&e), off), s2);
    o[t] = *reinterpret_cast<uint32_t*>(&a);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ uint4 q4ax8(uint32_t wd, __half s, __half m) {  // fp16(fp32(nib * s) + m)
  const float sf = __half2float(s), mf = __half2float(m);
  uint32_t o[4];
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const uint32_t e = (wd >> (4 * t)) & 0x000F000Fu;
    const float n0 = static_cast<float>(e & 0xF), n1 = static_cast<float>(e >> 16);
    o[t] = pack_half2(__fadd_rn(__fmul_rn(n0, sf), mf), __fadd_rn(__fmul_rn(n1, sf), mf));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// FMT: WF_Q8, WF_Q4 or WF_Q4A. units = N K / 8 < 2^32; upr = K / 8 units per row.
template <int FMT>
__global__ void __launch_bounds__(EXP_THREADS) expand_kernel(const uint8_t* __restrict__ u, const __half* __restrict__ sc,
                                                             const __half* __restrict__ mn, uint32_t N, uint32_t upr,
                                                             uint32_t units, uint32_t gshift, uint4* __restrict__ w) {
  grid_dep_wait();  // the previous user of the scratch (the GEMM before) has finished reading it
  grid_dep_launch();
  const uint32_t stride = gridDim.x * EXP_THREADS * UNROLL;
  for (uint32_t base = blockIdx.x * EXP_THREADS * UNROLL + threadIdx.x; base < units; base += stride) {
    uint2 v8[UNROLL];
    uint32_t v4[UNROLL];
    __half s[UNROLL], m[UNROLL];
#pragma unroll
    for (int r = 0; r < UNROLL; ++r) {
      const uint32_t i = base + r * EXP_THREADS;
      if (i < units) {
        const uint32_t n = i / upr, k0 = (i - n * upr) * 8;
        const size_t g = static_cast<size_t>(k0 >> gshift) * N + n;  // scale [K / group][N]
        if constexpr (FMT == WF_Q8) v8[r] = __ldg(reinterpret_cast<const uint2*>(u) + i);
        else v4[r] = __ldg(reinterpret_cast<const uint32_t*>(u) + i);
        s[r] = __ldg(sc + g);
        if constexpr (FMT == WF_Q4A) m[r] = __ldg(mn + g);
      }
    }
#pragma unroll
    for (int r = 0; r < UNROLL; ++r) {
      const uint32_t i = base + r * EXP_THREADS;
      if (i < units) {
        if constexpr (FMT == WF_Q8) w[i] = q8x8(v8[r], s[r]);
        else if constexpr (FMT == WF_Q4) w[i] = q4x8(v4[r], s[r]);
        else w[i] = q4ax8(v4[r], s[r], m[r]);
      }
    }
  }
}

}  // namespace

cudaError_t expand_launch(const DevMat& W, __half* dst, cudaStream_t s) {
  if (!W.w || !dst || W.N <= 0 || W.K <= 0 || W.K % 32) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(W.w) % 16 || reinterpret_cast<uintptr_t>(dst) % 16) return cudaErrorInvalidValue;
  const size_t units = static_cast<size_t>(W.N) * (W.K / 8);
  if (units >= (1ull << 32)) return cudaErrorInvalidValue;
  if (!W.scale || (W.fmt == WF_Q4A && !W.minv)) return cudaErrorInvalidValue;
  if (W.fmt == WF_Q8 ? (W.group != 32 && W.group != 64) : W.group != 32) return cudaErrorInvalidValue;
  const uint32_t gshift = W.group == 64 ? 6 : 5;
  const size_t per_block = static_cast<size_t>(EXP_THREADS) * UNROLL;
  const int grid = static_cast<int>(std::min<size_t>((units + per_block - 1) / per_block, static_cast<size_t>(sm_count()) * 8));
  const auto* u = static_cast<const uint8_t*>(W.w);
  auto* out = reinterpret_cast<uint4*>(dst);
  const uint32_t N = W.N, upr = W.K / 8, nu = static_cast<uint32_t>(units);
  const __half* no_min = nullptr;
  cudaError_t e = cudaSuccess;
  switch (W.fmt) {
    case WF_Q8:
      e = launch_pdl(expand_kernel<WF_Q8>, dim3(grid), dim3(EXP_THREADS), 0, s, u, W.scale, no_min, N, upr, nu, gshift, out);
      break;
    case WF_Q4:
      e = launch_pdl(expand_kernel<WF_Q4>, dim3(grid), dim3(EXP_THREADS), 0, s, u, W.scale, no_min, N, upr, nu, gshift, out);
      break;
    case WF_Q4A:
      e = launch_pdl(expand_kernel<WF_Q4A>, dim3(grid), dim3(EXP_THREADS), 0, s, u, W.scale, W.minv, N, upr, nu, gshift, out);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace hx

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

// Work unit: 8 consecutive k of one row (8 bytes of q8 or 4 of q4 in, one 16-byte fp16 store out). The grid
// is 2D: x runs over the units of a row (a warp's 32 units read 256 or 128 contiguous bytes and write 512),
// y over groups of EXP_ROWS rows, whose loads each thread issues before converting. No division: a
// thread's k and scale group are fixed, and the scales of consecutive rows are adjacent.
constexpr int EXP_THREADS = 256, EXP_ROWS = 4;

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

// FMT: WF_Q8, WF_Q4 or WF_Q4A; upr = K / 8 units per row; scale group = 1 << gshift
template <int FMT>
__global__ void __launch_bounds__(EXP_THREADS) expand_kernel(const uint8_t* __restrict__ u, const __half* __restrict__ sc,
                                                             const __half* __restrict__ mn, int N, int upr, int gshift,
                                                             uint4* __restrict__ w) {
  grid_dep_wait();  // the previous user of the scratch (the GEMM before) has finished reading it
  grid_dep_launch();
  const int j = blockIdx.x * EXP_THREADS + threadIdx.x;  // unit within the row: k = 8 j .. 8 j + 7
  if (j >= upr) return;
  const size_t goff = static_cast<size_t>((8 * j) >> gshift) * N;  // this thread's scale row
  for (int n0 = blockIdx.y * EXP_ROWS; n0 < N; n0 += gridDim.y * EXP_ROWS) {
    uint2 v8[EXP_ROWS];
    uint32_t v4[EXP_ROWS];
    __half s[EXP_ROWS], m[EXP_ROWS];
#pragma unroll
    for (int r = 0; r < EXP_ROWS; ++r) {
      const int n = n0 + r;
      if (n < N) {
        const size_t i = static_cast<size_t>(n) * upr + j;
        if constexpr (FMT == WF_Q8) v8[r] = __ldg(reinterpret_cast<const uint2*>(u) + i);
        else v4[r] = __ldg(reinterpret_cast<const uint32_t*>(u) + i);
        s[r] = __ldg(sc + goff + n);
        if constexpr (FMT == WF_Q4A) m[r] = __ldg(mn + goff + n);
      }
    }
#pragma unroll
    for (int r = 0; r < EXP_ROWS; ++r) {
      const int n = n0 + r;
      if (n < N) {
        const size_t i = static_cast<size_t>(n) * upr + j;
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
  if (!W.scale || (W.fmt == WF_Q4A && !W.minv)) return cudaErrorInvalidValue;
  if (W.fmt == WF_Q8 ? (W.group != 32 && W.group != 64) : W.group != 32) return cudaErrorInvalidValue;
  const int gshift = W.group == 64 ? 6 : 5;
  const int upr = W.K / 8;
  const int gx = (upr + EXP_THREADS - 1) / EXP_THREADS;
  const int row_groups = (W.N + EXP_ROWS - 1) / EXP_ROWS;
  const int gy = std::max(1, std::min(row_groups, sm_count() * 8 / gx));
  const dim3 grid(gx, gy);
  const auto* u = static_cast<const uint8_t*>(W.w);
  auto* out = reinterpret_cast<uint4*>(dst);
  const __half* no_min = nullptr;
  cudaError_t e = cudaSuccess;
  switch (W.fmt) {
    case WF_Q8:
      e = launch_pdl(expand_kernel<WF_Q8>, grid, dim3(EXP_THREADS), 0, s, u, W.scale, no_min, W.N, upr, gshift, out);
      break;
    case WF_Q4:
      e = launch_pdl(expand_kernel<WF_Q4>, grid, dim3(EXP_THREADS), 0, s, u, W.scale, no_min, W.N, upr, gshift, out);
      break;
    case WF_Q4A:
      e = launch_pdl(expand_kernel<WF_Q4A>, grid, dim3(EXP_THREADS), 0, s, u, W.scale, W.minv, W.N, upr, gshift, out);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace hx

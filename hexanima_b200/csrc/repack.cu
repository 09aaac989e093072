// Reference pack records -> device weight layouts (one-time, at load).
//
// Pack tiles are 32x32 "crouton" tiles of W[K][N] (hexagon/mega/export_all.py:7-8): halfword
// (k, n) of a tile sits at ((k%32)/2)*64 + (n%32)*2 + (k&1); tiles are ordered [n block][k block].
//  fp16 record : 2048 B, the halfwords above.
//  q8 record   : 1152 B = 128 B scale vector (halfword 2c = fp16 scale of column c) + 1024 B of
//                offset-binary bytes u = q + 128 at the same index (export_all_q8.py:10-18,
//                read back by mkblk_test.py:23-27).
// Device layouts: fp16 W[N][K]; q8 u8 W[N][K] (offset binary kept) + fp16 scale[K/32][N].
// row_perm selects which pack column feeds device row r:
//  0 identity
//  1 SiTU interleave: the MOSS up_gate pack alternates 32-column blocks (up_j, gate_j)
//    (export_moss.py:17-19); device rows are grouped per 256: [0,128) up and [128,256) gate of the
//    same 128 outputs, so one 128x256 GEMM tile holds both halves of its outputs.
#include "hx_internal.h"

namespace hx {

namespace {

__device__ __forceinline__ int src_col(int r, int mode) {
  if (mode == 1) {
    const int t = r / 256, l = r % 256;
    const int o = t * 128 + (l & 127);
    return 64 * (o / 32) + (l >= 128 ? 32 : 0) + (o % 32);
  }
  return r;
}

// dst / scale address the fused device matrix; this pack matrix lands at rows [row0, row0 + 32 nb)
// of a matrix with nrows_total rows (the scale row stride).
template <bool Q8>
__global__ void repack_kernel(const uint8_t* __restrict__ rec, int nb, int kb, void* __restrict__ dst,
                              __half* __restrict__ scale, int row0, int nrows_total, int mode) {
  const int K = kb * 32, N = nb * 32;
  const long total = static_cast<long>(N) * (K / 8);
  const long idx = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int r = static_cast<int>(idx / (K / 8)), k0 = static_cast<int>(idx % (K / 8)) * 8;
  const int n = src_col(r, mode);
  const long tile = static_cast<long>(n / 32) * kb + k0 / 32;
  if (Q8) {
    const uint8_t* t = rec + tile * 1152;
    uint8_t v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int k = k0 + e;
      v[e] = t[128 + ((k % 32) / 2) * 64 + (n % 32) * 2 + (k & 1)];
    }
    uint8_t* d = static_cast<uint8_t*>(dst) + static_cast<size_t>(row0 + r) * K + k0;
    *reinterpret_cast<uint2*>(d) = *reinterpret_cast<const uint2*>(v);
    if (k0 % 32 == 0) {
      unsigned short s = static_cast<unsigned short>(t[(n % 32) * 4]) |
                         static_cast<unsigned short>(t[(n % 32) * 4 + 1] << 8);
      scale[static_cast<size_t>(k0 / 32) * nrows_total + row0 + r] = __ushort_as_half(s);
    }
  } else {
    const unsigned short* t = reinterpret_cast<const unsigned short*>(rec + tile * 2048);
    unsigned short v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int k = k0 + e;
      v[e] = t[((k % 32) / 2) * 64 + (n % 32) * 2 + (k & 1)];
    }
    unsigned short* d = static_cast<unsigned short*>(dst) + static_cast<size_t>(row0 + r) * K + k0;
    *reinterpret_cast<uint4*>(d) = *reinterpret_cast<const uint4*>(v);
  }
}

}  // namespace

cudaError_t repack_tiles_launch(const uint8_t* rec, int nb, int kb, bool q8, void* dst, __half* scale, int row0,
                                int nrows_total, int mode, cudaStream_t s) {
  const long total = static_cast<long>(nb) * 32 * (kb * 32 / 8);
  const int threads = 256;
  const unsigned grid = static_cast<unsigned>((total + threads - 1) / threads);
  if (q8) repack_kernel<true><<<grid, threads, 0, s>>>(rec, nb, kb, dst, scale, row0, nrows_total, mode);
  else repack_kernel<false><<<grid, threads, 0, s>>>(rec, nb, kb, dst, scale, row0, nrows_total, mode);
  return cudaGetLastError();
}

}  // namespace hx

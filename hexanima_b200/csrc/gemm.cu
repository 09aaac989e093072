// Weight-only-quantised GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), fed by TMA.
//
// Replaces the reference GEMM engine gemm_run_geo (hexagon/mega/gemm2.c:96-137,
// moss/hexagon/mega/gemm2.c:145-193): O[M x N] = A[M x K] * W^T with W stored [N][K], weights
// dequantised while they stream in (dq_tile gemm2.c:20-35, dq4_tile moss gemm2.c:39-56), the
// LoRA "extra K tiles" of geo.A2 (moss gemm2.h:16) as a second A source, and the flush
// epilogues of job_fn (gemm2.c:58-82, moss gemm2.c:89-123) fused into the TMEM read-out.
//
// Device weight layouts (chosen for this kernel, converted from the pack records at load time):
//   WF_F16 : fp16 W[N][K]
//   WF_Q8  : u8   W[N][K], offset binary u = q + 128; fp16 scale[K/g][N]; value = fp16(q * s)
//   WF_Q4  : u8   W[N][K/2]; every 32-bit word holds 8 consecutive k, k at nibble (k>>1) + 4(k&1);
//            fp16 scale[K/32][N]; value = fp16((nib - 8) * s)
//   WF_Q4A : as WF_Q4 plus fp16 min[K/32][N]; value = fp16(fp32(nib * s) + m)   (export_te.py:33-40)
//
// CTA = 14 warps, one CTA per SM, persistent over 128x256 output tiles:
//   warps 0-3  epilogue (TMEM lanes 0-127 = tile rows)
//   warp  4    TMA producer (A tile, raw weight tile, scales)
//   warp  5    TMEM allocator + single-thread tcgen05.mma issuer
//   warps 6-13 dequantisers: raw int8/int4 -> fp16 in the 128B-swizzled K-major operand layout
// TMEM holds two 128x256 fp32 accumulators so the epilogue of tile i overlaps the mainloop of
// tile i+1.
#include <cudaTypedefs.h>
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "hx_internal.h"
#include "hx_gelu.cuh"
#include "hx_ptx.cuh"

namespace hx {

namespace {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int EPI_WARPS = 4, TMA_WARP = 4, MMA_WARP = 5, DQ_WARP0 = 6, DQ_WARPS = 8;
constexpr int GEMM_THREADS = (DQ_WARP0 + DQ_WARPS) * 32;
constexpr int A_BYTES = BM * BK * 2;      // 16 KB
constexpr int WDQ_BYTES = BN * BK * 2;    // 32 KB
constexpr int SC_BYTES = 2048;            // scales (and q4a mins) of one k-block

template <int FMT>
struct Cfg {
  static constexpr int RAW_BYTES = FMT == WF_F16 ? 0 : FMT == WF_Q8 ? BN * BK : BN * BK / 2;
  static constexpr int STAGE_BYTES = A_BYTES + WDQ_BYTES + RAW_BYTES + (FMT == WF_F16 ? 0 : SC_BYTES);
  static constexpr int STAGES = FMT == WF_F16 ? 4 : 3;
  static constexpr int OUT_STAGE = 16384;  // residual epilogue: 128 rows x 32 fp32, 128B-swizzled
  static constexpr int SMEM = STAGES * STAGE_BYTES + OUT_STAGE + 1024 /*barriers*/ + 1024 /*alignment slack*/;
};

struct KParams {
  int M, N, nkb, nkb1, group;
  int num_m_tiles, num_tiles;
  int num_n_tiles, n_fastest;  // tile order: n_fastest walks the N tiles of one M block consecutively
  int group_m;                 // otherwise, > 0: bands of group_m M tiles walk all N tiles, M fastest in a band
  int streamk;                 // CTA-pair kernel, residual epilogue: stream-K schedule (Sched)
  __half* out;
  int ldo;
  float* x;
  int ldx;
  const float* gate;
  long vec_bstride;
  int rows_per_img;
  const float* gain0;
  const float* gain1;
  int seg1, seg2, rope0, rope1;
  const float* cosT;
  const float* sinT;
  float eps;
  int* status;
};

// tile t -> (M tile, N tile) in the launch's order. Banded order (group_m > 0): band b holds M tiles
// [b*group_m, b*group_m + gm) (gm smaller in the last band) and walks them for N tile 0, then 1, ...; the
// A rows of one band stay in L2 across all N tiles and each weight block is reused by the band's gm
// tiles at once, so neither operand of a large GEMM is re-read from HBM while the output streams out.
__device__ __forceinline__ int tile_m(const KParams& p, int t) {
  if (p.n_fastest) return t / p.num_n_tiles;
  if (p.group_m > 0) {
    const int per = p.group_m * p.num_n_tiles, b = t / per, r = t - b * per;
    const int gm = min(p.group_m, p.num_m_tiles - b * p.group_m);
    return b * p.group_m + r % gm;
  }
  return t % p.num_m_tiles;
}
__device__ __forceinline__ int tile_n(const KParams& p, int t) {
  if (p.n_fastest) return t % p.num_n_tiles;
  if (p.group_m > 0) {
    const int per = p.group_m * p.num_n_tiles, b = t / per, r = t - b * per;
    const int gm = min(p.group_m, p.num_m_tiles - b * p.group_m);
    return r / gm;
  }
  return t / p.num_m_tiles;
}

// The work units of CTA pair `pair` in order. Tile schedule: tiles pair, pair + npairs, ..., each over
// all k-blocks. Stream-K (residual epilogue): the whole waves of tiles keep that order (which keeps the
// operand blocks the concurrent pairs share in L2); the tiles of the last, partial wave are cut into an
// equal share of (tile, k-block) iterations per pair, taken tile after tile; a tile cut between two pairs
// gets two partial sums, each reduce-added into x. Every role of the pair walks the same units.
struct Sched {
  int nkb, t, step, full, it, it1;
  __device__ __forceinline__ Sched(const KParams& p, int pair, int npairs)
      : nkb(p.nkb), t(pair), step(npairs), full(p.num_tiles), it(0), it1(0) {
    if (p.streamk) {
      full = p.num_tiles / npairs * npairs;
      const long long rem = static_cast<long long>(p.num_tiles - full) * p.nkb, base = static_cast<long long>(full) * p.nkb;
      it = static_cast<int>(base + rem * pair / npairs);
      it1 = static_cast<int>(base + rem * (pair + 1) / npairs);
    }
  }
  __device__ __forceinline__ bool next(const KParams& p, int& tile, int& kb0, int& kb1) {
    (void)p;
    if (t < full) {
      tile = t;
      kb0 = 0;
      kb1 = nkb;
      t += step;
      return true;
    }
    if (it >= it1) return false;
    tile = it / nkb;
    kb0 = it % nkb;
    kb1 = min(nkb, kb0 + (it1 - it));
    it += kb1 - kb0;
    return true;
  }
};

// ---------------------------------------------------------------- dequantisers
// One k-block (64 k) of a 256-row weight tile: raw smem -> fp16 SW128 K-major smem.
// ROWS weight rows per k-block (256 for the 1-CTA tile, 128 or 112 per CTA of a pair); 256 dequant threads.
// A last, partial pass (ROWS = 112) is skipped by whole warps (8 rows per warp for q8, 16 for q4).
template <int FMT, int ROWS = BN>
__device__ __forceinline__ void dequant_kblock(uint32_t raw, uint32_t dq, const __half* sc, int group, int dt) {
  if constexpr (FMT == WF_Q8) {
    const int c = dt & 3, r0 = dt >> 2;
    const __half2 off = __half2half2(__ushort_as_half(0x6480));  // 1152.0
#pragma unroll
    for (int pass = 0; pass < (ROWS + 63) / 64; ++pass) {
      const int n = pass * 64 + r0;
      if (ROWS % 64 != 0 && n >= ROWS) break;
      const uint4 v = ld_shared_v4(raw + n * 64 + c * 16);
      const __half s = group == 64 ? sc[n] : sc[(c >> 1) * ROWS + n];
      const __half2 s2 = __half2half2(s);
      uint32_t o[8];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t lo = __byte_perm(w[j], 0x64646464u, 0x4140);
        uint32_t hi = __byte_perm(w[j], 0x64646464u, 0x4342);
        __half2 a = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&lo), off), s2);
        __half2 b = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&hi), off), s2);
        o[2 * j] = *reinterpret_cast<uint32_t*>(&a);
        o[2 * j + 1] = *reinterpret_cast<uint32_t*>(&b);
      }
      const uint32_t rowb = dq + n * 128, sw = n & 7;
      st_shared_v4(rowb + (((2 * c) ^ sw) << 4), o[0], o[1], o[2], o[3]);
      st_shared_v4(rowb + (((2 * c + 1) ^ sw) << 4), o[4], o[5], o[6], o[7]);
    }
  } else {
    // q4 / q4a: 32 raw bytes per row, two threads per row, each thread one 32-k group
    const int c = dt & 1, r0 = dt >> 1;
#pragma unroll
    for (int pass = 0; pass < (ROWS + 127) / 128; ++pass) {
      const int n = pass * 128 + r0;
      if (ROWS % 128 != 0 && n >= ROWS) break;
      const uint4 v = ld_shared_v4(raw + n * 32 + c * 16);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      const __half s = sc[c * ROWS + n];
      const uint32_t rowb = dq + n * 128, sw = n & 7;
      if constexpr (FMT == WF_Q4) {
        const __half2 off = __half2half2(__ushort_as_half(0x6408));  // 1032.0
        const __half2 s2 = __half2half2(s);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t o[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            uint32_t e = ((w[j] >> (4 * t)) & 0x000F000Fu) | 0x64006400u;
            __half2 a = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&e), off), s2);
            o[t] = *reinterpret_cast<uint32_t*>(&a);
          }
          st_shared_v4(rowb + (((4 * c + j) ^ sw) << 4), o[0], o[1], o[2], o[3]);
        }
      } else {
        const float sf = __half2float(s);
        const float mf = __half2float(sc[2 * ROWS + c * ROWS + n]);  // mins follow the two scale rows
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t o[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const uint32_t e = (w[j] >> (4 * t)) & 0x000F000Fu;
            const float n0 = static_cast<float>(e & 0xF), n1 = static_cast<float>(e >> 16);
            const float v0 = __fadd_rn(__fmul_rn(n0, sf), mf), v1 = __fadd_rn(__fmul_rn(n1, sf), mf);
            o[t] = pack_half2(v0, v1);
          }
          st_shared_v4(rowb + (((4 * c + j) ^ sw) << 4), o[0], o[1], o[2], o[3]);
        }
      }
    }
  }
}

// ---------------------------------------------------------------- epilogue helpers
__device__ __forceinline__ void store_row32_f16(__half* dst, const float* v) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q)
    d[q] = make_uint4(pack_half2(v[8 * q], v[8 * q + 1]), pack_half2(v[8 * q + 2], v[8 * q + 3]),
                      pack_half2(v[8 * q + 4], v[8 * q + 5]), pack_half2(v[8 * q + 6], v[8 * q + 7]));
}

__device__ __forceinline__ float situ(float h, float g) {
  return (4.0f * tanhf(g * 0.25f) * (1.0f / (1.0f + expf(-g)))) * (25.0f * tanhf(h * 0.04f));
}

// TN: the tile's accumulator columns (256, or 224 for the CTA-pair GELU / store tiles that fill the
// waves of an N = 8192 GEMM better)
template <int EPI, int TN = BN>
__device__ __forceinline__ void epilogue_tile(const KParams& p, uint32_t tacc, int m0, int n0, int warp, int lane,
                                              const CUtensorMap* tmX, uint8_t* stage_ptr) {
  static_assert(TN == BN || ((EPI == EPI_GELU || EPI == EPI_STORE) && TN % 32 == 0), "tile width");
  const int m = m0 + warp * 32 + lane;
  const bool row_ok = m < p.M;
  const uint32_t tl = tacc + (static_cast<uint32_t>(warp * 32) << 16);
  const int img = row_ok ? m / p.rows_per_img : 0;
  const uint32_t stage = smem_u32(stage_ptr);
  (void)stage;
  (void)tmX;
  uint32_t r[32];
  float v[32];
  if constexpr (EPI == EPI_STORE32) {
#pragma unroll 1
    for (int c = 0; c < TN / 32; ++c) {
      const int n = n0 + 32 * c;
      if (n >= p.N) break;
      tmem_ld32(tl + 32 * c, r);
      tmem_ld_wait();
      if (!row_ok) continue;
      float4* xr = reinterpret_cast<float4*>(p.x + static_cast<size_t>(m) * p.ldx + n);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        xr[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]), __uint_as_float(r[4 * q + 2]),
                            __uint_as_float(r[4 * q + 3]));
    }
  } else if constexpr (EPI == EPI_STORE || EPI == EPI_GELU) {
    // fp16 out: 64 columns at a time staged in the 128-B swizzled stage, written by one TMA store
    // (the tensor map clips rows >= M and columns >= N); a last 32 columns (TN = 224) by plain row stores,
    // since a 64-column box would overwrite the next tile's first columns
    const int row = warp * 32 + lane;
#pragma unroll 1
    for (int g = 0; g < (TN + 63) / 64; ++g) {
      if (n0 + 64 * g >= p.N) break;  // uniform over the epilogue warps
      if (TN % 64 != 0 && g == TN / 64) {
        tmem_ld32(tl + 64 * g, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        if constexpr (EPI == EPI_GELU) {
          gelu32(v);
        }
        if (row_ok) store_row32_f16(p.out + static_cast<size_t>(m) * p.ldo + n0 + 64 * g, v);
        break;
      }
      if (threadIdx.x == 0) bulk_wait_read<0>();  // the previous group's store has read the stage
      named_bar(1, EPI_WARPS * 32);
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        tmem_ld32(tl + 64 * g + 32 * h, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        if constexpr (EPI == EPI_GELU) {
          gelu32(v);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
          st_shared_v4(stage + row * 128 + (((4 * h + q) ^ (row & 7)) << 4), pack_half2(v[8 * q], v[8 * q + 1]),
                       pack_half2(v[8 * q + 2], v[8 * q + 3]), pack_half2(v[8 * q + 4], v[8 * q + 5]),
                       pack_half2(v[8 * q + 6], v[8 * q + 7]));
      }
      fence_proxy_async_smem();
      named_bar(1, EPI_WARPS * 32);
      if (threadIdx.x == 0) {
        if constexpr (EPI == EPI_GELU) tma_store_2d_evict_first(tmX, stage_ptr, n0 + 64 * g, m0);  // mlp hidden
        else tma_store_2d(tmX, stage_ptr, n0 + 64 * g, m0);
        bulk_commit();
      }
    }
  } else if constexpr (EPI == EPI_RESID) {
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      const int n = n0 + 32 * c;
      if (n >= p.N) break;  // warp-uniform
      tmem_ld32(tl + 32 * c, r);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
      if constexpr (EPI == EPI_RESID) {
        // x += gate * acc: stage gate*acc in shared memory and let TMA add it into x in L2
        // (no read of x by the SM). Chunk c of the previous iteration must have left the buffer.
        const float* g = p.gate + img * p.vec_bstride + n;
        const int row = warp * 32 + lane;
        if (threadIdx.x == 0) bulk_wait_read<0>();
        named_bar(1, EPI_WARPS * 32);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 gq = *reinterpret_cast<const float4*>(g + 4 * q);
          const uint32_t addr = stage + row * 128 + ((q ^ (row & 7)) << 4);
          st_shared_v4(addr, __float_as_uint(gq.x * v[4 * q]), __float_as_uint(gq.y * v[4 * q + 1]),
                       __float_as_uint(gq.z * v[4 * q + 2]), __float_as_uint(gq.w * v[4 * q + 3]));
        }
        fence_proxy_async_smem();
        named_bar(1, EPI_WARPS * 32);
        if (threadIdx.x == 0) {
          tma_reduce_add_2d(tmX, stage_ptr, n, m0);
          bulk_commit();
        }
      }
    }
  } else if constexpr (EPI == EPI_RMS) {
    // Both 128-column heads of the tile in a RoPE segment (q or k): their rows share one token, so each
    // chunk of 16 angles loads the row's cos / sin once for both heads.
    auto segment = [&](int cb, const float*& g, int& rp) {
      g = nullptr;
      rp = 0;
      if (cb < p.seg1) {
        g = p.gain0;
        rp = p.rope0;
      } else if (cb < p.seg2) {
        g = p.gain1;
        rp = p.rope1;
      }
    };
    const float *g0, *g1;
    int rp0, rp1;
    segment(n0, g0, rp0);
    segment(n0 + 128, g1, rp1);
    if (n0 + 128 < p.N && g0 && g1 && rp0 && rp1) {  // uniform over the epilogue warps
      uint32_t r2[32];
      float ss0 = 0.f, ss1 = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        tmem_ld32(tl + 32 * c, r);
        tmem_ld32(tl + 128 + 32 * c, r2);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float t0 = __uint_as_float(r[i]), t1 = __uint_as_float(r2[i]);
          ss0 = fmaf(t0, t0, ss0);
          ss1 = fmaf(t1, t1, ss1);
        }
      }
      const float rs0 = rsqrtf(ss0 * (1.0f / 128.0f) + p.eps), rs1 = rsqrtf(ss1 * (1.0f / 128.0f) + p.eps);
      const int tok = row_ok ? m % p.rows_per_img : 0;
      const float* cs = p.cosT + static_cast<size_t>(tok) * 64;
      const float* sn = p.sinT + static_cast<size_t>(tok) * 64;
      __half* orow = p.out + static_cast<size_t>(m) * p.ldo + n0;
      uint32_t a16[16], b16[16];
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {  // 16 angles at a time: cos / sin loaded once, then each head's pairs
        float cov[16], siv[16];
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 16; i += 4) {
            const float4 co = *reinterpret_cast<const float4*>(cs + 16 * c + i);
            const float4 si = *reinterpret_cast<const float4*>(sn + 16 * c + i);
            cov[i] = co.x; cov[i + 1] = co.y; cov[i + 2] = co.z; cov[i + 3] = co.w;
            siv[i] = si.x; siv[i + 1] = si.y; siv[i + 2] = si.z; siv[i + 3] = si.w;
          }
        }
#pragma unroll 1
        for (int hd = 0; hd < 2; ++hd) {
          const float* g = hd ? g1 : g0;
          const float rs = hd ? rs1 : rs0;
          tmem_ld16(tl + 128 * hd + 16 * c, a16);
          tmem_ld16(tl + 128 * hd + 64 + 16 * c, b16);
          tmem_ld_wait();
          if (!row_ok) continue;
#pragma unroll
          for (int i = 0; i < 16; i += 4) {
            const float4 ga = *reinterpret_cast<const float4*>(g + 16 * c + i);
            const float4 gb = *reinterpret_cast<const float4*>(g + 16 * c + i + 64);
            const float gav[4] = {ga.x, ga.y, ga.z, ga.w}, gbv[4] = {gb.x, gb.y, gb.z, gb.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float av = __uint_as_float(a16[i + e]) * rs * gav[e];
              const float bv = __uint_as_float(b16[i + e]) * rs * gbv[e];
              a16[i + e] = __float_as_uint(av * cov[i + e] - bv * siv[i + e]);
              b16[i + e] = __float_as_uint(bv * cov[i + e] + av * siv[i + e]);
            }
          }
          uint4* lo4 = reinterpret_cast<uint4*>(orow + 128 * hd + 16 * c);
          uint4* hi4 = reinterpret_cast<uint4*>(orow + 128 * hd + 64 + 16 * c);
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const float* fa = reinterpret_cast<const float*>(a16) + 8 * q;
            const float* fb = reinterpret_cast<const float*>(b16) + 8 * q;
            lo4[q] = make_uint4(pack_half2(fa[0], fa[1]), pack_half2(fa[2], fa[3]), pack_half2(fa[4], fa[5]),
                                pack_half2(fa[6], fa[7]));
            hi4[q] = make_uint4(pack_half2(fb[0], fb[1]), pack_half2(fb[2], fb[3]), pack_half2(fb[4], fb[5]),
                                pack_half2(fb[6], fb[7]));
          }
        }
      }
      return;
    }
#pragma unroll 1
    for (int hh = 0; hh < BN / 128; ++hh) {
      const int cb = n0 + 128 * hh;
      if (cb >= p.N) break;
      const float* gain = nullptr;
      int rope = 0;
      if (cb < p.seg1) {
        gain = p.gain0;
        rope = p.rope0;
      } else if (cb < p.seg2) {
        gain = p.gain1;
        rope = p.rope1;
      }
      const uint32_t th = tl + 128 * hh;
      if (gain == nullptr) {  // plain columns (e.g. v)
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          tmem_ld32(th + 32 * c, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
          if (row_ok) store_row32_f16(p.out + static_cast<size_t>(m) * p.ldo + cb + 32 * c, v);
        }
        continue;
      }
      float ss = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        tmem_ld32(th + 32 * c, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float t = __uint_as_float(r[i]);
          ss = fmaf(t, t, ss);
        }
      }
      const float rs = rsqrtf(ss * (1.0f / 128.0f) + p.eps);
      __half* orow = p.out + static_cast<size_t>(m) * p.ldo + cb;
      if (rope) {
        const int tok = row_ok ? m % p.rows_per_img : 0;
        const float* cs = p.cosT + static_cast<size_t>(tok) * 64;
        const float* sn = p.sinT + static_cast<size_t>(tok) * 64;
        uint32_t a16[16], b16[16];
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {  // pairs (d, d+64), 16 angles at a time
          tmem_ld16(th + 16 * c, a16);
          tmem_ld16(th + 64 + 16 * c, b16);
          tmem_ld_wait();
          if (!row_ok) continue;
#pragma unroll
          for (int i = 0; i < 16; i += 4) {
            const int d = 16 * c + i;
            const float4 ga = *reinterpret_cast<const float4*>(gain + d);
            const float4 gb = *reinterpret_cast<const float4*>(gain + d + 64);
            const float4 co = *reinterpret_cast<const float4*>(cs + d);
            const float4 si = *reinterpret_cast<const float4*>(sn + d);
            const float gav[4] = {ga.x, ga.y, ga.z, ga.w}, gbv[4] = {gb.x, gb.y, gb.z, gb.w};
            const float cov[4] = {co.x, co.y, co.z, co.w}, siv[4] = {si.x, si.y, si.z, si.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float av = __uint_as_float(a16[i + e]) * rs * gav[e];
              const float bv = __uint_as_float(b16[i + e]) * rs * gbv[e];
              a16[i + e] = __float_as_uint(av * cov[e] - bv * siv[e]);  // low half of the pair
              b16[i + e] = __float_as_uint(bv * cov[e] + av * siv[e]);  // high half
            }
          }
          uint4* lo4 = reinterpret_cast<uint4*>(orow + 16 * c);
          uint4* hi4 = reinterpret_cast<uint4*>(orow + 64 + 16 * c);
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const float* fa = reinterpret_cast<const float*>(a16) + 8 * q;
            const float* fb = reinterpret_cast<const float*>(b16) + 8 * q;
            lo4[q] = make_uint4(pack_half2(fa[0], fa[1]), pack_half2(fa[2], fa[3]), pack_half2(fa[4], fa[5]),
                                pack_half2(fa[6], fa[7]));
            hi4[q] = make_uint4(pack_half2(fb[0], fb[1]), pack_half2(fb[2], fb[3]), pack_half2(fb[4], fb[5]),
                                pack_half2(fb[6], fb[7]));
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          tmem_ld32(th + 32 * c, r);
          tmem_ld_wait();
          if (!row_ok) continue;
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const float4 gq = *reinterpret_cast<const float4*>(gain + 32 * c + i);
            v[i] = __uint_as_float(r[i]) * rs * gq.x;
            v[i + 1] = __uint_as_float(r[i + 1]) * rs * gq.y;
            v[i + 2] = __uint_as_float(r[i + 2]) * rs * gq.z;
            v[i + 3] = __uint_as_float(r[i + 3]) * rs * gq.w;
          }
          store_row32_f16(orow + 32 * c, v);
        }
      }
    }
  } else if constexpr (EPI == EPI_SITU) {
    // weight rows are interleaved per 256-row tile: [0,128) up_j, [128,256) gate_j of the same outputs
    uint32_t r2[32];
    const int o0 = n0 / 2;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      tmem_ld32(tl + 32 * c, r);
      tmem_ld32(tl + 128 + 32 * c, r2);
      tmem_ld_wait();
      if (!row_ok) continue;
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = situ(__uint_as_float(r[i]), __uint_as_float(r2[i]));
      store_row32_f16(p.out + static_cast<size_t>(m) * p.ldo + o0 + 32 * c, v);
    }
  }
}

// ---------------------------------------------------------------- the kernel
template <int FMT, int EPI>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmS,
                const __grid_constant__ CUtensorMap tmMin, const __grid_constant__ CUtensorMap tmX, const KParams p) {
  using C = Cfg<FMT>;
  constexpr int S = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* out_stage = smem + S * C::STAGE_BYTES;  // 1024-aligned
  uint64_t* bars = reinterpret_cast<uint64_t*>(out_stage + C::OUT_STAGE);
  uint64_t* full = bars;            // TMA data landed        (count 1 + tx)
  uint64_t* dqfull = bars + S;      // dequantised tile ready (count DQ_WARPS)
  uint64_t* empty = bars + 2 * S;   // MMAs done with stage   (count 1, tcgen05.commit)
  uint64_t* tfull = bars + 3 * S;   // accumulator ready      (count 1, tcgen05.commit)
  uint64_t* tempty = tfull + 2;     // accumulator drained    (count EPI_WARPS)
  uint64_t* drain = tempty + 2;     // abort path: last MMAs complete
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto stage_a = [&](int s) { return smem + s * C::STAGE_BYTES; };
  auto stage_wdq = [&](int s) { return smem + s * C::STAGE_BYTES + A_BYTES; };
  auto stage_raw = [&](int s) { return smem + s * C::STAGE_BYTES + A_BYTES + WDQ_BYTES; };
  auto stage_sc = [&](int s) { return smem + s * C::STAGE_BYTES + A_BYTES + WDQ_BYTES + C::RAW_BYTES; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&dqfull[i], DQ_WARPS);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], EPI_WARPS);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(tmem_base_slot, 512);
    tmem_relinquish();
  }
  if (warp == TMA_WARP && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmW);
    if (p.nkb1 < p.nkb) prefetch_tmap(&tmA2);
    if (FMT != WF_F16) prefetch_tmap(&tmS);
    if (EPI == EPI_RESID || EPI == EPI_STORE || EPI == EPI_GELU) prefetch_tmap(&tmX);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_slot;
  grid_dep_wait();  // the previous kernel's outputs (A, x) are complete
  grid_dep_launch();

  const int ntiles_mine = (p.num_tiles > static_cast<int>(blockIdx.x))
                              ? (p.num_tiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                              : 0;

  if (warp == TMA_WARP) {
    if (lane == 0) {
      constexpr uint32_t raw_tx = FMT == WF_F16 ? WDQ_BYTES : C::RAW_BYTES;
      const uint32_t sc_rows = FMT == WF_F16 ? 0 : (BK / p.group);
      const uint32_t sc_tx = sc_rows * BN * 2 * (FMT == WF_Q4A ? 2 : 1);
      const uint32_t tx = A_BYTES + raw_tx + sc_tx;
      int it = 0;
      bool ok = true;
      for (int ti = 0; ti < ntiles_mine && ok; ++ti) {
        const int t = blockIdx.x + ti * gridDim.x;
        const int m0 = tile_m(p, t) * BM, n0 = tile_n(p, t) * BN;
        for (int kb = 0; kb < p.nkb; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, p.status, 101)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], tx);
          if (kb < p.nkb1) tma_load_2d(stage_a(s), &tmA, &full[s], kb * BK, m0);
          else tma_load_2d(stage_a(s), &tmA2, &full[s], (kb - p.nkb1) * BK, m0);
          if constexpr (FMT == WF_F16) {
            tma_load_2d(stage_wdq(s), &tmW, &full[s], kb * BK, n0);
          } else {
            tma_load_2d(stage_raw(s), &tmW, &full[s], FMT == WF_Q8 ? kb * BK : kb * (BK / 2), n0);
            tma_load_2d(stage_sc(s), &tmS, &full[s], n0, kb * static_cast<int>(sc_rows));
            if constexpr (FMT == WF_Q4A)
              tma_load_2d(stage_sc(s) + 2 * BN * 2, &tmMin, &full[s], n0, kb * static_cast<int>(sc_rows));
          }
        }
      }
      if (!ok) {  // drain loads still in flight before the CTA may exit
        for (int j = (it > S ? it - S : 0); j < it; ++j) mbar_wait(&full[j % S], (j / S) & 1, nullptr, 0);
      }
    }
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(BM, BN, 0, 0);
      int it = 0;
      bool ok = true, issued = false;
      for (int ti = 0; ti < ntiles_mine && ok; ++ti) {
        const int acc = ti & 1;
        if (!mbar_wait(&tempty[acc], ((ti >> 1) & 1) ^ 1, p.status, 102)) { ok = false; break; }
        tc_fence_after();
        const uint32_t dt = tmem + acc * BN;
        for (int kb = 0; kb < p.nkb; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          if (!mbar_wait(&full[s], ph, p.status, 103)) { ok = false; break; }
          if constexpr (FMT != WF_F16) {
            if (!mbar_wait(&dqfull[s], ph, p.status, 104)) { ok = false; break; }
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(stage_a(s)), b0 = smem_u32(stage_wdq(s));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            mma_f16_ss(dt, sdesc_sw128(a0 + 32 * k, 16, 1024), sdesc_sw128(b0 + 32 * k, 16, 1024), idesc,
                       (kb | k) != 0);
          }
          issued = true;
          mma_commit(&empty[s]);
        }
        if (!ok) break;
        mma_commit(&tfull[acc]);
      }
      if (!ok && issued) {
        mma_commit(drain);
        mbar_wait(drain, 0, nullptr, 0);
      }
    }
  } else if (warp >= DQ_WARP0) {
    if constexpr (FMT != WF_F16) {
      const int dt = threadIdx.x - DQ_WARP0 * 32;
      int it = 0;
      bool ok = true;
      for (int ti = 0; ti < ntiles_mine && ok; ++ti) {
        for (int kb = 0; kb < p.nkb; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          if (!mbar_wait(&full[s], ph, p.status, 105)) { ok = false; break; }
          dequant_kblock<FMT>(smem_u32(stage_raw(s)), smem_u32(stage_wdq(s)),
                              reinterpret_cast<const __half*>(stage_sc(s)), p.group, dt);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&dqfull[s]);
        }
      }
    }
  } else {  // epilogue warps 0..3
    bool ok = true;
    for (int ti = 0; ti < ntiles_mine && ok; ++ti) {
      const int t = blockIdx.x + ti * gridDim.x;
      const int m0 = tile_m(p, t) * BM, n0 = tile_n(p, t) * BN;
      const int acc = ti & 1;
      // the epilogue warps meet at named barrier 1 in epilogue_tile: they leave together or not at all
      if (!bar_and(2, EPI_WARPS * 32, mbar_wait(&tfull[acc], (ti >> 1) & 1, p.status, 106))) {
        ok = false;
        break;
      }
      tc_fence_after();
      epilogue_tile<EPI>(p, tmem + acc * BN, m0, n0, warp, lane, &tmX, out_stage);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    if constexpr (EPI == EPI_RESID || EPI == EPI_STORE || EPI == EPI_GELU) {
      if (threadIdx.x == 0) bulk_wait<0>();  // stores / reductions complete before the shared memory goes away
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == MMA_WARP) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------- CTA-pair kernel (cta_group::2)
// 256x256 output tile per cluster of 2 CTAs. CTA r loads A rows [m0 + 128r, +128) and weight rows
// [n0 + 128r, +128) and dequantises only those 128 weight rows; the leader (r = 0) issues
// tcgen05.mma.cta_group::2 (M 256, N 256, K 16) which reads A and B halves from both CTAs' shared
// memory at the same offsets and writes each CTA's 128 accumulator rows into its own TMEM.
// Barrier protocol (after the SM100 mixed-input transform kernel of CUTLASS):
//   full_a  (leader): both CTAs' A (and fp16 B) TMA loads complete on it; the leader's producer
//                     arrives once with the pair's transaction bytes
//   raw_full(each)  : local raw int8/int4 + scale loads, waited by the local dequant warps
//   dq_full (leader): every dequant warp of both CTAs arrives after its 128 rows are written
//   empty   (each)  : the leader's MMA commit, multicast to both CTAs
//   tfull   (each)  : accumulator ready, commit multicast; tempty (leader): 4 epilogue warps per CTA
constexpr int HALF = 128;

// TN: the pair tile's N (256, or 224: each CTA then holds 112 weight rows of the B operand). Every stage
// part stays a multiple of 1 KB, the alignment of the 128-byte swizzled operand tiles.
template <int FMT, int TN = BN>
struct Cfg2 {
  static constexpr int HB = TN / 2;  // weight rows per CTA
  static constexpr int A_B = HALF * BK * 2;
  static constexpr int WDQ_B = HB * BK * 2;
  static constexpr int RAW_B = FMT == WF_F16 ? 0 : FMT == WF_Q8 ? HB * BK : HB * BK / 2;
  static constexpr int SC_B = FMT == WF_F16 ? 0 : 1024;
  static constexpr int STAGE = A_B + WDQ_B + RAW_B + SC_B;
  static constexpr int STAGES = FMT == WF_F16 ? 6 : 5;
  static constexpr int OUT_STAGE = 16384;
  static constexpr int SMEM = STAGES * STAGE + OUT_STAGE + 1024 + 1024;
  static_assert(WDQ_B % 1024 == 0 && RAW_B % 1024 == 0 && STAGE % 1024 == 0, "stage alignment");
  static_assert(TN == BN || TN == 224, "pair tile width");
};

__device__ __forceinline__ void spin_ns(uint64_t ns) {
  const uint64_t t0 = globaltimer();
  while (globaltimer() - t0 < ns) {
  }
}

template <int FMT, int EPI, int TN = BN>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                 const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmS,
                 const __grid_constant__ CUtensorMap tmMin, const __grid_constant__ CUtensorMap tmX,
                 const KParams p) {
  using C = Cfg2<FMT, TN>;
  constexpr int HB = C::HB;
  constexpr int S = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* out_stage = smem + S * C::STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(out_stage + C::OUT_STAGE);
  uint64_t* full_a = bars;
  uint64_t* raw_full = bars + S;
  uint64_t* dq_full = bars + 2 * S;
  uint64_t* empty = bars + 3 * S;
  uint64_t* tfull = bars + 4 * S;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  auto st_a = [&](int s) { return smem + s * C::STAGE; };
  auto st_w = [&](int s) { return smem + s * C::STAGE + C::A_B; };
  auto st_raw = [&](int s) { return smem + s * C::STAGE + C::A_B + C::WDQ_B; };
  auto st_sc = [&](int s) { return smem + s * C::STAGE + C::A_B + C::WDQ_B + C::RAW_B; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_a[i], 1);
      mbar_init(&raw_full[i], 1);
      mbar_init(&dq_full[i], 2 * DQ_WARPS);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 2 * EPI_WARPS);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc_pair(tmem_base_slot, 512);
    tmem_relinquish_pair();
  }
  if (warp == TMA_WARP && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmW);
    if (p.nkb1 < p.nkb) prefetch_tmap(&tmA2);
    if (FMT != WF_F16) prefetch_tmap(&tmS);
    if (EPI == EPI_RESID || EPI == EPI_STORE || EPI == EPI_GELU) prefetch_tmap(&tmX);
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM of the pair allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_base_slot;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int row0 = static_cast<int>(rank) * HALF;  // this CTA's A rows in the pair tile
  const int brow0 = static_cast<int>(rank) * HB;   // and its weight rows
  // Quantised weight tiles and scales are constant during inference (no kernel that can precede this one
  // with programmatic dependent launch writes them; fp16 weights can be an expansion just before, so they
  // wait), so the producer loads the first ring of them before waiting for the previous kernel.
  int npre = 0;
  if constexpr (FMT != WF_F16) {
    if (warp == TMA_WARP && lane == 0) {
      Sched sched(p, pair, npairs);
      int t, kb0, kb1;
      if (sched.next(p, t, kb0, kb1)) {
        const uint32_t sc_rows = BK / p.group;
        const uint32_t raw_tx = C::RAW_B + sc_rows * HB * 2 * (FMT == WF_Q4A ? 2 : 1);
        const int n0 = tile_n(p, t) * TN + brow0;
        npre = kb1 - kb0 < S ? kb1 - kb0 : S;
        for (int i = 0; i < npre; ++i) {  // stages i are empty on the first pass
          const int kb = kb0 + i;
          mbar_arrive_expect_tx(&raw_full[i], raw_tx);
          tma_load_2d(st_raw(i), &tmW, &raw_full[i], FMT == WF_Q8 ? kb * BK : kb * (BK / 2), n0);
          tma_load_2d(st_sc(i), &tmS, &raw_full[i], n0, kb * static_cast<int>(sc_rows));
          if constexpr (FMT == WF_Q4A)
            tma_load_2d(st_sc(i) + 2 * HB * 2, &tmMin, &raw_full[i], n0, kb * static_cast<int>(sc_rows));
        }
      }
    }
  }
  grid_dep_wait();  // the previous kernel's outputs (A, x) are complete
  grid_dep_launch();

  if (warp == TMA_WARP) {
    if (lane == 0) {
      const uint32_t tx_a = 2u * (C::A_B + (FMT == WF_F16 ? C::WDQ_B : 0));
      const uint32_t sc_rows = FMT == WF_F16 ? 0 : (BK / p.group);
      const uint32_t raw_tx = C::RAW_B + sc_rows * HB * 2 * (FMT == WF_Q4A ? 2 : 1);
      int it = 0;
      bool ok = true;
      Sched sched(p, pair, npairs);
      int t, kb0, kb1;
      while (ok && sched.next(p, t, kb0, kb1)) {
        const int m0 = tile_m(p, t) * 2 * HALF + row0, n0 = tile_n(p, t) * TN + brow0;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, p.status, 111)) { ok = false; break; }
          if (leader) mbar_arrive_expect_tx(&full_a[s], tx_a);
          if (kb < p.nkb1) tma_load_2d_pair(st_a(s), &tmA, &full_a[s], kb * BK, m0);
          else tma_load_2d_pair(st_a(s), &tmA2, &full_a[s], (kb - p.nkb1) * BK, m0);
          if constexpr (FMT == WF_F16) {
            tma_load_2d_pair(st_w(s), &tmW, &full_a[s], kb * BK, n0);
          } else if (it >= npre) {  // the first npre were loaded before the dependency wait
            mbar_arrive_expect_tx(&raw_full[s], raw_tx);
            tma_load_2d(st_raw(s), &tmW, &raw_full[s], FMT == WF_Q8 ? kb * BK : kb * (BK / 2), n0);
            tma_load_2d(st_sc(s), &tmS, &raw_full[s], n0, kb * static_cast<int>(sc_rows));
            if constexpr (FMT == WF_Q4A)
              tma_load_2d(st_sc(s) + 2 * HB * 2, &tmMin, &raw_full[s], n0, kb * static_cast<int>(sc_rows));
          }
        }
      }
      if (!ok) spin_ns(2000000);  // loads issued before the abort land long before this
    }
  } else if (warp == MMA_WARP) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = idesc_f16(2 * HALF, TN, 0, 0);
      int it = 0;
      bool ok = true, issued = false;
      Sched sched(p, pair, npairs);
      int t, kb0, kb1;
      for (int ti = 0; ok && sched.next(p, t, kb0, kb1); ++ti) {
        const int acc = ti & 1;
        if (!mbar_wait(&tempty[acc], ((ti >> 1) & 1) ^ 1, p.status, 112)) { ok = false; break; }
        tc_fence_after();
        const uint32_t dt = tmem + acc * BN;  // accumulators at columns 0 and 256 (TN <= 256 each)
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          if (!mbar_wait(&full_a[s], ph, p.status, 113)) { ok = false; break; }
          if constexpr (FMT != WF_F16) {
            if (!mbar_wait(&dq_full[s], ph, p.status, 114)) { ok = false; break; }
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(st_a(s)), b0 = smem_u32(st_w(s));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_f16_ss_pair(dt, sdesc_sw128(a0 + 32 * k, 16, 1024), sdesc_sw128(b0 + 32 * k, 16, 1024), idesc,
                            (kb != kb0 || k != 0));
          issued = true;
          mma_commit_pair_mc(&empty[s], 0x3);
        }
        if (!ok) break;
        mma_commit_pair_mc(&tfull[acc], 0x3);
      }
      if (!ok && issued) {
        mma_commit_pair(drain);
        mbar_wait(drain, 0, nullptr, 0);
      }
    }
  } else if (warp >= DQ_WARP0) {
    if constexpr (FMT != WF_F16) {
      const int dt = threadIdx.x - DQ_WARP0 * 32;
      int it = 0;
      bool ok = true;
      Sched sched(p, pair, npairs);
      int t, kb0, kb1;
      while (ok && sched.next(p, t, kb0, kb1)) {
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          if (!mbar_wait(&raw_full[s], ph, p.status, 115)) { ok = false; break; }
          dequant_kblock<FMT, HB>(smem_u32(st_raw(s)), smem_u32(st_w(s)), reinterpret_cast<const __half*>(st_sc(s)),
                                    p.group, dt);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive_leader(&dq_full[s]);
        }
      }
    }
  } else {  // epilogue warps 0..3: this CTA's 128 rows of the pair tile
    bool ok = true;
    Sched sched(p, pair, npairs);
    int t, kb0, kb1;
    for (int ti = 0; ok && sched.next(p, t, kb0, kb1); ++ti) {
      const int m0 = tile_m(p, t) * 2 * HALF + row0, n0 = tile_n(p, t) * TN;
      const int acc = ti & 1;
      // the epilogue warps meet at named barrier 1 in epilogue_tile: they leave together or not at all
      if (!bar_and(2, EPI_WARPS * 32, mbar_wait(&tfull[acc], (ti >> 1) & 1, p.status, 116))) {
        ok = false;
        break;
      }
      tc_fence_after();
      epilogue_tile<EPI, TN>(p, tmem + acc * BN, m0, n0, warp, lane, &tmX, out_stage);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_leader(&tempty[acc]);
    }
    if constexpr (EPI == EPI_RESID || EPI == EPI_STORE || EPI == EPI_GELU) {
      if (threadIdx.x == 0) bulk_wait<0>();  // stores and reduce-adds of the last tile complete
    }
  }

  tc_fence_before();
  cluster_sync();  // the pair's MMAs and epilogues are done before either CTA frees TMEM
  tc_fence_after();
  if (warp == MMA_WARP) tmem_dealloc_pair(tmem, 512);
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

}  // namespace

// 2D row-major tensor [outer][inner] with row pitch `pitch_bytes`; box [box_outer][box_inner].
bool make_tmap_2d(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* base, uint64_t inner,
                  uint64_t outer, uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_outer,
                  CUtensorMapSwizzle sw) {
  auto fn = encode_fn();
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (pitch_bytes & 15) || ((box_inner * esize) & 15)) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_tmap_3d(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* base, uint64_t d0, uint64_t d1,
                  uint64_t d2, uint64_t pitch1, uint64_t pitch2, uint32_t b0, uint32_t b1, uint32_t b2,
                  CUtensorMapSwizzle sw) {
  auto fn = encode_fn();
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (pitch1 & 15) || (pitch2 & 15) || ((b0 * esize) & 15))
    return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {pitch1, pitch2};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int expand_min_rows() {
  static const int rows = [] {
    const char* e = getenv("HX_EXPAND_ROWS");
    return e && *e ? atoi(e) : 3072;
  }();
  return rows;
}

// HX_GROUP_M: M tiles per band of the banded tile order (-1 = not set: the library's choice)
int group_m_override() {
  static const int g = [] {
    const char* e = getenv("HX_GROUP_M");
    return e && *e ? atoi(e) : -1;
  }();
  return g;
}

int pair_tn_override() {
  static const int t = [] {
    const char* e = getenv("HX_PAIR_TN");
    return e && *e ? atoi(e) : 0;
  }();
  return t;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("HX_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

int sm_count() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!n[dev]) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
  return n[dev] ? n[dev] : 148;
}

template <int FMT, int EPI>
static cudaError_t launch_t(const GemmArgs& a, const KParams& p, const CUtensorMap& tA, const CUtensorMap& tA2,
                            const CUtensorMap& tW, const CUtensorMap& tS, const CUtensorMap& tMin,
                            const CUtensorMap& tX, cudaStream_t s) {
  using C = Cfg<FMT>;
  static uint64_t attr_set = 0;  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set >> dev & 1)) {
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel<FMT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    attr_set |= 1ull << dev;
  }
  int grid = sm_count();
  if (a.max_ctas > 0 && a.max_ctas < grid) grid = a.max_ctas;
  if (p.num_tiles < grid) grid = p.num_tiles;
  const cudaError_t e = launch_pdl(gemm_kernel<FMT, EPI>, dim3(grid), dim3(GEMM_THREADS), C::SMEM, s, tA, tA2, tW, tS,
                                   tMin, tX, p);
  return e != cudaSuccess ? e : cudaGetLastError();
}

template <int FMT, int EPI, int TN = BN>
static cudaError_t launch_pair_t(const GemmArgs& a, const KParams& p, const CUtensorMap& tA, const CUtensorMap& tA2,
                                 const CUtensorMap& tW, const CUtensorMap& tS, const CUtensorMap& tMin,
                                 const CUtensorMap& tX, cudaStream_t s) {
  using C = Cfg2<FMT, TN>;
  static uint64_t attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set >> dev & 1)) {
    cudaError_t e = cudaFuncSetAttribute(gemm2_kernel<FMT, EPI, TN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    attr_set |= 1ull << dev;
  }
  int npairs = sm_count() / 2;
  if (a.max_ctas > 0 && a.max_ctas / 2 < npairs) npairs = a.max_ctas / 2 > 0 ? a.max_ctas / 2 : 1;
  const long long units = p.streamk ? static_cast<long long>(p.num_tiles) * p.nkb : p.num_tiles;
  if (units < npairs) npairs = static_cast<int>(units);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * npairs);
  cfg.blockDim = dim3(GEMM_THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_attr(attr, 1);
  return cudaLaunchKernelEx(&cfg, gemm2_kernel<FMT, EPI, TN>, tA, tA2, tW, tS, tMin, tX, p);
}

template <int FMT>
static cudaError_t launch_pair_fmt(const GemmArgs& a, const KParams& p, const CUtensorMap& tA, const CUtensorMap& tA2,
                                   const CUtensorMap& tW, const CUtensorMap& tS, const CUtensorMap& tMin,
                                   const CUtensorMap& tX, cudaStream_t s, int tn) {
  if constexpr (FMT == WF_F16 || FMT == WF_Q8) {
    if (tn == 224) {
      if (a.epi == EPI_GELU) return launch_pair_t<FMT, EPI_GELU, 224>(a, p, tA, tA2, tW, tS, tMin, tX, s);
      if (a.epi == EPI_STORE) return launch_pair_t<FMT, EPI_STORE, 224>(a, p, tA, tA2, tW, tS, tMin, tX, s);
      return cudaErrorInvalidValue;
    }
  }
  if (tn != BN) return cudaErrorInvalidValue;
  switch (a.epi) {
    case EPI_STORE: return launch_pair_t<FMT, EPI_STORE>(a, p, tA, tA2, tW, tS, tMin, tX, s);
    case EPI_RESID: return launch_pair_t<FMT, EPI_RESID>(a, p, tA, tA2, tW, tS, tMin, tX, s);
    case EPI_GELU: return launch_pair_t<FMT, EPI_GELU>(a, p, tA, tA2, tW, tS, tMin, tX, s);
    case EPI_RMS: return launch_pair_t<FMT, EPI_RMS>(a, p, tA, tA2, tW, tS, tMin, tX, s);
    case EPI_SITU: return launch_pair_t<FMT, EPI_SITU>(a, p, tA, tA2, tW, tS, tMin, tX, s);
    case EPI_STORE32: return launch_pair_t<FMT, EPI_STORE32>(a, p, tA, tA2, tW, tS, tMin, tX, s);
  }
  return cudaErrorInvalidValue;
}

template <int FMT>
static cudaError_t launch_fmt(const GemmArgs& a, const KParams& p, const CUtensorMap& tA, const CUtensorMap& tA2,
                              const CUtensorMap& tW, const CUtensorMap& tS, const CUtensorMap& tMin,
                              const CUtensorMap& tX, cudaStream_t s) {
  switch (a.epi) {
    case EPI_STORE: return launch_t<FMT, EPI_STORE>(a, p, tA, tA2, tW, tS, tMin, tX, s);
    case EPI_RESID: return launch_t<FMT, EPI_RESID>(a, p, tA, tA2, tW, tS, tMin, tX, s);
    case EPI_GELU: return launch_t<FMT, EPI_GELU>(a, p, tA, tA2, tW, tS, tMin, tX, s);
    case EPI_RMS: return launch_t<FMT, EPI_RMS>(a, p, tA, tA2, tW, tS, tMin, tX, s);
    case EPI_SITU: return launch_t<FMT, EPI_SITU>(a, p, tA, tA2, tW, tS, tMin, tX, s);
    case EPI_STORE32: return launch_t<FMT, EPI_STORE32>(a, p, tA, tA2, tW, tS, tMin, tX, s);
  }
  return cudaErrorInvalidValue;
}

// The launch decisions of gemm_launch for a GEMM on a GPU with `sms` SMs, made on the host alone (also
// answered by hx_gemm_query). `have_scratch`: the caller's fp16 scratch can hold the expanded weights.
cudaError_t gemm_choose(const GemmArgs& a, int sms, bool have_scratch, GemmChoice& c) {
  const DevMat* W = a.W;
  if (!W || !a.A || a.M <= 0 || W->N <= 0 || W->K <= 0 || sms < 2) return cudaErrorInvalidValue;
  const int N = W->N, K = W->K;
  if (K % BK || a.K1 % BK || a.K1 <= 0 || a.K1 > K || N % 32) return cudaErrorInvalidValue;
  if (a.K1 < K && (!a.A2 || a.lda2 < K - a.K1)) return cudaErrorInvalidValue;
  if ((a.epi == EPI_RMS && N % 128) || (a.epi == EPI_SITU && N % BN)) return cudaErrorInvalidValue;
  if (a.epi == EPI_RESID && (!a.x || !a.gate)) return cudaErrorInvalidValue;
  if (a.epi == EPI_STORE32 && (!a.x || a.ldx % 4)) return cudaErrorInvalidValue;
  if (a.epi != EPI_RESID && a.epi != EPI_STORE32 && !a.out) return cudaErrorInvalidValue;
  // fp16 outputs are written 16 bytes at a time (and by TMA stores): 16-byte aligned rows
  if (a.epi != EPI_RESID && a.epi != EPI_STORE32 &&
      (a.ldo % 8 || reinterpret_cast<uintptr_t>(a.out) % 16 || a.ldo < (a.epi == EPI_SITU ? N / 2 : N)))
    return cudaErrorInvalidValue;
  if (W->fmt == WF_Q8 && W->group != 32 && W->group != 64) return cudaErrorInvalidValue;
  if ((W->fmt == WF_Q4 || W->fmt == WF_Q4A) && W->group != 32) return cudaErrorInvalidValue;
  c = GemmChoice();

  // Quantised weights with enough rows to amortise it: expand W to fp16 in the caller's scratch (one
  // memory-bound pass, 3 bytes per q8 weight), then run the fp16 kernels, which move no raw tile or
  // scales through shared memory and need no dequant warps in the main loop. On the 8-image Anima block
  // the q8 GEMMs run 12-21 % faster this way; the pass costs about N K 3 bytes of HBM / L2 traffic, so
  // it pays from about two images (3072 rows) up.
  if (W->fmt != WF_F16 && a.tile != 3 && (a.tile == 4 || (a.tile == 0 && a.M >= expand_min_rows()))) {
    if (have_scratch) {
      c.expand = true;
      return cudaSuccess;  // the fp16 GEMM that follows is chosen for fp16 weights and tile 0
    }
    if (a.tile == 4) return cudaErrorInvalidValue;  // forced, but no scratch of N K fp16
  }

  // tile configuration: CTA pairs (256x256 per cluster) unless single-CTA 128x256 tiles need fewer waves
  // (a pair moves half the weight tile per SM, so at equal waves it is the faster of the two: at one
  // image the down projection runs 67 us in pairs against 86 us in single CTAs)
  const int npairs = sms / 2;
  const int pair_tiles = ((a.M + 2 * HALF - 1) / (2 * HALF)) * ((N + BN - 1) / BN);
  // residual GEMMs with a long K and fewer than two waves of pair tiles take the stream-K schedule below
  const bool streamk_candidate = a.epi == EPI_RESID && a.max_ctas == 0 && pair_tiles < sms &&
                                 static_cast<long long>(pair_tiles % npairs) * (K / BK) >= 32LL * npairs;

  // q8 weights below the expansion threshold: the kernel that keeps the dequantised weights in TMEM takes
  // the RMS (q/k/v projection) epilogue when its tiles fill the GPU (2-3 % faster there than the CTA-pair
  // kernel, which is 3-7 % faster with the store, GELU and residual epilogues at several waves)
  if (a.tile == 3) {
    if (!gemm_wt_eligible(a)) return cudaErrorInvalidValue;
    c.kernel = 3;
    return cudaSuccess;
  }
  if (a.tile == 0 && gemm_wt_eligible(a)) {
    const int wt_tiles = gemm_wt_tiles(a);
    // at most one wave of tiles with a residual or RMS epilogue (the N = 2048 projections at one image):
    // each pair has a single tile, so its epilogue is not hidden behind another tile's main loop, and the
    // TMEM-weight kernel's 8 epilogue warps per CTA with double-buffered per-warp boxes drain it faster
    // than the CTA-pair kernel's 4 warps and single staging buffer (o projection at one image: 22.5
    // against 25.6 us)
    if ((a.epi == EPI_RMS && wt_tiles >= npairs) ||
        ((a.epi == EPI_RESID || a.epi == EPI_RMS) && wt_tiles <= npairs && a.max_ctas == 0 && !streamk_candidate)) {
      c.kernel = 3;
      return cudaSuccess;
    }
  }

  const int single_tiles = ((a.M + BM - 1) / BM) * ((N + BN - 1) / BN);
  bool pair = a.tile == 2 || (a.tile == 0 && (pair_tiles + npairs - 1) / npairs <= (single_tiles + sms - 1) / sms);
  // residual GEMMs with fewer than two waves of pair tiles (one or two images per GPU): the CTA-pair
  // kernel with a stream-K tail, so no pair idles through a mostly empty last wave (one image: 48 tiles on
  // 74 pairs; down projection 68 -> 55 us, two images 122 -> 93 us). Tiles cut between two pairs reduce-add two
  // partial sums into x, in no fixed order. From two waves up the plain tile schedule stays: at 4 and 8
  // images the GEMMs run at the power cap, where the idle tail costs energy rather than time, and both
  // schedules measured the same, so x stays bit-reproducible there.
  // Each pair's share of the tail must be at least 32 k-blocks: shorter units (the o projection, K = 2048,
  // at one or two images: 21 and 10 k-blocks) lose more to their pipeline fill and extra partial tiles
  // than the balance gains.
  int streamk = 0;
  if (a.tile == 0 && streamk_candidate) {
    pair = true;
    streamk = 1;
  }
  // CTA-pair GELU tiles 224 columns wide when they take no more waves than 256-column tiles: N = 8192
  // makes 32 tiles of 256 per 256-row band but 37 of 224 (the last 128 wide), so at 1536 rows 222 tiles
  // are exactly 3 waves on 74 pairs, as are 192 tiles of 256 (the last wave 60 % full), and at 3072 rows
  // 444 against 384 tiles both take 6. A 224-column tile costs about 0.955 of a 256-column one (the A
  // tile is loaded whole either way), so measured mlp.layer1: one image 54.0 -> 53.2 us (q8 in the main
  // loop), 45.0 -> 43.7 (fp16), two images 92.8 -> 92.3; at four images (12 against 11 waves) 224 was
  // slower (175.5 against 168.1) and is not taken. tile 5 forces 224 (GELU or plain store),
  // HX_PAIR_TN=256 / 224 in the environment overrides the choice.
  int tn = BN;
  if (a.tile == 5) {
    if ((a.epi != EPI_GELU && a.epi != EPI_STORE) || (W->fmt != WF_F16 && W->fmt != WF_Q8))
      return cudaErrorInvalidValue;
    pair = true;
    tn = 224;
  } else if (pair && !streamk && a.epi == EPI_GELU && (W->fmt == WF_F16 || W->fmt == WF_Q8)) {
    const int ov = pair_tn_override();
    if (ov == 224) {
      tn = 224;
    } else if (ov != BN) {
      int np = npairs;
      if (a.max_ctas > 0 && a.max_ctas / 2 < np) np = a.max_ctas / 2 > 0 ? a.max_ctas / 2 : 1;
      const long long mt = (a.M + 2 * HALF - 1) / (2 * HALF);
      const long long w256 = (mt * ((N + BN - 1) / BN) + np - 1) / np;
      const long long w224 = (mt * ((N + 223) / 224) + np - 1) / np;
      if (w224 <= w256) tn = 224;
    }
  }
  c.kernel = pair ? 2 : 1;
  c.tile_n = tn;
  c.streamk = streamk;
  c.tiles = pair ? static_cast<int>(((a.M + 2 * HALF - 1) / (2 * HALF)) * ((N + tn - 1) / tn)) : single_tiles;
  return cudaSuccess;
}

cudaError_t gemm_launch(const GemmArgs& a, cudaStream_t s) {
  const DevMat* W = a.W;
  const size_t need = W ? static_cast<size_t>(W->N) * W->K * 2 : 0;
  GemmChoice c;
  cudaError_t ce = gemm_choose(a, sm_count(), a.wexp && a.wexp_bytes >= need, c);
  if (ce != cudaSuccess) return ce;
  const int N = W->N, K = W->K;
  if (c.expand) {
    cudaError_t e = expand_launch(*W, a.wexp, s);
    if (e != cudaSuccess) return e;
    DevMat f;
    f.fmt = WF_F16;
    f.N = N;
    f.K = K;
    f.group = 64;
    f.w = a.wexp;
    GemmArgs b = a;
    b.W = &f;
    b.tile = 0;
    b.wexp = nullptr;
    b.wexp_bytes = 0;
    return gemm_launch(b, s);
  }
  if (c.kernel == 3) return gemm_wt_launch(a, s);
  const bool pair = c.kernel == 2;
  const int tn = c.tile_n, streamk = c.streamk;
  const uint32_t wrows = pair ? static_cast<uint32_t>(tn / 2) : BN;

  CUtensorMap tA, tA2, tW, tS, tMin, tX;
  memset(&tA2, 0, sizeof tA2);
  memset(&tS, 0, sizeof tS);
  memset(&tMin, 0, sizeof tMin);
  memset(&tX, 0, sizeof tX);
  if (a.epi == EPI_RESID &&
      !make_tmap_2d(&tX, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a.x, N, a.M, static_cast<uint64_t>(a.ldx) * 4, 32, BM,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if ((a.epi == EPI_STORE || a.epi == EPI_GELU) &&
      !make_tmap_2d(&tX, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.out, N, a.M, static_cast<uint64_t>(a.ldo) * 2, 64, BM,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (!make_tmap_2d(&tA, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.A, a.K1, a.M, static_cast<uint64_t>(a.lda) * 2, BK,
                    BM, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (a.K1 < K && !make_tmap_2d(&tA2, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.A2, K - a.K1, a.M,
                                static_cast<uint64_t>(a.lda2) * 2, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  bool ok = true;
  switch (W->fmt) {
    case WF_F16:
      ok = make_tmap_2d(&tW, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, W->w, K, N, static_cast<uint64_t>(K) * 2, BK, wrows,
                        CU_TENSOR_MAP_SWIZZLE_128B);
      break;
    case WF_Q8:
      ok = make_tmap_2d(&tW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, W->w, K, N, K, BK, wrows, CU_TENSOR_MAP_SWIZZLE_NONE);
      break;
    default:
      ok = make_tmap_2d(&tW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, W->w, K / 2, N, K / 2, BK / 2, wrows,
                        CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  if (ok && W->fmt != WF_F16)
    ok = make_tmap_2d(&tS, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, W->scale, N, K / W->group,
                      static_cast<uint64_t>(N) * 2, wrows, BK / W->group, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (ok && W->fmt == WF_Q4A)
    ok = make_tmap_2d(&tMin, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, W->minv, N, K / W->group,
                      static_cast<uint64_t>(N) * 2, wrows, BK / W->group, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!ok) return cudaErrorInvalidValue;

  KParams p;
  p.M = a.M;
  p.N = N;
  p.nkb = K / BK;
  p.nkb1 = a.K1 / BK;
  p.group = W->fmt == WF_F16 ? 64 : W->group;
  p.num_m_tiles = pair ? (a.M + 2 * HALF - 1) / (2 * HALF) : (a.M + BM - 1) / BM;
  p.num_n_tiles = (N + tn - 1) / tn;
  p.streamk = streamk;
  p.num_tiles = p.num_m_tiles * p.num_n_tiles;
  // default order walks M tiles under one weight block (the weight block stays in L2); when the A
  // operand is far larger than L2 but the weights fit (the mlp down projection reading the 8-image
  // hidden state), walk the N tiles of one A block instead so A streams from HBM once
  {
    const double a_bytes = static_cast<double>(a.M) * K * 2;
    const double w_bytes = static_cast<double>(N) * K * (W->fmt == WF_F16 ? 2.0 : W->fmt == WF_Q8 ? 1.0 : 0.5);
    p.n_fastest = a_bytes > 64e6 && w_bytes < 64e6 ? 1 : 0;
    // banded order when A exceeds 32 MB: bands of about 8 MB of A rows (HX_GROUP_M overrides the band in M
    // tiles; 0 = off). Measured on the mlp.layer1 GEMM: at 12288 rows (A 50 MB) DRAM traffic per call
    // 365.8 -> 304.8 MB and +2.7 % speed; at 3072-6144 rows (A 12-25 MB) the M-fastest order moves less
    const int rows = pair ? 2 * HALF : BM;
    const int gm = group_m_override();
    p.group_m = gm >= 0 ? gm : (a_bytes > 32e6 ? std::max(1, static_cast<int>(8e6 / (static_cast<double>(rows) * K * 2))) : 0);
    if (p.n_fastest || p.group_m >= p.num_m_tiles) p.group_m = 0;
  }
  p.out = a.out;
  p.ldo = a.ldo;
  p.x = a.x;
  p.ldx = a.ldx;
  p.gate = a.gate;
  p.vec_bstride = a.vec_bstride;
  p.rows_per_img = a.rows_per_img > 0 ? a.rows_per_img : (1 << 30);
  p.gain0 = a.gain0;
  p.gain1 = a.gain1;
  p.seg1 = a.seg1;
  p.seg2 = a.seg2;
  p.rope0 = a.rope0;
  p.rope1 = a.rope1;
  p.cosT = a.cosT;
  p.sinT = a.sinT;
  p.eps = a.eps;
  p.status = a.status;
  if ((p.rope0 || p.rope1) && (!p.cosT || !p.sinT)) return cudaErrorInvalidValue;

  if (pair) {
    switch (W->fmt) {
      case WF_F16: return launch_pair_fmt<WF_F16>(a, p, tA, tA2, tW, tS, tMin, tX, s, tn);
      case WF_Q8: return launch_pair_fmt<WF_Q8>(a, p, tA, tA2, tW, tS, tMin, tX, s, tn);
      case WF_Q4: return launch_pair_fmt<WF_Q4>(a, p, tA, tA2, tW, tS, tMin, tX, s, tn);
      case WF_Q4A: return launch_pair_fmt<WF_Q4A>(a, p, tA, tA2, tW, tS, tMin, tX, s, tn);
    }
    return cudaErrorInvalidValue;
  }
  switch (W->fmt) {
    case WF_F16: return launch_fmt<WF_F16>(a, p, tA, tA2, tW, tS, tMin, tX, s);
    case WF_Q8: return launch_fmt<WF_Q8>(a, p, tA, tA2, tW, tS, tMin, tX, s);
    case WF_Q4: return launch_fmt<WF_Q4>(a, p, tA, tA2, tW, tS, tMin, tX, s);
    case WF_Q4A: return launch_fmt<WF_Q4A>(a, p, tA, tA2, tW, tS, tMin, tX, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace hx

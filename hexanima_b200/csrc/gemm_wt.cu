// q8 GEMM with the dequantised weights held in tensor memory.
//
// The same operation as the q8 path of gemm.cu (O = A * W^T, W int8 in K-groups with fp16 scales;
// the reference's gemm_run_geo with dq_tile, hexagon/mega/gemm2.c:20-35 and :96-137) and the same
// epilogues (job_fn flushes, gemm2.c:58-82), with the operand roles swapped at the tensor core:
// D^T = W * A^T. The weight rows are the MMA's M side: each dequantiser thread turns one weight row
// of a k-block from int8 into fp16 in registers and writes it into TMEM with tcgen05.st, and
// tcgen05.mma reads that A operand from TMEM. The tokens are the N side, fed from shared memory by
// TMA. Per CTA and k-block, shared memory then carries the token tile (TMA write, MMA read) and the
// raw int8 tile (TMA write, dequantiser read), but no fp16 weight tile.
//
// CTA pair (cluster of 2, tcgen05.mma.cta_group::2) per output tile of 256 weight rows x 256 tokens:
// each CTA dequantises 128 weight rows (its TMEM lanes) and loads 128 tokens; each CTA's D is its 128
// weight rows x all 256 tokens in fp32. (N = 256 per MMA: 192- and 224-token tiles, which would let
// two whole accumulators fit beside the weight slots, ran the tensor pipe 15-20 % slower.)
// TMEM columns: [0,128) four dequantised k-blocks of 64 k (32 columns each); tile i's accumulator at
// columns [128,384) for even i and [256,512) for odd i. Consecutive tiles share columns [256,384):
// the epilogue reads that half first (into registers) and releases it, so the next tile's MMAs run
// while the epilogue works through the rest.
// 14 warps per CTA:
//   warp  0     TMEM allocator + tcgen05.mma issuer (leader CTA)
//   warp  1     TMA producer (token tile, raw weight tile, scales)
//   warps 2-5   dequantisers: warp w writes TMEM lanes 32(w%4).., one weight row of a k-block per thread
//   warps 6-13  epilogue: warp w takes TMEM lanes 32(w%4).. (32 output columns) x 64 tokens of each
//               accumulator half ((w-6)/4 picks which 64), 32 tokens at a time, and writes them
//               transposed into its own shared-memory box, which one TMA store (fp16 out) or TMA
//               reduce-add (fp32 residual) moves to global memory
#include <cudaTypedefs.h>

#include "hx_internal.h"
#include "hx_gelu.cuh"
#include "hx_ptx.cuh"

namespace hx {

bool make_tmap_2d(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* base, uint64_t inner,
                  uint64_t outer, uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_outer,
                  CUtensorMapSwizzle sw);

namespace {

constexpr int WT_ROWS = 128;         // weight rows per CTA = TMEM lanes
constexpr int WT_TOK = 256;          // tokens per pair tile (MMA N)
constexpr int WT_HTOK = WT_TOK / 2;  // tokens loaded per CTA
constexpr int WT_BK = 64;
constexpr int WT_TA = 4;             // dequantised k-blocks resident in TMEM, columns [0, 128)
constexpr uint32_t WT_D0 = 128;      // accumulator of even tiles: [128, 384); odd tiles: [256, 512)
constexpr uint32_t WT_HOT = 256;     // the columns [256, 384) both accumulators use
// the producers take the lowest warp ids (MMA issuer, TMA, dequantisers), the epilogue the highest
constexpr int MMA_WARP = 0, TMA_WARP = 1, DQ_WARP0 = 2, DQ_WARPS = 4, EPI_WARP0 = 6, EPI_WARPS = 8;
constexpr int WT_THREADS = (EPI_WARP0 + EPI_WARPS) * 32;
constexpr int X_B = WT_HTOK * WT_BK * 2;  // 16 KB token tile (SW128, K-major)
constexpr int RAW_B = WT_ROWS * WT_BK;    // 8 KB int8 tile (SW64: 64-byte rows)
constexpr int SC_B = 1024;                // scales of the k-block: [64/group][128] fp16, padded
constexpr int STAGE_B = X_B + RAW_B + SC_B;

template <int EPI>
struct WtCfg {
  // per epilogue warp and buffer: 32 tokens x 32 columns, fp32 for the residual, else fp16
  static constexpr int BOX = EPI == EPI_RESID ? 4096 : 2048;
  static constexpr int S = EPI == EPI_STORE || EPI == EPI_GELU ? 7 : 6;
  static constexpr int OUT = EPI_WARPS * 2 * BOX;
  static constexpr int RED = EPI == EPI_RMS ? 2 * 2 * 128 * 4 : 0;       // [sub][buf][128]
  static constexpr int XCH = EPI == EPI_RMS ? 2 * 4 * 32 * 32 * 4 : 0;  // [sub][quarter][32 x 32]
  static constexpr int SMEM = S * STAGE_B + OUT + RED + XCH + 1024 /*barriers*/ + 1024 /*alignment slack*/;
};

struct WtParams {
  int M, N, nkb, nkb1, group;
  int num_m_tiles, num_n_tiles, num_tiles, n_fastest;  // m: token tiles of 256, n: weight tiles of 256
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

__device__ __forceinline__ int wt_tile_m(const WtParams& p, int t) {
  return p.n_fastest ? t / p.num_n_tiles : t % p.num_m_tiles;
}
__device__ __forceinline__ int wt_tile_n(const WtParams& p, int t) {
  return p.n_fastest ? t % p.num_n_tiles : t / p.num_m_tiles;
}

__device__ __forceinline__ void spin_ns(uint64_t ns) {
  const uint64_t t0 = globaltimer();
  while (globaltimer() - t0 < ns) {
  }
}

// a bounded wait whose outcome is the same in all lanes (warp-collective tcgen05 ops follow)
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, status, code));
}


// Column sums of a 32 x 32 block held one row per lane: returns, in lane l, the sum over the 32 lanes
// of x[l] (five butterfly steps, each halving the columns a lane carries).
__device__ __forceinline__ float transpose_sum32(const float (&x)[32], int lane) {
  float y16[16], y8[8], y4[4], y2[2];
  const bool b16 = lane & 16, b8 = lane & 8, b4 = lane & 4, b2 = lane & 2, b1 = lane & 1;
#pragma unroll
  for (int i = 0; i < 16; ++i)
    y16[i] = (b16 ? x[16 + i] : x[i]) + __shfl_xor_sync(0xffffffffu, b16 ? x[i] : x[16 + i], 16);
#pragma unroll
  for (int i = 0; i < 8; ++i)
    y8[i] = (b8 ? y16[8 + i] : y16[i]) + __shfl_xor_sync(0xffffffffu, b8 ? y16[i] : y16[8 + i], 8);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    y4[i] = (b4 ? y8[4 + i] : y8[i]) + __shfl_xor_sync(0xffffffffu, b4 ? y8[i] : y8[4 + i], 4);
#pragma unroll
  for (int i = 0; i < 2; ++i)
    y2[i] = (b2 ? y4[2 + i] : y4[i]) + __shfl_xor_sync(0xffffffffu, b2 ? y4[i] : y4[2 + i], 2);
  return (b1 ? y2[1] : y2[0]) + __shfl_xor_sync(0xffffffffu, b1 ? y2[0] : y2[1], 1);
}

// fp16 box of 32 tokens x 32 columns (64-byte rows, 64-byte swizzle) -> TMA store at (col0, tok0)
template <bool EVICT_FIRST>
__device__ __forceinline__ void store_box_f16(const CUtensorMap* tmO, uint8_t* box, const float (&v)[32], int lane,
                                              int col0, int tok0) {
  const uint32_t b = smem_u32(box);
#pragma unroll
  for (int t = 0; t < 32; ++t)
    st_shared_b16(b + t * 64 + ((((lane >> 3) ^ ((t >> 1) & 3))) << 4) + (lane & 7) * 2,
                  __half_as_ushort(__float2half_rn(v[t])));
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if constexpr (EVICT_FIRST) tma_store_2d_evict_first(tmO, box, col0, tok0);
    else tma_store_2d(tmO, box, col0, tok0);
    bulk_commit();
  }
}

// What an epilogue warp knows about its columns of the current tile.
struct EpiCols {
  int col0;           // this warp's 32 output columns
  int d;              // this lane's column within the CTA's 128 (RMS: within the head)
  const float* gain;  // RMS segment of the CTA's head (nullptr: plain columns)
  float gd;           // gain[d]
  int rope;
};

// One chunk: this warp's 32 columns x 32 tokens from tok0, v[token] = fp32 sums of this lane's column.
// For RMS the 4 warps of a sub-group (lane quarters 0-3, the same tokens) meet at named barrier 1+sub.
template <int EPI>
__device__ __forceinline__ void epi_chunk(const WtParams& p, const CUtensorMap* tmO, float (&v)[32], int tok0,
                                          const EpiCols& e, uint8_t* box, float* red, float* xch, int q, int lane,
                                          int sub, int& gate_img, float& gate_c) {
  if (lane == 0) bulk_wait_read<1>();  // the copy out of this buffer two boxes ago has read it
  __syncwarp();
  if constexpr (EPI == EPI_RESID) {
    // x += gate[image] * acc, reduce-added by TMA (the SM never reads x)
    // rows_per_img >= 32 (checked on the host): a chunk spans at most two images
    const int img0 = tok0 / p.rows_per_img;
    if (img0 != gate_img) {
      gate_c = p.gate[img0 * p.vec_bstride + e.col0 + lane];
      gate_img = img0;
    }
    const int split = (img0 + 1) * p.rows_per_img - tok0;  // tokens i >= split are in image img0 + 1
    if (split >= 32) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] *= gate_c;
    } else {
      const float g1 = p.gate[(img0 + 1) * p.vec_bstride + e.col0 + lane];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] *= i < split ? gate_c : g1;
    }
    const uint32_t b = smem_u32(box);
#pragma unroll
    for (int i = 0; i < 32; ++i)
      st_shared_b32(b + i * 128 + ((((lane >> 2) ^ (i & 7))) << 4) + (lane & 3) * 4, __float_as_uint(v[i]));
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_reduce_add_2d(tmO, box, e.col0, tok0);
      bulk_commit();
    }
  } else if constexpr (EPI == EPI_GELU) {
    gelu32(v);
    store_box_f16<true>(tmO, box, v, lane, e.col0, tok0);  // the mlp hidden stream is larger than L2
  } else if constexpr (EPI == EPI_STORE) {
    store_box_f16<false>(tmO, box, v, lane, e.col0, tok0);
  } else if constexpr (EPI == EPI_RMS) {
    if (e.gain) {
      // per-token sum of squares over the head's 128 columns: this warp's 32 by a butterfly, then
      // the sub-group's 4 partial sums through shared memory (red is double-buffered by the caller)
      float sq[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) sq[i] = v[i] * v[i];
      red[q * 32 + lane] = transpose_sum32(sq, lane);  // token tok0 + lane
      named_bar(1 + sub, 128);
      const float ss = (red[lane] + red[32 + lane]) + (red[64 + lane] + red[96 + lane]);
      const float rs = rsqrtf(ss * (1.0f / 128.0f) + p.eps);
      const float gd = e.gd;
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = v[i] * __shfl_sync(0xffffffffu, rs, i) * gd;
      if (e.rope) {
        // pairs (d, d + 64) are lane quarters q and q ^ 2. One buffer: a warp writes it for the next
        // chunk only after the next chunk's first barrier, which every warp reaches after reading.
#pragma unroll
        for (int i = 0; i < 32; ++i) xch[q * 1024 + i * 32 + lane] = v[i];
        named_bar(1 + sub, 128);
        const float* pb = xch + (q ^ 2) * 1024;
        const int dd = e.d & 63;
        // table row of token min(tok0 + i, M - 1) within its image, stepped instead of divided
        int r = min(tok0, p.M - 1) % p.rows_per_img;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float co = p.cosT[static_cast<size_t>(r) * 64 + dd];
          const float si = p.sinT[static_cast<size_t>(r) * 64 + dd];
          const float o = pb[i * 32 + lane];
          v[i] = q < 2 ? v[i] * co - o * si : v[i] * co + o * si;
          if (tok0 + i + 1 < p.M) r = r + 1 == p.rows_per_img ? 0 : r + 1;
        }
      }
    }
    store_box_f16<false>(tmO, box, v, lane, e.col0, tok0);
  }
}

__device__ __forceinline__ void regs_to_f32(const uint32_t (&r)[32], float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

template <int EPI>
__global__ void __launch_bounds__(WT_THREADS, 1)
    gemm_wt_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                   const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmS,
                   const __grid_constant__ CUtensorMap tmO, const WtParams p) {
  using C = WtCfg<EPI>;
  constexpr int S = C::S;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* outbox = smem + S * STAGE_B;
  float* red_all = reinterpret_cast<float*>(outbox + C::OUT);
  float* xch_all = reinterpret_cast<float*>(outbox + C::OUT + C::RED);
  uint64_t* bars = reinterpret_cast<uint64_t*>(outbox + C::OUT + C::RED + C::XCH);
  uint64_t* full_x = bars;             // [S] leader: the pair's token tiles landed
  uint64_t* raw_full = bars + S;       // [S] local: raw weights and scales landed
  uint64_t* empty = bars + 2 * S;      // [S] each CTA: the stage's MMAs completed (commit multicast)
  uint64_t* dq_full = bars + 3 * S;    // [TA] leader: the 8 dequantiser warps of the pair wrote the slot
  uint64_t* a_free = dq_full + WT_TA;  // [TA] each CTA: the MMAs reading the slot completed
  uint64_t* tfull = a_free + WT_TA;    // [tile parity] each CTA: accumulator complete
  uint64_t* hot_free = tfull + 2;      // [tile parity] leader: the 16 epilogue warps read columns [256,384)
  uint64_t* drain = hot_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  auto st_x = [&](int s) { return smem + s * STAGE_B; };
  auto st_raw = [&](int s) { return smem + s * STAGE_B + X_B; };
  auto st_sc = [&](int s) { return smem + s * STAGE_B + X_B + RAW_B; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_x[i], 1);
      mbar_init(&raw_full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < WT_TA; ++i) {
      mbar_init(&dq_full[i], 2 * DQ_WARPS);
      mbar_init(&a_free[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&hot_free[i], 2 * EPI_WARPS);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  if (warp == TMA_WARP && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmS);
    prefetch_tmap(&tmO);
    if (p.nkb1 < p.nkb) prefetch_tmap(&tmA2);
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM of the pair allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int ntiles_mine = p.num_tiles > pair ? (p.num_tiles - 1 - pair) / npairs + 1 : 0;
  // The raw weight tiles and scales are constant during inference (no kernel that can precede this one
  // with programmatic dependent launch writes them), so the producer loads the first ring of them before
  // waiting for the previous kernel; everything else waits first.
  const bool early_weights = warp == TMA_WARP && lane == 0;
  const int npre = ntiles_mine > 0 ? (p.nkb < S ? p.nkb : S) : 0;
  if (early_weights && npre > 0) {
    const uint32_t sc_rows = WT_BK / p.group;
    const uint32_t raw_tx = RAW_B + sc_rows * WT_ROWS * 2;
    const int w0 = wt_tile_n(p, pair) * 2 * WT_ROWS + static_cast<int>(rank) * WT_ROWS;
    for (int kb = 0; kb < npre; ++kb) {  // stages kb are empty on the first pass
      mbar_arrive_expect_tx(&raw_full[kb], raw_tx);
      tma_load_2d(st_raw(kb), &tmW, &raw_full[kb], kb * WT_BK, w0);
      tma_load_2d(st_sc(kb), &tmS, &raw_full[kb], w0, kb * static_cast<int>(sc_rows));
    }
  }
  grid_dep_wait();  // the previous kernel's outputs (the token rows) are complete
  grid_dep_launch();

  if (warp == TMA_WARP) {
    if (lane == 0) {
      const uint32_t sc_rows = WT_BK / p.group;
      const uint32_t raw_tx = RAW_B + sc_rows * WT_ROWS * 2;
      int it = 0;
      bool ok = true;
      for (int ti = 0; ti < ntiles_mine && ok; ++ti) {
        const int t = pair + ti * npairs;
        const int tok0 = wt_tile_m(p, t) * WT_TOK + static_cast<int>(rank) * WT_HTOK;
        const int w0 = wt_tile_n(p, t) * 2 * WT_ROWS + static_cast<int>(rank) * WT_ROWS;
        for (int kb = 0; kb < p.nkb; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, p.status, 131)) { ok = false; break; }
          if (leader) mbar_arrive_expect_tx(&full_x[s], 2u * X_B);
          if (kb < p.nkb1) tma_load_2d_pair(st_x(s), &tmA, &full_x[s], kb * WT_BK, tok0);
          else tma_load_2d_pair(st_x(s), &tmA2, &full_x[s], (kb - p.nkb1) * WT_BK, tok0);
          if (it < npre) continue;  // loaded before the dependency wait
          mbar_arrive_expect_tx(&raw_full[s], raw_tx);
          tma_load_2d(st_raw(s), &tmW, &raw_full[s], kb * WT_BK, w0);
          tma_load_2d(st_sc(s), &tmS, &raw_full[s], w0, kb * static_cast<int>(sc_rows));
        }
      }
      if (!ok) spin_ns(2000000);  // loads issued before the abort land long before this
    }
  } else if (warp == MMA_WARP) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = idesc_f16(2 * WT_ROWS, WT_TOK, 0, 0);
      int it = 0;
      bool ok = true, issued = false;
      for (int ti = 0; ti < ntiles_mine && ok; ++ti) {
        // columns [256,384) were the previous tile's: its epilogue has read them, and before that all
        // of the tile before it, whose columns this tile's other half reuses
        if (ti > 0 && !mbar_wait(&hot_free[(ti - 1) & 1], ((ti - 1) >> 1) & 1, p.status, 132)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t dt = tmem + WT_D0 + (ti & 1) * 128;
        for (int kb = 0; kb < p.nkb; ++kb, ++it) {
          const int s = it % S, a = it % WT_TA;
          if (!mbar_wait(&full_x[s], (it / S) & 1, p.status, 133)) { ok = false; break; }
          if (!mbar_wait(&dq_full[a], (it / WT_TA) & 1, p.status, 134)) { ok = false; break; }
          tc_fence_after();
          const uint32_t x0 = smem_u32(st_x(s)), ta = tmem + 32 * a;
#pragma unroll
          for (int k = 0; k < WT_BK / 16; ++k)
            mma_f16_ts_pair(dt, ta + 8 * k, sdesc_sw128(x0 + 32 * k, 16, 1024), idesc, (kb | k) != 0);
          issued = true;
          mma_commit_pair_mc(&empty[s], 0x3);
          mma_commit_pair_mc(&a_free[a], 0x3);
        }
        if (!ok) break;
        mma_commit_pair_mc(&tfull[ti & 1], 0x3);
      }
      if (!ok && issued) {
        mma_commit_pair(drain);
        mbar_wait(drain, 0, nullptr, 0);
      }
    }
  } else if (warp < EPI_WARP0) {
    // weight row `row` of this CTA's 128, all 64 k of each k-block
    const int quarter = warp & 3;
    const int row = 32 * quarter + lane;
    const uint32_t tl = tmem + (static_cast<uint32_t>(32 * quarter) << 16);
    const uint32_t swz = (row >> 1) & 3;  // 64-byte swizzle of the raw tile: chunk c sits at c ^ swz
    const __half2 off = __half2half2(__ushort_as_half(0x6480));  // 1152 = 1024 + the offset 128
    int it = 0;
    bool ok = true;
    for (int ti = 0; ti < ntiles_mine && ok; ++ti) {
      for (int kb = 0; kb < p.nkb; ++kb, ++it) {
        const int s = it % S, a = it % WT_TA;
        if (!warp_wait(&raw_full[s], (it / S) & 1, p.status, 135)) { ok = false; break; }
        if (!warp_wait(&a_free[a], ((it / WT_TA) & 1) ^ 1, p.status, 136)) { ok = false; break; }
        tc_fence_after();
        const uint32_t rb = smem_u32(st_raw(s)) + row * 64;
        const __half* sc = reinterpret_cast<const __half*>(st_sc(s));
        uint32_t o[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 v = ld_shared_v4(rb + ((c ^ swz) << 4));
          const __half2 s2 = __half2half2(sc[(p.group == 64 ? 0 : (c >> 1)) * WT_ROWS + row]);
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            // bytes k, k+1 -> fp16 1024 + u in the two halves of one column; then (u - 128) * s
            uint32_t lo = __byte_perm(w[j], 0x64646464u, 0x4140);
            uint32_t hi = __byte_perm(w[j], 0x64646464u, 0x4342);
            __half2 x = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&lo), off), s2);
            __half2 y = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&hi), off), s2);
            o[8 * c + 2 * j] = *reinterpret_cast<uint32_t*>(&x);
            o[8 * c + 2 * j + 1] = *reinterpret_cast<uint32_t*>(&y);
          }
        }
        tmem_st32(tl + 32 * a, o);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_leader(&dq_full[a]);
      }
    }
  } else {
    // epilogue warp: lane quarter q (output columns), sub-group `sub` (which 64 tokens of each half)
    const int q = warp & 3, sub = (warp - EPI_WARP0) >> 2;
    const uint32_t tlane = static_cast<uint32_t>(32 * q) << 16;
    uint8_t* mybox = outbox + (warp - EPI_WARP0) * 2 * C::BOX;
    float* red = red_all + sub * 256;
    float* xch = xch_all + sub * 4096;
    int nbox = 0;  // boxes written by this warp: alternates the two buffers
    int gate_img = -1;
    float gate_c = 0.f;
    bool ok = true;
    for (int ti = 0; ti < ntiles_mine && ok; ++ti) {
      const int t = pair + ti * npairs;
      const int tok_base = wt_tile_m(p, t) * WT_TOK;
      const int head0 = wt_tile_n(p, t) * 2 * WT_ROWS + static_cast<int>(rank) * WT_ROWS;  // this CTA's 128
      EpiCols e;
      e.col0 = head0 + 32 * q;
      e.d = 32 * q + lane;
      e.gain = nullptr;
      e.gd = 1.f;
      e.rope = 0;
      if constexpr (EPI == EPI_RMS) {  // the CTA's 128 columns are one head
        if (head0 < p.seg1) {
          e.gain = p.gain0;
          e.rope = p.rope0;
        } else if (head0 < p.seg2) {
          e.gain = p.gain1;
          e.rope = p.rope1;
        }
        if (e.gain) e.gd = e.gain[e.d];
      }
      const int par = ti & 1;
      // the sub-group's 4 warps meet at named barrier 1 + sub: they leave together or not at all
      if (!bar_and(3 + sub, 128, warp_wait(&tfull[par], (ti >> 1) & 1, p.status, 137))) {
        ok = false;
        break;
      }
      tc_fence_after();
      // the shared columns [256,384) hold tokens [128,256) of an even tile, [0,128) of an odd one
      const int hot_tok = tok_base + (par ? 0 : 128) + 64 * sub;
      const int cold_tok = tok_base + (par ? 128 : 0) + 64 * sub;
      const uint32_t cold_col = par ? 384u : 128u;
      uint32_t h0[32], h1[32];
      tmem_ld32(tmem + tlane + WT_HOT + 64 * sub, h0);
      tmem_ld32(tmem + tlane + WT_HOT + 64 * sub + 32, h1);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_leader(&hot_free[par]);
      float v[32];
#pragma unroll  // unrolled so that the registers of h0 / h1 are free once their chunk is done
      for (int c = 0; c < 4; ++c) {
        const int tok0 = (c < 2 ? hot_tok : cold_tok) + 32 * (c & 1);
        if (c == 0) {
          regs_to_f32(h0, v);
        } else if (c == 1) {
          regs_to_f32(h1, v);
        } else {
          uint32_t r[32];
          tmem_ld32(tmem + tlane + cold_col + 64 * sub + 32 * (c & 1), r);
          tmem_ld_wait();
          regs_to_f32(r, v);
        }
        if (tok0 >= p.M) continue;  // uniform over the sub-group
        const int buf = nbox & 1;   // alternates on every box, across tiles too
        ++nbox;
        epi_chunk<EPI>(p, &tmO, v, tok0, e, mybox + buf * C::BOX, red + buf * 128, xch, q, lane, sub, gate_img,
                       gate_c);
      }
    }
    if (lane == 0) bulk_wait<0>();  // this warp's stores and reduce-adds are complete
  }

  tc_fence_before();
  cluster_sync();  // the pair's MMAs and epilogues are done before either CTA frees TMEM
  tc_fence_after();
  if (warp == MMA_WARP) tmem_dealloc_pair(tmem, 512);
}

template <int EPI>
cudaError_t launch_wt(const WtParams& p, const CUtensorMap& tA, const CUtensorMap& tA2, const CUtensorMap& tW,
                      const CUtensorMap& tS, const CUtensorMap& tO, int npairs, cudaStream_t s) {
  using C = WtCfg<EPI>;
  static uint64_t attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set >> dev & 1)) {
    cudaError_t e = cudaFuncSetAttribute(gemm_wt_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    attr_set |= 1ull << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * npairs);
  cfg.blockDim = dim3(WT_THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_attr(attr, 1);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_wt_kernel<EPI>, tA, tA2, tW, tS, tO, p);
  if (e != cudaSuccess) cudaGetLastError();  // a refused launch leaves no error for the next caller
  return e;
}

}  // namespace

bool gemm_wt_eligible(const GemmArgs& a) {
  const DevMat* W = a.W;
  if (!W || W->fmt != WF_Q8 || (W->group != 32 && W->group != 64)) return false;
  if (a.epi != EPI_STORE && a.epi != EPI_GELU && a.epi != EPI_RESID && a.epi != EPI_RMS) return false;
  if (W->N % (2 * WT_ROWS) || W->K % WT_BK || a.K1 % WT_BK) return false;
  if (a.epi == EPI_RMS && ((a.seg1 % WT_ROWS) || (a.seg2 % WT_ROWS))) return false;
  if (a.epi == EPI_RESID && (a.ldx % 4 || a.rows_per_img < 32)) return false;
  if (a.epi != EPI_RESID && a.ldo % 8) return false;
  return true;
}

// the number of pair tiles of this kernel for the GEMM (used to pick it only when it fills the GPU)
int gemm_wt_tiles(const GemmArgs& a) {
  return ((a.M + WT_TOK - 1) / WT_TOK) * (a.W->N / (2 * WT_ROWS));
}

cudaError_t gemm_wt_launch(const GemmArgs& a, cudaStream_t s) {
  if (!gemm_wt_eligible(a)) return cudaErrorInvalidValue;
  const DevMat* W = a.W;
  const int N = W->N, K = W->K;
  CUtensorMap tA, tA2, tW, tS, tO;
  memset(&tA2, 0, sizeof tA2);
  if (!make_tmap_2d(&tA, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.A, a.K1, a.M, static_cast<uint64_t>(a.lda) * 2, WT_BK,
                    WT_HTOK, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (a.K1 < K && !make_tmap_2d(&tA2, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.A2, K - a.K1, a.M,
                                static_cast<uint64_t>(a.lda2) * 2, WT_BK, WT_HTOK, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (!make_tmap_2d(&tW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, W->w, K, N, K, WT_BK, WT_ROWS, CU_TENSOR_MAP_SWIZZLE_64B))
    return cudaErrorInvalidValue;
  if (!make_tmap_2d(&tS, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, W->scale, N, K / W->group, static_cast<uint64_t>(N) * 2,
                    WT_ROWS, WT_BK / W->group, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  if (a.epi == EPI_RESID) {
    if (!make_tmap_2d(&tO, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a.x, N, a.M, static_cast<uint64_t>(a.ldx) * 4, 32, 32,
                      CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  } else if (!make_tmap_2d(&tO, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.out, N, a.M, static_cast<uint64_t>(a.ldo) * 2,
                           32, 32, CU_TENSOR_MAP_SWIZZLE_64B)) {
    return cudaErrorInvalidValue;
  }
  WtParams p;
  p.M = a.M;
  p.N = N;
  p.nkb = K / WT_BK;
  p.nkb1 = a.K1 / WT_BK;
  p.group = W->group;
  p.num_m_tiles = (a.M + WT_TOK - 1) / WT_TOK;
  p.num_n_tiles = N / (2 * WT_ROWS);
  p.num_tiles = p.num_m_tiles * p.num_n_tiles;
  {
    // as in gemm.cu: walk the weight tiles of one token block when the token operand is far larger
    // than L2 and the weights fit
    const double a_bytes = static_cast<double>(a.M) * K * 2, w_bytes = static_cast<double>(N) * K;
    p.n_fastest = a_bytes > 64e6 && w_bytes < 64e6 ? 1 : 0;
  }
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
  int npairs = sm_count() / 2;
  if (a.max_ctas > 0 && a.max_ctas / 2 < npairs) npairs = a.max_ctas / 2 > 0 ? a.max_ctas / 2 : 1;
  if (p.num_tiles < npairs) npairs = p.num_tiles;
  switch (a.epi) {
    case EPI_STORE: return launch_wt<EPI_STORE>(p, tA, tA2, tW, tS, tO, npairs, s);
    case EPI_GELU: return launch_wt<EPI_GELU>(p, tA, tA2, tW, tS, tO, npairs, s);
    case EPI_RESID: return launch_wt<EPI_RESID>(p, tA, tA2, tW, tS, tO, npairs, s);
    case EPI_RMS: return launch_wt<EPI_RMS>(p, tA, tA2, tW, tS, tO, npairs, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace hx

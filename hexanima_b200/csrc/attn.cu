// Flash-style attention on tcgen05 tensor cores, head_dim 128, online softmax.
//
// Replaces attn_run (hexagon/mega/blk.c:54-91; masked joint version moss/hexagon/mega/blk.c:54-94)
// with its table softmax k_softmax2p (hexagon/mega/kern.c:261-282; moss kern.c:262-285) and row
// normalisation k_rowscale_sum (kern.c:285-295): o = softmax(q k^T * scale) v per head. Keys at
// index >= nvalid get probability 0 (the reference masks the last key tile to -65504).
// The reference folds 1/sqrt(128) into the q RMS gain (export_all.py:31-32), so scale = 1 there.
//
// One CTA per (128 queries, head, image). 10 warps:
//   warps 0-7  softmax + output: warp w owns query rows 32(w%4)..+31 (its TMEM lane quarter) and
//              half w/4 of each tile: keys 64(w/4)..+63 of S and output dims 64(w/4)..+63
//   warp  8    TMA producer (Q once, then K and V tiles of 128 keys in 3-stage rings)
//   warp  9    TMEM allocator + tcgen05.mma issuer
// The two halves of a row exchange their partial row maxima through shared memory each tile and
// their partial row sums once at the end.
// TMEM columns: S [0,128) fp32; P double buffer [128,192) [192,256), fp16 packed two per column;
// P.V partials double buffer [256,384) [384,512).
// S = Q K^T (both K-major, from shared memory); O_part = P V with P read from TMEM and V MN-major
// straight from its row-major tile. The running output stays in registers:
// o = o * exp2(m_old - m_new) + O_part.
#include <cmath>
#include <cstring>

#include "hx_internal.h"
#include "hx_ptx.cuh"

namespace hx {

bool make_tmap_3d(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* base, uint64_t d0, uint64_t d1,
                  uint64_t d2, uint64_t pitch1, uint64_t pitch2, uint32_t b0, uint32_t b1, uint32_t b2,
                  CUtensorMapSwizzle sw);

namespace {

constexpr int QT = 128, KT = 128, HD = 128;
constexpr int SM_WARPS = 8;  // softmax warps
constexpr int TMA_WARP = SM_WARPS, MMA_WARP = SM_WARPS + 1;
constexpr int ATT_THREADS = (SM_WARPS + 2) * 32;
constexpr int KV_STAGES = 3;
constexpr int TILE_BYTES = 128 * 128 * 2;  // 32 KB: two 64-column swizzled halves
// small region first (barriers, TMEM slot, max/sum exchange), then the 1024-aligned tiles:
// Q | K0 V0 | K1 V1 | K2 V2
constexpr int SMALL_BYTES = 2560;
constexpr int SM_XCH = 512;  // float [2 parities][2 halves][128 rows]
constexpr int TILES_BYTES = TILE_BYTES * (1 + 2 * KV_STAGES);
// the CTA's dynamic shared memory starts 1024-aligned after the 1 KB the driver reserves, so the tiles
// begin at offset 3072 and end exactly at the 232448-byte opt-in limit; the kernel checks this.
constexpr int ATT_SMEM = 3072 + TILES_BYTES;
constexpr uint32_t TM_S = 0, TM_P = 128, TM_O = 256;

// one MUFU op: 2^x (flush-to-zero; the inputs here are <= 0 and the results feed fp16 probabilities)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct AParams {
  int Tq, Tk, nvalid, H, nkt;
  float scale_log2;
  __half* o;
  int ldo;
  int* status;
};

// packed fp32 pairs (sm_100 f32x2 arithmetic: two lanes per instruction, each rounded like the scalar op)
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// three-input maximum (sm_100); like fmaxf, a NaN operand is ignored
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// max over 32 raw scores at keys kbase..kbase+31 into 8 partial maxima (keys >= limit skipped)
template <bool FULL>
__device__ __forceinline__ void max32(float (&mxp)[8], const uint32_t (&r)[32], int kbase, int limit) {
  if constexpr (FULL) {
#pragma unroll
    for (int t = 0; t < 32; t += 2)
      mxp[(t >> 1) & 7] = fmax3(mxp[(t >> 1) & 7], __uint_as_float(r[t]), __uint_as_float(r[t + 1]));
  } else {
#pragma unroll
    for (int t = 0; t < 32; ++t)
      if (kbase + t < limit) mxp[t & 7] = fmaxf(mxp[t & 7], __uint_as_float(r[t]));
  }
}

// p = 2^(s*scale_log2 - m) for 32 scores, fp16-packed into pk, pairwise partial sums into sum2
template <bool FULL>
__device__ __forceinline__ void exp32(uint32_t (&pk)[16], uint64_t (&sum2)[4], const uint32_t (&r)[32],
                                      uint64_t scale2, uint64_t negm2, int kbase, int limit) {
#pragma unroll
  for (int t = 0; t < 32; t += 2) {
    float x0, x1;
    f2unpack(ffma2(f2pack(__uint_as_float(r[t]), __uint_as_float(r[t + 1])), scale2, negm2), x0, x1);
    float e0 = ex2(x0), e1 = ex2(x1);
    if constexpr (!FULL) {
      if (kbase + t >= limit) e0 = 0.f;
      if (kbase + t + 1 >= limit) e1 = 0.f;
    }
    sum2[(t >> 1) & 3] = fadd2(sum2[(t >> 1) & 3], f2pack(e0, e1));
    pk[t / 2] = pack_half2(e0, e1);
  }
}

__global__ void __launch_bounds__(ATT_THREADS, 1)
    attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const AParams p, int q_col0, int k_col0, int v_col0) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* tiles =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + SMALL_BYTES + 1023) & ~uintptr_t(1023));
  if (tiles + TILES_BYTES > smem_raw + ATT_SMEM) {  // uniform over the CTA: nothing has started yet
    if (threadIdx.x == 0 && p.status) atomicCAS(p.status, 0, 220);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;    // [3]
  uint64_t* k_empty = bars + 4;   // [3]
  uint64_t* v_full = bars + 7;    // [3]
  uint64_t* v_empty = bars + 10;  // [3]
  uint64_t* s_full = bars + 13;
  uint64_t* s_empty = bars + 14;
  uint64_t* p_full = bars + 15;   // [2]
  uint64_t* p_empty = bars + 17;  // [2]
  uint64_t* o_full = bars + 19;   // [2]
  uint64_t* o_empty = bars + 21;  // [2]
  uint64_t* xbar = bars + 23;     // [2 parities][4 row groups]
  uint64_t* drain = bars + 31;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 32);
  float* xch = reinterpret_cast<float*>(smem_raw + SM_XCH);
  uint8_t* sQ = tiles;
  uint8_t* sK = tiles + TILE_BYTES;  // stage s: K at sK + 2s*TILE, V right after it

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int nkt = p.nkt;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < KV_STAGES; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, SM_WARPS);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], SM_WARPS);
      mbar_init(&p_empty[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], SM_WARPS);
    }
    for (int i = 0; i < 8; ++i) mbar_init(&xbar[i], 2);  // the two warps of a row group
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == TMA_WARP) {
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      const int qc = q_col0 + h * HD, kc = k_col0 + h * HD, vc = v_col0 + h * HD;
      mbar_arrive_expect_tx(q_full, TILE_BYTES);
      tma_load_3d(sQ, &tmQ, q_full, qc, qt * QT, b);
      tma_load_3d(sQ + TILE_BYTES / 2, &tmQ, q_full, qc + 64, qt * QT, b);
      int nk = 0, nv = 0;  // K and V tiles issued
      for (int j = 0; j < nkt; ++j) {
        const int st = j % KV_STAGES, ph = (j / KV_STAGES) & 1;
        uint8_t* kbuf = sK + st * 2 * TILE_BYTES;
        if (!mbar_wait(&k_empty[st], ph ^ 1, p.status, 201)) break;
        mbar_arrive_expect_tx(&k_full[st], TILE_BYTES);
        tma_load_3d(kbuf, &tmK, &k_full[st], kc, j * KT, b);
        tma_load_3d(kbuf + TILE_BYTES / 2, &tmK, &k_full[st], kc + 64, j * KT, b);
        ++nk;
        if (!mbar_wait(&v_empty[st], ph ^ 1, p.status, 211)) break;
        mbar_arrive_expect_tx(&v_full[st], TILE_BYTES);
        tma_load_3d(kbuf + TILE_BYTES, &tmV, &v_full[st], vc, j * KT, b);
        tma_load_3d(kbuf + TILE_BYTES + TILE_BYTES / 2, &tmV, &v_full[st], vc + 64, j * KT, b);
        ++nv;
      }
      if (nv < nkt) {  // aborted: let the copies in flight land before the CTA exits
        mbar_wait(q_full, 0, nullptr, 0);
        for (int i = (nk > KV_STAGES ? nk - KV_STAGES : 0); i < nk; ++i)
          mbar_wait(&k_full[i % KV_STAGES], (i / KV_STAGES) & 1, nullptr, 0);
        for (int i = (nv > KV_STAGES ? nv - KV_STAGES : 0); i < nv; ++i)
          mbar_wait(&v_full[i % KV_STAGES], (i / KV_STAGES) & 1, nullptr, 0);
      }
    }
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_f16(QT, KT, 0, 0);  // S = Q K^T, both K-major
      constexpr uint32_t id_o = idesc_f16(QT, HD, 0, 1);  // O = P V, P K-major in TMEM, V MN-major
      const uint32_t q0 = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, p.status, 202);
      bool issued = false;
      auto issue_pv = [&](int i) -> bool {
        const int st = i % KV_STAGES, pb = i & 1;
        if (!mbar_wait(&v_full[st], (i / KV_STAGES) & 1, p.status, 212)) return false;
        if (!mbar_wait(&p_full[pb], (i >> 1) & 1, p.status, 203)) return false;
        if (!mbar_wait(&o_empty[pb], ((i >> 1) & 1) ^ 1, p.status, 204)) return false;
        tc_fence_after();
        const uint32_t vb = smem_u32(sK + st * 2 * TILE_BYTES + TILE_BYTES);
#pragma unroll
        for (int k = 0; k < KT / 16; ++k) {
          const uint64_t bd = sdesc_sw128(vb + 2048 * k, TILE_BYTES / 2, 1024);
          mma_f16_ts(tmem + TM_O + pb * 128, tmem + TM_P + pb * 64 + 8 * k, bd, id_o, k != 0);
        }
        issued = true;
        mma_commit(&o_full[pb]);
        mma_commit(&v_empty[st]);
        mma_commit(&p_empty[pb]);
        return true;
      };
      for (int j = 0; j < nkt && ok; ++j) {
        const int st = j % KV_STAGES;
        if (!mbar_wait(&k_full[st], (j / KV_STAGES) & 1, p.status, 205)) { ok = false; break; }
        if (!mbar_wait(s_empty, (j & 1) ^ 1, p.status, 206)) { ok = false; break; }  // S(j-1) read
        tc_fence_after();
        const uint32_t kb = smem_u32(sK + st * 2 * TILE_BYTES);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = (k >> 2) * (TILE_BYTES / 2) + 32 * (k & 3);
          mma_f16_ss(tmem + TM_S, sdesc_sw128(q0 + off, 16, 1024), sdesc_sw128(kb + off, 16, 1024), id_s, k != 0);
        }
        issued = true;
        mma_commit(s_full);
        mma_commit(&k_empty[st]);
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok && nkt > 0) ok = issue_pv(nkt - 1);
      if (!ok && issued) {
        mma_commit(drain);
        mbar_wait(drain, 0, nullptr, 0);
      }
    }
  } else {
    // softmax warps: thread owns query row `row`, half `hf` of the keys and of the output dims
    const int g = warp & 3, hf = warp >> 2;
    const int row = g * 32 + lane;
    const uint32_t tl = static_cast<uint32_t>(g * 32) << 16;
    const int limit = p.nvalid;  // keys >= limit are masked
    uint64_t o2[HD / 4];  // this half's 64 output dims as fp32 pairs
#pragma unroll
    for (int i = 0; i < HD / 4; ++i) o2[i] = 0;
    float m_run = -INFINITY, l_run = 0.f, alpha_pend = 0.f;
    uint32_t sa[32], r[32];
    bool ok = true;
    auto consume_pv = [&](int i, float alpha) -> bool {
      const int ob = i & 1;
      if (!mbar_wait(&o_full[ob], (i >> 1) & 1, p.status, 207)) return false;
      tc_fence_after();
      const uint32_t ta = tmem + tl + TM_O + ob * 128 + 64 * hf;
      tmem_ld32(ta, sa);
      tmem_ld32(ta + 32, r);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[ob]);
      const uint64_t a2 = f2pack(alpha, alpha);
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        o2[t] = ffma2(o2[t], a2, f2pack(__uint_as_float(sa[2 * t]), __uint_as_float(sa[2 * t + 1])));
        o2[16 + t] = ffma2(o2[16 + t], a2, f2pack(__uint_as_float(r[2 * t]), __uint_as_float(r[2 * t + 1])));
      }
      return true;
    };
    // exchange one float per row with the other half: write, arrive (one per warp), wait, read
    auto exchange = [&](int par, int phase, float mine, float& theirs) -> bool {
      xch[(par * 2 + hf) * 128 + row] = mine;
      __syncwarp();
      if (lane == 0) mbar_arrive(&xbar[par * 4 + g]);
      if (!mbar_wait(&xbar[par * 4 + g], phase & 1, p.status, 213)) return false;
      theirs = xch[(par * 2 + (hf ^ 1)) * 128 + row];
      return true;
    };
    const uint64_t scale2 = f2pack(p.scale_log2, p.scale_log2);
    for (int j = 0; j < nkt && ok; ++j) {
      const int pb = j & 1;
      if (!mbar_wait(s_full, j & 1, p.status, 208)) { ok = false; break; }
      tc_fence_after();
      const int key0 = j * KT, kown = key0 + 64 * hf;
      const bool full_tile = key0 + KT <= limit;
      tmem_ld32(tmem + tl + TM_S + 64 * hf, sa);
      tmem_ld32(tmem + tl + TM_S + 64 * hf + 32, r);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_empty);  // S is in registers: the MMA may overwrite it
      float mxp[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) mxp[t] = -INFINITY;
      if (full_tile) {
        max32<true>(mxp, sa, kown, limit);
        max32<true>(mxp, r, kown + 32, limit);
      } else {
        max32<false>(mxp, sa, kown, limit);
        max32<false>(mxp, r, kown + 32, limit);
      }
      const float pm = fmax3(fmax3(mxp[0], mxp[1], mxp[2]), fmax3(mxp[3], mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7]));
      float om;
      if (!exchange(j & 1, j >> 1, pm, om)) { ok = false; break; }
      const float mx = fmaxf(pm, om) * p.scale_log2;
      const float m_new = fmaxf(m_run, mx);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = ex2(m_run - m_use);  // 0 on the first tile
      // P buffer pb is free once P.V of tile j-2 has completed
      if (!mbar_wait(&p_empty[pb], ((j >> 1) & 1) ^ 1, p.status, 209)) { ok = false; break; }
      uint64_t sum2[4] = {0, 0, 0, 0};
      const uint64_t negm2 = f2pack(-m_use, -m_use);
      // keys 64hf + t -> P column 32hf + t/2 of buffer pb
      const uint32_t tp = tmem + tl + TM_P + pb * 64 + 32 * hf;
      {
        uint32_t pk[16];
        if (full_tile) {
          exp32<true>(pk, sum2, sa, scale2, negm2, kown, limit);
          tmem_st16(tp, pk);
          exp32<true>(pk, sum2, r, scale2, negm2, kown + 32, limit);
          tmem_st16(tp + 16, pk);
        } else {
          exp32<false>(pk, sum2, sa, scale2, negm2, kown, limit);
          tmem_st16(tp, pk);
          exp32<false>(pk, sum2, r, scale2, negm2, kown + 32, limit);
          tmem_st16(tp + 16, pk);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[pb]);
      const uint64_t s01 = fadd2(fadd2(sum2[0], sum2[1]), fadd2(sum2[2], sum2[3]));
      float slo, shi;
      f2unpack(s01, slo, shi);
      l_run = fmaf(l_run, alpha, slo + shi);
      m_run = m_new;
      if (j >= 1 && !consume_pv(j - 1, alpha_pend)) { ok = false; break; }
      alpha_pend = alpha;
    }
    if (ok && nkt > 0) ok = consume_pv(nkt - 1, alpha_pend);
    // full row sum = the two halves' partial sums
    float l_other = 0.f;
    if (ok) ok = exchange(nkt & 1, nkt >> 1, l_run, l_other);
    const int q = qt * QT + row;
    if (ok && q < p.Tq) {
      const float l = l_run + l_other;
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      __half* dst = p.o + (static_cast<size_t>(b) * p.Tq + q) * p.ldo + h * HD + 64 * hf;
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int u = 0; u < HD / 16; ++u) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) f2unpack(o2[4 * u + e], v[2 * e], v[2 * e + 1]);
        d4[u] = make_uint4(pack_half2(v[0] * inv, v[1] * inv), pack_half2(v[2] * inv, v[3] * inv),
                           pack_half2(v[4] * inv, v[5] * inv), pack_half2(v[6] * inv, v[7] * inv));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == MMA_WARP) tmem_dealloc(tmem, 512);
}

}  // namespace

cudaError_t attn_launch(const AttnArgs& a, cudaStream_t s) {
  if (!a.q || !a.k || !a.v || !a.o || a.B <= 0 || a.H <= 0 || a.Tq <= 0 || a.Tk <= 0) return cudaErrorInvalidValue;
  if ((a.ldq | a.ldk | a.ldv | a.ldo | a.q_col0 | a.k_col0 | a.v_col0) & 7) return cudaErrorInvalidValue;
  if (!(a.scale > 0.f)) return cudaErrorInvalidValue;  // the row max is taken on unscaled scores
  CUtensorMap tQ, tK, tV;
  const uint64_t qp = static_cast<uint64_t>(a.ldq) * 2, kp = static_cast<uint64_t>(a.ldk) * 2,
                 vp = static_cast<uint64_t>(a.ldv) * 2;
  if (!make_tmap_3d(&tQ, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.q, a.ldq, a.Tq, a.B, qp, qp * a.Tq, 64, QT, 1,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_3d(&tK, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.k, a.ldk, a.Tk, a.B, kp, kp * a.Tk, 64, KT, 1,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_3d(&tV, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.v, a.ldv, a.Tk, a.B, vp, vp * a.Tk, 64, KT, 1,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  static uint64_t attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set >> dev & 1)) {
    cudaError_t e = cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_SMEM);
    if (e != cudaSuccess) return e;
    attr_set |= 1ull << dev;
  }
  AParams p;
  p.Tq = a.Tq;
  p.Tk = a.Tk;
  p.nvalid = (a.nvalid > 0 && a.nvalid < a.Tk) ? a.nvalid : a.Tk;
  p.H = a.H;
  p.nkt = (a.Tk + KT - 1) / KT;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.o = a.o;
  p.ldo = a.ldo;
  p.status = a.status;
  dim3 grid((a.Tq + QT - 1) / QT, a.H, a.B);
  attn_kernel<<<grid, ATT_THREADS, ATT_SMEM, s>>>(tQ, tK, tV, p, a.q_col0, a.k_col0, a.v_col0);
  return cudaGetLastError();
}

}  // namespace hx

// Flash-style attention on tcgen05 tensor cores, head_dim 128, online softmax.
//
// Replaces attn_run (hexagon/mega/blk.c:54-91; masked joint version moss/hexagon/mega/blk.c:54-94)
// with its table softmax k_softmax2p (hexagon/mega/kern.c:261-282; moss kern.c:262-285) and row
// normalisation k_rowscale_sum (kern.c:285-295): o = softmax(q k^T * scale) v per head. Keys at
// index >= nvalid get probability 0 (the reference masks the last key tile to -65504).
// The reference folds 1/sqrt(128) into the q RMS gain (export_all.py:31-32), so scale = 1 there.
//
// One CTA per (128 queries, head, image). 6 warps:
//   warps 0-3  softmax + output: thread i owns query row i (TMEM lane i)
//   warp  4    TMA producer (Q once, K/V tiles of 128 keys in a 2-stage ring)
//   warp  5    TMEM allocator + tcgen05.mma issuer
// TMEM: S double buffer (cols 0,128) and P.V partials double buffer (cols 256,384).
// S = Q K^T (both K-major); O_part = P V with P (fp16, K-major) staged in shared memory and
// V read MN-major straight from its row-major tile. The running output stays in registers:
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
constexpr int ATT_THREADS = 192;
constexpr int TILE_BYTES = 128 * 128 * 2;  // 32 KB: two 64-column swizzled halves
constexpr int SMEM_Q = 0, SMEM_KV = TILE_BYTES, SMEM_P = TILE_BYTES * 5;
constexpr int ATT_SMEM = TILE_BYTES * 6 + 1024 + 1024;

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

__global__ void __launch_bounds__(ATT_THREADS, 1)
    attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const AParams p, int q_col0, int k_col0, int v_col0) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TILE_BYTES * 6);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* s_empty = bars + 7;   // [2]
  uint64_t* p_full = bars + 9;
  uint64_t* p_empty = bars + 10;
  uint64_t* o_full = bars + 11;   // [2]
  uint64_t* o_empty = bars + 13;  // [2]
  uint64_t* drain = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int nkt = p.nkt;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(p_empty, 1);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      const int qc = q_col0 + h * HD, kc = k_col0 + h * HD, vc = v_col0 + h * HD;
      mbar_arrive_expect_tx(q_full, TILE_BYTES);
      tma_load_3d(smem + SMEM_Q, &tmQ, q_full, qc, qt * QT, b);
      tma_load_3d(smem + SMEM_Q + TILE_BYTES / 2, &tmQ, q_full, qc + 64, qt * QT, b);
      int j = 0;
      bool ok = true;
      for (; j < nkt; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1, p.status, 201)) { ok = false; break; }
        uint8_t* kbuf = smem + SMEM_KV + st * 2 * TILE_BYTES;
        uint8_t* vbuf = kbuf + TILE_BYTES;
        mbar_arrive_expect_tx(&kv_full[st], 2 * TILE_BYTES);
        tma_load_3d(kbuf, &tmK, &kv_full[st], kc, j * KT, b);
        tma_load_3d(kbuf + TILE_BYTES / 2, &tmK, &kv_full[st], kc + 64, j * KT, b);
        tma_load_3d(vbuf, &tmV, &kv_full[st], vc, j * KT, b);
        tma_load_3d(vbuf + TILE_BYTES / 2, &tmV, &kv_full[st], vc + 64, j * KT, b);
      }
      if (!ok) {
        mbar_wait(q_full, 0, nullptr, 0);
        for (int i = (j > 2 ? j - 2 : 0); i < j; ++i) mbar_wait(&kv_full[i & 1], (i >> 1) & 1, nullptr, 0);
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_f16(QT, KT, 0, 0);  // S = Q K^T, both K-major
      constexpr uint32_t id_o = idesc_f16(QT, HD, 0, 1);  // O = P V, V MN-major
      const uint32_t q0 = smem_u32(smem + SMEM_Q), pb = smem_u32(smem + SMEM_P);
      bool ok = mbar_wait(q_full, 0, p.status, 202);
      bool issued = false;
      auto issue_pv = [&](int i) -> bool {
        const int st = i & 1, ob = i & 1;
        if (!mbar_wait(p_full, i & 1, p.status, 203)) return false;
        if (!mbar_wait(&o_empty[ob], ((i >> 1) & 1) ^ 1, p.status, 204)) return false;
        tc_fence_after();
        const uint32_t vb = smem_u32(smem + SMEM_KV + st * 2 * TILE_BYTES + TILE_BYTES);
#pragma unroll
        for (int k = 0; k < KT / 16; ++k) {
          const uint64_t ad = sdesc_sw128(pb + (k >> 2) * (TILE_BYTES / 2) + 32 * (k & 3), 16, 1024);
          const uint64_t bd = sdesc_sw128(vb + 2048 * k, TILE_BYTES / 2, 1024);
          mma_f16_ss(tmem + 256 + ob * 128, ad, bd, id_o, k != 0);
        }
        issued = true;
        mma_commit(&o_full[ob]);
        mma_commit(&kv_empty[st]);
        mma_commit(p_empty);
        return true;
      };
      for (int j = 0; j < nkt && ok; ++j) {
        const int st = j & 1, sb = j & 1;
        if (!mbar_wait(&kv_full[st], (j >> 1) & 1, p.status, 205)) { ok = false; break; }
        if (!mbar_wait(&s_empty[sb], ((j >> 1) & 1) ^ 1, p.status, 206)) { ok = false; break; }
        tc_fence_after();
        const uint32_t kb = smem_u32(smem + SMEM_KV + st * 2 * TILE_BYTES);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = (k >> 2) * (TILE_BYTES / 2) + 32 * (k & 3);
          mma_f16_ss(tmem + sb * 128, sdesc_sw128(q0 + off, 16, 1024), sdesc_sw128(kb + off, 16, 1024), id_s, k != 0);
        }
        issued = true;
        mma_commit(&s_full[sb]);
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok && nkt > 0) ok = issue_pv(nkt - 1);
      if (!ok && issued) {
        mma_commit(drain);
        mbar_wait(drain, 0, nullptr, 0);
      }
    }
  } else {
    // softmax warps: thread owns one query row
    const int row = warp * 32 + lane;
    const uint32_t tl = static_cast<uint32_t>(warp * 32) << 16;
    const int limit = p.nvalid;  // keys >= limit are masked
    float o[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) o[i] = 0.f;
    float m_run = -INFINITY, l_run = 0.f, alpha_pend = 0.f;
    uint32_t r[32];
    const uint32_t pb = smem_u32(smem + SMEM_P);
    bool ok = true;
    auto consume_pv = [&](int i, float alpha) -> bool {
      const int ob = i & 1;
      if (!mbar_wait(&o_full[ob], (i >> 1) & 1, p.status, 207)) return false;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        tmem_ld32(tmem + tl + 256 + ob * 128 + 32 * c, r);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 32; ++t) o[32 * c + t] = fmaf(o[32 * c + t], alpha, __uint_as_float(r[t]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[ob]);
      return true;
    };
    for (int j = 0; j < nkt && ok; ++j) {
      const int sb = j & 1;
      if (!mbar_wait(&s_full[sb], (j >> 1) & 1, p.status, 208)) { ok = false; break; }
      tc_fence_after();
      const uint32_t ts = tmem + tl + sb * 128;
      const int key0 = j * KT;
      const bool full_tile = key0 + KT <= limit;
      // row max of the raw scores (scale > 0), 8 independent partial maxima per 32 columns
      float mxp[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) mxp[t] = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < KT / 32; ++c) {
        tmem_ld32(ts + 32 * c, r);
        tmem_ld_wait();
        if (full_tile) {
#pragma unroll
          for (int t = 0; t < 32; ++t) mxp[t & 7] = fmaxf(mxp[t & 7], __uint_as_float(r[t]));
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t)
            if (key0 + 32 * c + t < limit) mxp[t & 7] = fmaxf(mxp[t & 7], __uint_as_float(r[t]));
        }
      }
      const float mx = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                             fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7]))) * p.scale_log2;
      const float m_new = fmaxf(m_run, mx);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = ex2(m_run - m_use);  // 0 on the first tile
      // the P buffer is free once the previous P.V has been issued and completed
      if (!mbar_wait(p_empty, (j & 1) ^ 1, p.status, 209)) { ok = false; break; }
      float sump[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) sump[t] = 0.f;
#pragma unroll 1
      for (int c = 0; c < KT / 32; ++c) {
        tmem_ld32(ts + 32 * c, r);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          const bool v0 = full_tile || (key0 + 32 * c + t < limit);
          const bool v1 = full_tile || (key0 + 32 * c + t + 1 < limit);
          const float e0 = v0 ? ex2(fmaf(__uint_as_float(r[t]), p.scale_log2, -m_use)) : 0.f;
          const float e1 = v1 ? ex2(fmaf(__uint_as_float(r[t + 1]), p.scale_log2, -m_use)) : 0.f;
          sump[(t >> 1) & 7] += e0 + e1;
          pk[t / 2] = pack_half2(e0, e1);
        }
        // keys 32c..32c+31 -> half (c/2) of P, 16-byte units 4(c%2)..4(c%2)+3, swizzled by row
        const uint32_t base = pb + (c >> 1) * (TILE_BYTES / 2) + row * 128;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t unit = (4 * (c & 1) + u) ^ (row & 7);
          st_shared_v4(base + unit * 16, pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s_empty[sb]);
        mbar_arrive(p_full);
      }
      const float rowsum = ((sump[0] + sump[1]) + (sump[2] + sump[3])) + ((sump[4] + sump[5]) + (sump[6] + sump[7]));
      l_run = fmaf(l_run, alpha, rowsum);
      m_run = m_new;
      if (j >= 1 && !consume_pv(j - 1, alpha_pend)) { ok = false; break; }
      alpha_pend = alpha;
    }
    if (ok && nkt > 0) ok = consume_pv(nkt - 1, alpha_pend);
    const int q = qt * QT + row;
    if (ok && q < p.Tq) {
      const float inv = l_run > 0.f ? 1.0f / l_run : 0.f;
      __half* dst = p.o + (static_cast<size_t>(b) * p.Tq + q) * p.ldo + h * HD;
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int u = 0; u < HD / 8; ++u)
        d4[u] = make_uint4(pack_half2(o[8 * u] * inv, o[8 * u + 1] * inv), pack_half2(o[8 * u + 2] * inv, o[8 * u + 3] * inv),
                           pack_half2(o[8 * u + 4] * inv, o[8 * u + 5] * inv), pack_half2(o[8 * u + 6] * inv, o[8 * u + 7] * inv));
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem, 512);
}

}  // namespace

cudaError_t attn_launch(const AttnArgs& a, cudaStream_t s) {
  if (!a.q || !a.k || !a.v || !a.o || a.B <= 0 || a.H <= 0 || a.Tq <= 0 || a.Tk <= 0) return cudaErrorInvalidValue;
  if ((a.ldq | a.ldk | a.ldv | a.ldo | a.q_col0 | a.k_col0 | a.v_col0) & 7) return cudaErrorInvalidValue;
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

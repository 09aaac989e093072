// Flash-style attention on tcgen05 tensor cores, head_dim 128, online softmax.
//
// Replaces attn_run (hexagon/mega/blk.c:54-91; masked joint version moss/hexagon/mega/blk.c:54-94)
// with its table softmax k_softmax2p (hexagon/mega/kern.c:261-282; moss kern.c:262-285) and row
// normalisation k_rowscale_sum (kern.c:285-295): o = softmax(q k^T * scale) v per head. Keys at
// index >= nvalid get probability 0 (the reference masks the last key tile to -65504).
// The reference folds 1/sqrt(128) into the q RMS gain (export_all.py:31-32), so scale = 1 there.
//
// Persistent: one CTA per SM walks items (256 queries = two 128-row Q tiles A and B, head, image), the
// next item's Q, K and V loads overlapping the current item's softmax. 16 warps in four warpgroups:
//   warpgroup 0 softmax of Q tile A, warpgroup 1 softmax of Q tile B: thread = one query row (TMEM lane
//              32(w%4) + lane) with the row's 128 scores of a K tile in registers (one TMEM load wait);
//              P is published in two parts so the P V MMA starts on keys [0, 96) while the rest is
//              computed, and the row sum is taken after P is published
//   warpgroup 2 epilogue: O_X / l of each item to global memory, while the softmax warps go on with the
//              next item
//   warpgroup 3 warp 12 TMA producer (Q tiles once, then K and V tiles of 128 keys in 2- and 3-stage rings),
//              warp 13 TMEM allocator + tcgen05.mma issuer, warps 14-15 idle
// setmaxnreg gives the softmax warpgroups 192 registers, the epilogue 32 and the control warpgroup 96.
// TMEM columns: S_A [0,128), S_B [128,256) fp32; O_A [256,384), O_B [384,512) fp32 accumulators.
// P_X (fp16, two per column) is written over columns [0,64) of S_X once they are read, and O_X += P_X V
// reads it from TMEM. S_X(j+1) overwrites P_X(j); the MMA thread issues it directly after
// O_X += P_X(j) V, and the tensor pipe runs the MMAs of one thread in issue order. The commit that
// signals S_X(j+1) to the softmax warps also covers every earlier MMA, so by then O_X += P_X(j) V is
// complete and O_X may be rescaled.
// Online softmax with a lazy reference maximum: P = 2^(s*scale_log2 - m_ref) and the row sum use m_ref,
// which moves (rescaling the row of O in TMEM and the running sum) only when the tile maximum exceeds
// it by more than 8, so P <= 256. o = O / l at the end is independent of m_ref.
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "hx_internal.h"
#include "hx_ptx.cuh"
#include "hx_softmax.cuh"

namespace hx {

bool make_tmap_3d(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* base, uint64_t d0, uint64_t d1,
                  uint64_t d2, uint64_t pitch1, uint64_t pitch2, uint32_t b0, uint32_t b1, uint32_t b2,
                  CUtensorMapSwizzle sw);

namespace {

using namespace smx;

constexpr int QT = 128, KT = 128, HD = 128;
constexpr int QPAIR = 2 * QT;  // queries per CTA
// 16 warps: warpgroups 0 and 1 softmax (Q tiles A and B), 2 epilogue, 3 control (TMA warp, MMA warp, 2 idle)
constexpr int ATT_WARPS = 16, ATT_THREADS = ATT_WARPS * 32;
constexpr int EPI_WG = 2;
constexpr int TMA_WARP = 12, MMA_WARP = 13;
constexpr int REG_SOFTMAX = 192, REG_EPI = 32, REG_CTRL = 96;  // setmaxnreg split of the 128 a thread starts with
static_assert(2 * REG_SOFTMAX + REG_EPI + REG_CTRL <= 4 * 128, "register split exceeds the launch allocation");
constexpr int P_SPLIT = 96;   // keys of P published first (the P V MMA starts on them)
constexpr int K_STAGES = 2, V_STAGES = 3;  // V waits longer for its ring slot (freed by P V, not by S)
constexpr int TILE_BYTES = 128 * 128 * 2;  // 32 KB: two 64-column swizzled halves
// Q_A | Q_B | K0 K1 | V0 V1 V2, then barriers, then the row sums handed to the epilogue
constexpr int SMEM_Q = 0, SMEM_K = 2 * TILE_BYTES, SMEM_V = SMEM_K + K_STAGES * TILE_BYTES;
constexpr int SMEM_BARS = SMEM_V + V_STAGES * TILE_BYTES;
constexpr int SMEM_L = SMEM_BARS + 256;
constexpr int ATT_SMEM = SMEM_L + 2 * QT * 4 + 1024;  // + alignment slack
constexpr uint32_t TM_S = 0, TM_O = 256;
constexpr float RESCALE_LOG2 = 8.0f;  // move m_ref only when the tile max exceeds it by more than this

struct AParams {
  int Tq, Tk, nvalid, H, nkt;
  int B, nqp;  // images, 256-query blocks per image
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
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SMEM_BARS);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* k_empty = bars + 3;   // [2]
  uint64_t* v_full = bars + 5;    // [3]
  uint64_t* v_empty = bars + 8;   // [3]
  uint64_t* s_full = bars + 11;   // [Q tile] S_X(g) committed
  uint64_t* p_part = bars + 13;   // [Q tile] P_X(g) keys [0, P_SPLIT) stored, one arrival per softmax warp
  uint64_t* p_full = bars + 15;   // [Q tile] all of P_X(g) stored
  uint64_t* pv_done = bars + 17;  // [Q tile] O_X += P_X(g) V committed
  uint64_t* l_full = bars + 19;   // [Q tile] the item's row sums are in sm_l, one arrival per softmax warp
  uint64_t* l_free = bars + 21;   // [Q tile] the epilogue warps have read them
  uint64_t* o_free = bars + 23;   // [Q tile] the epilogue warps have read O_X: the next item may overwrite it
  uint64_t* q_empty = bars + 25;  // the item's S MMAs have read Q: the next item's Q may load
  uint64_t* drain = bars + 26;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 28);
  float* sm_l = reinterpret_cast<float*>(smem + SMEM_L);  // [Q tile][128] row sums handed to the epilogue

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, wg = warp >> 2;
  const int nkt = p.nkt;
  // persistent: this CTA's items n = 0, 1, ... are blockIdx.x + n * gridDim.x; item -> (Q-tile pair, head,
  // image) with the Q-tile pair fastest so that CTAs running at the same time share K and V in L2
  const int nitems = p.nqp * p.H * p.B;
  const int nmine = nitems > static_cast<int>(blockIdx.x)
                        ? (nitems - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                        : 0;
  auto item_of = [&](int n, int& qp, int& h, int& b) {
    const int it = static_cast<int>(blockIdx.x) + n * static_cast<int>(gridDim.x);
    qp = it % p.nqp;
    h = (it / p.nqp) % p.H;
    b = it / (p.nqp * p.H);
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < K_STAGES; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < V_STAGES; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&p_part[x], 4);
      mbar_init(&p_full[x], 4);
      mbar_init(&pv_done[x], 1);
      mbar_init(&l_full[x], 4);
      mbar_init(&l_free[x], 4);
      mbar_init(&o_free[x], 4);
    }
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
  grid_dep_wait();  // the previous kernel's outputs (q, k, v) are complete
  grid_dep_launch();

  // registers: the block starts with 128 per thread (65536); each role branch first sets its warpgroup's
  // share: softmax 192, epilogue 32, control 96, so 128 threads x (192 + 192 + 32 + 96) = 65536, and per
  // SMSP (one warp of each warpgroup) 32 x 512 = 16384, its register bank
  if (wg == 3) {
    setmaxnreg_dec<REG_CTRL>();
  if (warp == TMA_WARP) {
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      int nq = 0, nk = 0, nv = 0;  // Q, K and V loads issued
      bool ok = true;
      for (int n = 0; n < nmine && ok; ++n) {
        int qp, h, b;
        item_of(n, qp, h, b);
        const int qc = q_col0 + h * HD, kc = k_col0 + h * HD, vc = v_col0 + h * HD;
        if (!mbar_wait(q_empty, (n & 1) ^ 1, p.status, 214)) { ok = false; break; }
        mbar_arrive_expect_tx(q_full, 2 * TILE_BYTES);
        for (int x = 0; x < 2; ++x) {
          uint8_t* qb = smem + SMEM_Q + x * TILE_BYTES;
          tma_load_3d(qb, &tmQ, q_full, qc, qp * QPAIR + x * QT, b);
          tma_load_3d(qb + TILE_BYTES / 2, &tmQ, q_full, qc + 64, qp * QPAIR + x * QT, b);
        }
        ++nq;
        for (int j = 0; j < nkt; ++j) {
          const int g = n * nkt + j;
          const int st = g & 1, ph = (g >> 1) & 1;          // K ring
          const int vs = g % V_STAGES, vph = (g / V_STAGES) & 1;  // V ring
          uint8_t* kb = smem + SMEM_K + st * TILE_BYTES;
          uint8_t* vb = smem + SMEM_V + vs * TILE_BYTES;
          if (!mbar_wait(&k_empty[st], ph ^ 1, p.status, 201)) { ok = false; break; }
          mbar_arrive_expect_tx(&k_full[st], TILE_BYTES);
          tma_load_3d(kb, &tmK, &k_full[st], kc, j * KT, b);
          tma_load_3d(kb + TILE_BYTES / 2, &tmK, &k_full[st], kc + 64, j * KT, b);
          ++nk;
          if (!mbar_wait(&v_empty[vs], vph ^ 1, p.status, 211)) { ok = false; break; }
          mbar_arrive_expect_tx(&v_full[vs], TILE_BYTES);
          tma_load_3d(vb, &tmV, &v_full[vs], vc, j * KT, b);
          tma_load_3d(vb + TILE_BYTES / 2, &tmV, &v_full[vs], vc + 64, j * KT, b);
          ++nv;
        }
      }
      if (!ok) {  // aborted: let the copies in flight land before the CTA exits
        if (nq > 0) mbar_wait(q_full, (nq - 1) & 1, nullptr, 0);
        for (int i = (nk > K_STAGES ? nk - K_STAGES : 0); i < nk; ++i)
          mbar_wait(&k_full[i & 1], (i >> 1) & 1, nullptr, 0);
        for (int i = (nv > V_STAGES ? nv - V_STAGES : 0); i < nv; ++i)
          mbar_wait(&v_full[i % V_STAGES], (i / V_STAGES) & 1, nullptr, 0);
      }
    }
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_f16(QT, KT, 0, 0);  // S = Q K^T, both K-major
      constexpr uint32_t id_o = idesc_f16(QT, HD, 0, 1);  // O += P V, P K-major in TMEM, V MN-major
      bool ok = true;
      bool issued = false;
      // S_x(g) overwrites P_x(g-1), the A operand of O_x += P_x(g-1) V: it is issued right after that MMA by
      // this thread, and the tensor pipe runs one thread's MMAs in issue order
      auto issue_s = [&](int x, int g) {
        const uint32_t q0 = smem_u32(smem + SMEM_Q + x * TILE_BYTES);
        const uint32_t kb = smem_u32(smem + SMEM_K + (g & 1) * TILE_BYTES);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = (k >> 2) * (TILE_BYTES / 2) + 32 * (k & 3);
          mma_f16_ss(tmem + TM_S + x * 128, sdesc_sw128(q0 + off, 16, 1024), sdesc_sw128(kb + off, 16, 1024), id_s,
                     k != 0);
        }
        issued = true;
        mma_commit(&s_full[x]);
      };
      // O_x (+)= P_x(g) V(g) in two parts: keys [0, P_SPLIT) as soon as the softmax warps have stored them,
      // the rest when all of P is stored; the first tile of an item overwrites O_x once the previous item's
      // O_x was read
      auto issue_pv = [&](int x, int g, int n, bool first) -> bool {
        if (first && n > 0 && !mbar_wait(&o_free[x], (n - 1) & 1, p.status, 215)) return false;
        const uint32_t vb = smem_u32(smem + SMEM_V + (g % V_STAGES) * TILE_BYTES);
        if (!mbar_wait(&p_part[x], g & 1, p.status, 204)) return false;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < P_SPLIT / 16; ++k) {
          const uint64_t bd = sdesc_sw128(vb + 2048 * k, TILE_BYTES / 2, 1024);
          mma_f16_ts(tmem + TM_O + x * 128, tmem + TM_S + x * 128 + 8 * k, bd, id_o, (!first || k != 0) ? 1u : 0u);
        }
        issued = true;
        if (!mbar_wait(&p_full[x], g & 1, p.status, 216)) return false;
        tc_fence_after();
#pragma unroll
        for (int k = P_SPLIT / 16; k < KT / 16; ++k) {
          const uint64_t bd = sdesc_sw128(vb + 2048 * k, TILE_BYTES / 2, 1024);
          mma_f16_ts(tmem + TM_O + x * 128, tmem + TM_S + x * 128 + 8 * k, bd, id_o, 1u);
        }
        mma_commit(&pv_done[x]);
        return true;
      };
      for (int n = 0; n < nmine && ok; ++n) {
        const int g0 = n * nkt;
        // per tile: PV_A(g) S_A(g+1) PV_B(g) S_B(g+1); the item starts with S_A(g0) S_B(g0)
        if (!(mbar_wait(q_full, n & 1, p.status, 202) && mbar_wait(&k_full[g0 & 1], (g0 >> 1) & 1, p.status, 205))) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_s(0, g0);
        issue_s(1, g0);
        mma_commit(&k_empty[g0 & 1]);
        if (nkt == 1) mma_commit(q_empty);
        for (int j = 0; j < nkt && ok; ++j) {
          const int g = g0 + j;
          const bool more = j + 1 < nkt;
          if (!mbar_wait(&v_full[g % V_STAGES], (g / V_STAGES) & 1, p.status, 206)) { ok = false; break; }
          if (!issue_pv(0, g, n, j == 0)) { ok = false; break; }
          if (more) {
            if (!mbar_wait(&k_full[(g + 1) & 1], ((g + 1) >> 1) & 1, p.status, 207)) { ok = false; break; }
            tc_fence_after();
            issue_s(0, g + 1);
          }
          if (!issue_pv(1, g, n, j == 0)) { ok = false; break; }
          mma_commit(&v_empty[g % V_STAGES]);
          if (more) {
            issue_s(1, g + 1);
            mma_commit(&k_empty[(g + 1) & 1]);
            if (j + 2 == nkt) mma_commit(q_empty);  // the item's last S is issued: Q may be replaced
          }
        }
      }
      if (!ok && issued) {
        mma_commit(drain);
        mbar_wait(drain, 0, nullptr, 0);
      }
    }
  }
  } else if (wg < 2) {
    setmaxnreg_inc<REG_SOFTMAX>();
    // softmax warps: thread owns query row `row` of Q tile `qx` of each item, the whole 128-key row of S in
    // registers
    const int qx = wg, g4 = warp & 3;
    const int row = g4 * 32 + lane;
    const uint32_t tl = static_cast<uint32_t>(g4 * 32) << 16;
    const uint32_t tS = tmem + tl + TM_S + qx * 128, tO = tmem + tl + TM_O + qx * 128;
    const int limit = p.nvalid;  // keys >= limit are masked
    const uint64_t scale2 = f2pack(p.scale_log2, p.scale_log2);
    uint32_t s[KT];
    bool ok = true;
    for (int n = 0; n < nmine && ok; ++n) {
      float m_ref = 0.f, l_run = 0.f;
      for (int j = 0; j < nkt && ok; ++j) {
        const int g = n * nkt + j;
        if (!warp_wait(&s_full[qx], g & 1, p.status, 208)) { ok = false; break; }
        tc_fence_after();
        const int key0 = j * KT;
        const bool full_tile = key0 + KT <= limit;
        tmem_ld32(tS, *reinterpret_cast<uint32_t(*)[32]>(s));
        tmem_ld32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(s + 32));
        tmem_ld32(tS + 64, *reinterpret_cast<uint32_t(*)[32]>(s + 64));
        tmem_ld32(tS + 96, *reinterpret_cast<uint32_t(*)[32]>(s + 96));
        tmem_ld_wait();
        float mxp[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) mxp[t] = -INFINITY;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (full_tile)
            max32<true>(mxp, *reinterpret_cast<uint32_t(*)[32]>(s + 32 * c), key0 + 32 * c, limit);
          else
            max32<false>(mxp, *reinterpret_cast<uint32_t(*)[32]>(s + 32 * c), key0 + 32 * c, limit);
        }
        const float mt =
            fmax3(fmax3(mxp[0], mxp[1], mxp[2]), fmax3(mxp[3], mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])) * p.scale_log2;
        if (j == 0) {
          m_ref = mt == -INFINITY ? 0.f : mt;  // O_X is written fresh by the item's first P V
        } else {
          const bool need = mt > m_ref + RESCALE_LOG2;
          if (__any_sync(0xffffffffu, need)) {
            // O_X += P_X(g-1) V has completed (the s_full commit of S_X(g), issued after it, covers it);
            // P_X(g) is not published yet
            const float alpha = need ? ex2(m_ref - mt) : 1.f;
            if (need) m_ref = mt;
            l_run *= alpha;
            const uint64_t a2 = f2pack(alpha, alpha);
            uint32_t ob[16];  // 16 columns at a time: the row of S stays live in registers meanwhile
#pragma unroll
            for (int c = 0; c < HD / 16; ++c) {
              tmem_ld16(tO + 16 * c, ob);
              tmem_ld_wait();
#pragma unroll
              for (int t = 0; t < 16; t += 2) {
                float x0, x1;
                f2unpack(ffma2(f2pack(__uint_as_float(ob[t]), __uint_as_float(ob[t + 1])), a2, 0ull), x0, x1);
                ob[t] = __float_as_uint(x0);
                ob[t + 1] = __float_as_uint(x1);
              }
              tmem_st16(tO + 16 * c, ob);
            }
          }
        }
        const uint64_t negm2 = f2pack(-m_ref, -m_ref);
        // 32 keys at a time: the probabilities go back into s (fp32, for the row sum) and, fp16-packed, into
        // P columns 16c .. 16c+15 over S columns already read; keys [0, P_SPLIT) are published first
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
          if (full_tile)
            exp32_keep<true>(pk, *reinterpret_cast<uint32_t(*)[32]>(s + 32 * c), scale2, negm2, key0 + 32 * c, limit);
          else
            exp32_keep<false>(pk, *reinterpret_cast<uint32_t(*)[32]>(s + 32 * c), scale2, negm2, key0 + 32 * c, limit);
          tmem_st16(tS + 16 * c, pk);
          if (32 * (c + 1) == P_SPLIT || c == 3) {
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(c == 3 ? &p_full[qx] : &p_part[qx]);
          }
        }
        // row sum of this tile's probabilities, off the path to the P V MMA
        uint64_t sum2[4] = {0, 0, 0, 0};
#pragma unroll
        for (int t = 0; t < KT; t += 2)
          sum2[(t >> 1) & 3] = fadd2(sum2[(t >> 1) & 3], f2pack(__uint_as_float(s[t]), __uint_as_float(s[t + 1])));
        const uint64_t s01 = fadd2(fadd2(sum2[0], sum2[1]), fadd2(sum2[2], sum2[3]));
        float slo, shi;
        f2unpack(s01, slo, shi);
        l_run += slo + shi;
      }
      if (!ok) break;
      // hand the item's row sums to the epilogue warps once they have read the previous item's
      if (n > 0 && !warp_wait(&l_free[qx], (n - 1) & 1, p.status, 210)) { ok = false; break; }
      sm_l[qx * QT + row] = l_run;
      __syncwarp();
      if (lane == 0) mbar_arrive(&l_full[qx]);
    }
  } else {
    setmaxnreg_dec<REG_EPI>();
    // epilogue warps: O_X / l of each item to global memory; warp 8 + g4 reads TMEM lanes 32 g4 .. +31
    const int g4 = warp & 3;
    const int row = g4 * 32 + lane;
    const uint32_t tl = static_cast<uint32_t>(g4 * 32) << 16;
    uint32_t ob[16];
    bool ok = true;
    for (int n = 0; n < nmine && ok; ++n) {
      int qp, h, b;
      item_of(n, qp, h, b);
      for (int x = 0; x < 2; ++x) {
        // the row sums first: the softmax warps publish them after the item's last S_X, so the item's P V
        // commits before the last have all arrived and the pv_done wait below is for the last one
        if (!warp_wait(&l_full[x], n & 1, p.status, 217)) { ok = false; break; }
        const float l = sm_l[x * QT + row];
        __syncwarp();
        if (lane == 0) mbar_arrive(&l_free[x]);
        if (!warp_wait(&pv_done[x], (n * nkt + nkt - 1) & 1, p.status, 209)) { ok = false; break; }
        tc_fence_after();
        const int q = qp * QPAIR + x * QT + row;
        const bool live = q < p.Tq;
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        uint4* d4 = reinterpret_cast<uint4*>(p.o + (static_cast<size_t>(b) * p.Tq + (live ? q : 0)) * p.ldo + h * HD);
        const uint32_t tO = tmem + tl + TM_O + x * 128;
#pragma unroll
        for (int c = 0; c < HD / 16; ++c) {  // 16 columns at a time (56 registers)
          tmem_ld16(tO + 16 * c, ob);
          tmem_ld_wait();
          if (c == HD / 16 - 1) {  // all of O_X read: the next item's first P V may overwrite it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&o_free[x]);
          }
          if (live) {
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const uint32_t* v = ob + 8 * u;
              d4[2 * c + u] = make_uint4(
                  pack_half2(__uint_as_float(v[0]) * inv, __uint_as_float(v[1]) * inv),
                  pack_half2(__uint_as_float(v[2]) * inv, __uint_as_float(v[3]) * inv),
                  pack_half2(__uint_as_float(v[4]) * inv, __uint_as_float(v[5]) * inv),
                  pack_half2(__uint_as_float(v[6]) * inv, __uint_as_float(v[7]) * inv));
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == MMA_WARP) tmem_dealloc(tmem, 512);
}

}  // namespace

// which kernel attn_launch runs for these arguments on a GPU with `sms` SMs: 1 the general kernel, 2 the
// short-key kernel, -1 invalid arguments (host-side; also answered by hx_attention_query)
int attn_choose(const AttnArgs& a, int sms) {
  if (!a.q || !a.k || !a.v || !a.o || a.B <= 0 || a.H <= 0 || a.Tq <= 0 || a.Tk <= 0 || sms < 1) return -1;
  if ((a.ldq | a.ldk | a.ldv | a.ldo | a.q_col0 | a.k_col0 | a.v_col0) & 7) return -1;
  if (!(a.scale > 0.f)) return -1;  // the row max is taken on unscaled scores
  if (a.kernel == 2) return a.Tk <= 2 * KT ? 2 : -1;
  if (a.kernel != 0 && a.kernel != 1) return -1;
  // at most 256 keys (the cross-attention over the context) and at most six 128-query tiles per SM: the
  // short-key kernel (attn_short.cu: K and V resident, Q tiles streamed, one exact softmax step), which
  // gets a CTA's few tiles done sooner (Anima cross-attention, 1 / 2 / 4 images: 11.9 -> 10.5, 17.6 -> 15.0,
  // 24.1 -> 23.7 us). With more tiles per SM its per-tile chain (S, softmax over 256 keys, P V, O read out
  // before the slot's next S) is longer than the general kernel's pipeline: 8 images 43 us against 49.
  // HX_ATTN_SHORT=0 / 1 in the environment: never / always for 128 < Tk <= 256. Its O goes out by TMA
  // stores, so the output must start on a 16-byte boundary.
  static const int short_mode = [] {
    const char* e = getenv("HX_ATTN_SHORT");
    return e && *e ? atoi(e) : -1;
  }();
  if (a.kernel == 0 && a.Tk > KT && a.Tk <= 2 * KT && short_mode != 0 && reinterpret_cast<uintptr_t>(a.o) % 16 == 0) {
    const long long units = static_cast<long long>((a.Tq + QT - 1) / QT) * a.H * a.B;
    if (short_mode == 1 || units <= 6LL * sms) return 2;
  }
  return 1;
}

cudaError_t attn_launch(const AttnArgs& a, cudaStream_t s) {
  const int k = attn_choose(a, sm_count());
  if (k < 0) return cudaErrorInvalidValue;
  if (k == 2) return attn_short_launch(a, s);
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
  p.B = a.B;
  p.nqp = (a.Tq + QPAIR - 1) / QPAIR;
  const long nitems = static_cast<long>(p.nqp) * a.H * a.B;
  const int grid = static_cast<int>(nitems < sm_count() ? nitems : sm_count());
  const cudaError_t e =
      launch_pdl(attn_kernel, dim3(grid), dim3(ATT_THREADS), ATT_SMEM, s, tQ, tK, tV, p, a.q_col0, a.k_col0, a.v_col0);
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace hx

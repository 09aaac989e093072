// Attention over at most 256 keys, head_dim 128: the Anima cross-attention over the 256 context tokens
// (hexagon/mega/blk.c:54-91 with Tk = C; softmax k_softmax2p, kern.c:261-282, and k_rowscale_sum,
// kern.c:285-295). o = softmax(q k^T * scale) v per head; keys at index >= nvalid get probability 0.
//
// The general kernel (attn.cu) walks 128-key tiles with an online softmax and reloads K and V for every
// 256-query item. With only two key tiles per item its time goes to item turnover: the next item's Q can
// load only once the current item's last S has read Q, and K / V come again with every item. Here a CTA
// owns a contiguous range of 128-query tiles, ordered (image, head, query tile); K and V of one (image,
// head) group are loaded once into shared memory (all 256 keys, 64 KB each) and stay resident while the
// group's Q tiles stream through a 3-deep ring, so the loads run two tiles ahead of their use.
//
// Each Q tile takes one TMEM slot of 256 columns (two slots, used by alternate tiles):
//   S = Q K^T over all 256 keys, fp32, columns [0, 256) of the slot (one N = 256 MMA per 16 of head_dim)
//   P (fp16, two per column): keys [0,128) in columns [128,192), keys [128,256) in [192,256)
//   O = P V (fp32) in columns [0,128)
// The softmax is exact in one step: a thread (one query row) reads S twice, first for the row maximum,
// then for the exponentials (keys 128-255 stay in registers from the first read and their P goes over
// columns S has already given up; keys 0-127 are read again), so no running maximum or rescaling of O is
// needed. P V is issued once all of P is stored, and O overwrites S columns read by then.
//
// 16 warps: warpgroup 0 / 1 softmax and epilogue of the even / odd Q tiles (thread = TMEM lane = query
// row; the row sum stays in the thread; O is read in one go, which releases the TMEM slot, then written
// as fp16 into the tile's own Q slot, which S no longer needs, and stored by TMA; the Q slot returns to
// the ring when the store has read it, and Q tiles are prefetched into L2 three tiles ahead),
// warpgroup 2 idle, warp 12 TMA, warp 13 TMEM allocator and MMA issuer. The MMA thread issues S(i+1)
// before P(i) V, so the tensor pipe computes the next tile's scores while the softmax works; S(i+2) into
// the same slot waits until O(i) has been read.
#include <cmath>
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

constexpr int QT = 128, HD = 128, KMAX = 256;
constexpr int SH_WARPS = 16, SH_THREADS = SH_WARPS * 32;
constexpr int TMA_WARP = 12, MMA_WARP = 13;
constexpr int REG_SOFTMAX = 216, REG_IDLE = 24, REG_CTRL = 56;
static_assert(2 * REG_SOFTMAX + REG_IDLE + REG_CTRL <= 4 * 128, "register split exceeds the launch allocation");
constexpr int Q_STAGES = 3;
constexpr int QTILE_BYTES = QT * HD * 2;   // 32 KB: two 64-column 128-byte-swizzled halves of 128 rows
constexpr int KV_BYTES = KMAX * HD * 2;    // 64 KB: two 64-column halves of 256 rows
constexpr int SMEM_K = 0, SMEM_V = KV_BYTES, SMEM_Q = 2 * KV_BYTES;
constexpr int SMEM_BARS = SMEM_Q + Q_STAGES * QTILE_BYTES;
constexpr int SH_SMEM = SMEM_BARS + 256 + 1024;  // + alignment slack
static_assert(SH_SMEM <= 232448, "shared memory per CTA");
constexpr uint32_t SLOT_COLS = 256, TM_P = 128;  // per slot: S [0,256), P [128,256), O [0,128)

struct SParams {
  int Tq, nvalid, H, nqt;  // nqt: 128-query tiles per (image, head)
  int U;                   // units: B * H * nqt query tiles
  float scale_log2;
  __half* o;
  int ldo;
  int* status;
};

__global__ void __launch_bounds__(SH_THREADS, 1)
    attn_short_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, const SParams p,
                      int q_col0, int k_col0, int v_col0) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SMEM_BARS);
  uint64_t* k_full = bars;        // K of the CTA's current group landed
  uint64_t* k_empty = bars + 1;   // the group's last S has completed: K may be replaced
  uint64_t* v_full = bars + 2;
  uint64_t* v_empty = bars + 3;   // the group's last P V has completed
  uint64_t* q_full = bars + 4;    // [3]
  uint64_t* q_empty = bars + 7;   // [3] the O staged in the Q slot (after its S) has been stored
  uint64_t* s_full = bars + 10;   // [slot]
  uint64_t* p_full = bars + 12;   // [slot] all of P stored, one arrival per softmax warp
  uint64_t* pv_done = bars + 14;  // [slot]
  uint64_t* o_free = bars + 16;   // [slot] O has been read: the slot's next S may overwrite it
  uint64_t* o_staged = bars + 18; // [slot] the tile's O rows are in its Q slot, one arrival per softmax warp
  uint64_t* drain = bars + 20;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 22);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, wg = warp >> 2;
  // this CTA's units [u0, u1): a contiguous, balanced range, so consecutive units mostly share a group
  const int u0 = static_cast<int>(static_cast<long long>(p.U) * blockIdx.x / gridDim.x);
  const int u1 = static_cast<int>(static_cast<long long>(p.U) * (blockIdx.x + 1) / gridDim.x);
  const int nmine = u1 - u0;
  auto group_of = [&](int i) { return (u0 + i) / p.nqt; };  // (image, head) group of local unit i
  auto new_group = [&](int i) { return i == 0 || group_of(i) != group_of(i - 1); };
  auto last_of_group = [&](int i) { return i == nmine - 1 || group_of(i + 1) != group_of(i); };

  if (threadIdx.x == 0) {
    mbar_init(k_full, 1);
    mbar_init(k_empty, 1);
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    for (int i = 0; i < Q_STAGES; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&p_full[x], 4);
      mbar_init(&pv_done[x], 1);
      mbar_init(&o_free[x], 4);
      mbar_init(&o_staged[x], 4);
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

  // registers: 128 per thread at launch (65536); softmax 216, idle 24, control 56 per warpgroup
  if (wg == 3) {
    setmaxnreg_dec<REG_CTRL>();
    if (warp == TMA_WARP) {
      if (lane == 0) {
        prefetch_tmap(&tmQ);
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
        prefetch_tmap(&tmO);
        int nk = 0, nv = 0, nq = 0;  // K, V (one per group) and Q tile loads issued
        bool ok = true;
        for (int i = 0; i < nmine && ok; ++i) {
          const int u = u0 + i, gr = u / p.nqt, qt = u - gr * p.nqt, h = gr % p.H, b = gr / p.H;
          const bool ng_here = new_group(i);
          if (ng_here) {
            if (!mbar_wait(k_empty, (nk & 1) ^ 1, p.status, 231)) { ok = false; break; }
            mbar_arrive_expect_tx(k_full, KV_BYTES);
            tma_load_3d(smem + SMEM_K, &tmK, k_full, k_col0 + h * HD, 0, b);
            tma_load_3d(smem + SMEM_K + KV_BYTES / 2, &tmK, k_full, k_col0 + h * HD + 64, 0, b);
            ++nk;
          }
          const int qs = i % Q_STAGES;
          if (!mbar_wait(&q_empty[qs], ((i / Q_STAGES) & 1) ^ 1, p.status, 232)) { ok = false; break; }
          mbar_arrive_expect_tx(&q_full[qs], QTILE_BYTES);
          uint8_t* qb = smem + SMEM_Q + qs * QTILE_BYTES;
          tma_load_3d(qb, &tmQ, &q_full[qs], q_col0 + h * HD, qt * QT, b);
          tma_load_3d(qb + QTILE_BYTES / 2, &tmQ, &q_full[qs], q_col0 + h * HD + 64, qt * QT, b);
          ++nq;
          if (i + Q_STAGES < nmine) {  // the tile that will take this slot next, into L2 ahead of its load
            const int u3 = u + Q_STAGES, gr3 = u3 / p.nqt, qt3 = u3 - gr3 * p.nqt, h3 = gr3 % p.H, b3 = gr3 / p.H;
            tma_prefetch_3d(&tmQ, q_col0 + h3 * HD, qt3 * QT, b3);
            tma_prefetch_3d(&tmQ, q_col0 + h3 * HD + 64, qt3 * QT, b3);
          }
          if (ng_here) {
            if (!mbar_wait(v_empty, (nv & 1) ^ 1, p.status, 233)) { ok = false; break; }
            mbar_arrive_expect_tx(v_full, KV_BYTES);
            tma_load_3d(smem + SMEM_V, &tmV, v_full, v_col0 + h * HD, 0, b);
            tma_load_3d(smem + SMEM_V + KV_BYTES / 2, &tmV, v_full, v_col0 + h * HD + 64, 0, b);
            ++nv;
          }
        }
        if (!ok) {  // aborted: let the copies in flight land before the CTA exits
          if (nk > 0) mbar_wait(k_full, (nk - 1) & 1, nullptr, 0);
          if (nv > 0) mbar_wait(v_full, (nv - 1) & 1, nullptr, 0);
          for (int i = (nq > Q_STAGES ? nq - Q_STAGES : 0); i < nq; ++i)
            mbar_wait(&q_full[i % Q_STAGES], (i / Q_STAGES) & 1, nullptr, 0);
        }
      }
    } else if (warp == MMA_WARP) {
      if (lane == 0) {
        constexpr uint32_t id_s = idesc_f16(QT, KMAX, 0, 0);  // S = Q K^T, both K-major, N = 256 keys
        constexpr uint32_t id_o = idesc_f16(QT, HD, 0, 1);    // O = P V, P K-major in TMEM, V MN-major
        bool ok = true, issued = false;
        int gs = 0, gv = 0;  // groups entered by the S and by the P V sequence
        auto issue_s = [&](int i) -> bool {
          const int x = i & 1, qs = i % Q_STAGES;
          if (!mbar_wait(&q_full[qs], (i / Q_STAGES) & 1, p.status, 234)) return false;
          if (new_group(i)) {
            if (!mbar_wait(k_full, gs & 1, p.status, 235)) return false;
            ++gs;
          }
          if (i >= 2 && !mbar_wait(&o_free[x], ((i >> 1) - 1) & 1, p.status, 236)) return false;
          tc_fence_after();
          const uint32_t q0 = smem_u32(smem + SMEM_Q + qs * QTILE_BYTES), k0 = smem_u32(smem + SMEM_K);
#pragma unroll
          for (int k = 0; k < HD / 16; ++k) {
            const uint32_t qo = (k >> 2) * (QTILE_BYTES / 2) + 32 * (k & 3);
            const uint32_t ko = (k >> 2) * (KV_BYTES / 2) + 32 * (k & 3);
            mma_f16_ss(tmem + x * SLOT_COLS, sdesc_sw128(q0 + qo, 16, 1024), sdesc_sw128(k0 + ko, 16, 1024), id_s,
                       k != 0);
          }
          issued = true;
          mma_commit(&s_full[x]);
          if (last_of_group(i)) mma_commit(k_empty);
          return true;
        };
        auto issue_pv = [&](int i) -> bool {
          const int x = i & 1;
          if (new_group(i)) {
            if (!mbar_wait(v_full, gv & 1, p.status, 237)) return false;
            ++gv;
          }
          if (!mbar_wait(&p_full[x], (i >> 1) & 1, p.status, 238)) return false;
          tc_fence_after();
          const uint32_t v0 = smem_u32(smem + SMEM_V);
#pragma unroll
          for (int k = 0; k < KMAX / 16; ++k) {
            const uint64_t bd = sdesc_sw128(v0 + 2048 * k, KV_BYTES / 2, 1024);
            mma_f16_ts(tmem + x * SLOT_COLS, tmem + x * SLOT_COLS + TM_P + 8 * k, bd, id_o, k != 0);
          }
          mma_commit(&pv_done[x]);
          if (last_of_group(i)) mma_commit(v_empty);
          return true;
        };
        if (nmine > 0) ok = issue_s(0);
        for (int i = 1; i <= nmine && ok; ++i) {
          if (i < nmine && !issue_s(i)) { ok = false; break; }
          if (!issue_pv(i - 1)) { ok = false; break; }
        }
        if (!ok && issued) {
          mma_commit(drain);
          mbar_wait(drain, 0, nullptr, 0);
        }
      }
    }
  } else if (wg < 2) {
    setmaxnreg_inc<REG_SOFTMAX>();
    // softmax warps: thread = query row `row` of the tiles i with i % 2 == wg
    const int x = wg, g4 = warp & 3;
    const int row = g4 * 32 + lane;
    const uint32_t tS = tmem + (static_cast<uint32_t>(g4 * 32) << 16) + x * SLOT_COLS;
    const int limit = p.nvalid;  // keys >= limit are masked
    const bool full = limit >= KMAX;
    const uint64_t scale2 = f2pack(p.scale_log2, p.scale_log2);
    uint32_t s[128];
    bool ok = true;
    for (int i = x; i < nmine && ok; i += 2) {
      const uint32_t ph = (i >> 1) & 1;
      if (!warp_wait(&s_full[x], ph, p.status, 239)) { ok = false; break; }
      tc_fence_after();
      float mxp[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) mxp[t] = -INFINITY;
      // first read: the maximum over all 256 keys (keys 0-127, then 128-255, which stay in s)
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tS + 128 * half + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(s + 32 * c));
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (full)
            max32<true>(mxp, *reinterpret_cast<uint32_t(*)[32]>(s + 32 * c), 128 * half + 32 * c, limit);
          else
            max32<false>(mxp, *reinterpret_cast<uint32_t(*)[32]>(s + 32 * c), 128 * half + 32 * c, limit);
        }
      }
      const float mt =
          fmax3(fmax3(mxp[0], mxp[1], mxp[2]), fmax3(mxp[3], mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])) * p.scale_log2;
      const float m = mt == -INFINITY ? 0.f : mt;
      const uint64_t negm2 = f2pack(-m, -m);
      uint64_t sum2[4] = {0, 0, 0, 0};
      // keys 128-255 from registers: P into columns [192, 256), S columns read already; the probabilities
      // go back into s (fp32) and are summed once the half's P is stored
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
        if (full)
          exp32_keep<true>(pk, *reinterpret_cast<uint32_t(*)[32]>(s + 32 * c), scale2, negm2, 128 + 32 * c, limit);
        else
          exp32_keep<false>(pk, *reinterpret_cast<uint32_t(*)[32]>(s + 32 * c), scale2, negm2, 128 + 32 * c, limit);
        tmem_st16(tS + TM_P + 64 + 16 * c, pk);
      }
#pragma unroll
      for (int t = 0; t < 128; t += 2)
        sum2[(t >> 1) & 3] = fadd2(sum2[(t >> 1) & 3], f2pack(__uint_as_float(s[t]), __uint_as_float(s[t + 1])));
      // keys 0-127 read again: P into columns [128, 192) (S of keys 128-191, in registers above)
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(s + 32 * c));
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
        if (full)
          exp32_keep<true>(pk, *reinterpret_cast<uint32_t(*)[32]>(s + 32 * c), scale2, negm2, 32 * c, limit);
        else
          exp32_keep<false>(pk, *reinterpret_cast<uint32_t(*)[32]>(s + 32 * c), scale2, negm2, 32 * c, limit);
        tmem_st16(tS + TM_P + 16 * c, pk);
      }
#pragma unroll
      for (int t = 0; t < 128; t += 2)
        sum2[(t >> 1) & 3] = fadd2(sum2[(t >> 1) & 3], f2pack(__uint_as_float(s[t]), __uint_as_float(s[t + 1])));
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[x]);
      const uint64_t s01 = fadd2(fadd2(sum2[0], sum2[1]), fadd2(sum2[2], sum2[3]));
      float slo, shi;
      f2unpack(s01, slo, shi);
      const float l = slo + shi;
      // the epilogue of the tile by the same threads: O = P V read from TMEM in one go (the slot is then
      // released to the next S at once), scaled by 1 / l and stored while the tensor pipe goes on
      if (!warp_wait(&pv_done[x], ph, p.status, 242)) { ok = false; break; }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(s + 32 * c));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[x]);
      // O / l as fp16 into the tile's Q slot (S(i) has read it), in the 128-byte swizzled layout of a
      // Q load, then one TMA store per 64 columns: row-contiguous writes instead of 16-byte pieces of
      // 128 rows. The slot goes back to the Q ring once the store has read it.
      const int qs = i % Q_STAGES;
      uint8_t* ob = smem + SMEM_Q + qs * QTILE_BYTES;
      const uint32_t orow = smem_u32(ob) + row * 128;
      const float inv = l > 0.f ? 1.0f / l : 0.f;
#pragma unroll
      for (int w = 0; w < HD / 8; ++w) {
        const uint32_t* v = s + 8 * w;
        st_shared_v4(orow + (w >> 3) * (QTILE_BYTES / 2) + (((w & 7) ^ (row & 7)) << 4),
                     pack_half2(__uint_as_float(v[0]) * inv, __uint_as_float(v[1]) * inv),
                     pack_half2(__uint_as_float(v[2]) * inv, __uint_as_float(v[3]) * inv),
                     pack_half2(__uint_as_float(v[4]) * inv, __uint_as_float(v[5]) * inv),
                     pack_half2(__uint_as_float(v[6]) * inv, __uint_as_float(v[7]) * inv));
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_staged[x]);
      bool stored = true;
      if (g4 == 0 && lane == 0) {
        stored = mbar_wait(&o_staged[x], ph, p.status, 243);
        if (stored) {
          const int u = u0 + i, gr = u / p.nqt, qt = u - gr * p.nqt, h = gr % p.H, b = gr / p.H;
          tma_store_3d(&tmO, ob, h * HD, qt * QT, b);  // rows >= Tq are not written
          tma_store_3d(&tmO, ob + QTILE_BYTES / 2, h * HD + 64, qt * QT, b);
          bulk_commit();
          bulk_wait_read<0>();
          mbar_arrive(&q_empty[qs]);
        }
      }
      if (g4 == 0) stored = __all_sync(0xffffffffu, stored);  // the warp leaves the loop together
      if (!stored) { ok = false; break; }
    }
    if (g4 == 0 && lane == 0) bulk_wait<0>();  // the last stores complete before the CTA exits
  } else {
    setmaxnreg_dec<REG_IDLE>();  // warpgroup 2: idle
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == MMA_WARP) tmem_dealloc(tmem, 512);
}

}  // namespace

// Tk <= 256 only; the caller (attn_launch) validates the common arguments
cudaError_t attn_short_launch(const AttnArgs& a, cudaStream_t s) {
  if (a.Tk > KMAX) return cudaErrorInvalidValue;
  CUtensorMap tQ, tK, tV, tO;
  const uint64_t op = static_cast<uint64_t>(a.ldo) * 2;
  const uint64_t qp = static_cast<uint64_t>(a.ldq) * 2, kp = static_cast<uint64_t>(a.ldk) * 2,
                 vp = static_cast<uint64_t>(a.ldv) * 2;
  // K and V boxes of 256 rows: keys >= Tk are zero-filled by the copy and masked in the softmax
  if (!make_tmap_3d(&tQ, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.q, a.ldq, a.Tq, a.B, qp, qp * a.Tq, 64, QT, 1,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_3d(&tK, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.k, a.ldk, a.Tk, a.B, kp, kp * a.Tk, 64, KMAX, 1,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_3d(&tV, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.v, a.ldv, a.Tk, a.B, vp, vp * a.Tk, 64, KMAX, 1,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_3d(&tO, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.o, a.ldo, a.Tq, a.B, op, op * a.Tq, 64, QT, 1,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  static uint64_t attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set >> dev & 1)) {
    cudaError_t e = cudaFuncSetAttribute(attn_short_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SH_SMEM);
    if (e != cudaSuccess) return e;
    attr_set |= 1ull << dev;
  }
  SParams p;
  p.Tq = a.Tq;
  p.nvalid = (a.nvalid > 0 && a.nvalid < a.Tk) ? a.nvalid : a.Tk;
  p.H = a.H;
  p.nqt = (a.Tq + QT - 1) / QT;
  const long long units = static_cast<long long>(p.nqt) * a.H * a.B;
  if (units > (1LL << 30)) return cudaErrorInvalidValue;
  p.U = static_cast<int>(units);
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.o = a.o;
  p.ldo = a.ldo;
  p.status = a.status;
  const int grid = static_cast<int>(units < sm_count() ? units : sm_count());
  const cudaError_t e = launch_pdl(attn_short_kernel, dim3(grid), dim3(SH_THREADS), SH_SMEM, s, tQ, tK, tV, tO, p,
                                   a.q_col0, a.k_col0, a.v_col0);
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace hx

// C ABI of libhxdit.so (declared in include/hxdit.h): handles, device buffers, weight sets, the
// per-block operator and the chain runner.
//
// Block orchestration follows the reference site order:
//  Anima  mega_block_impl, hexagon/mega/blk.c:148-175 (three sites: self-attn, cross-attn, MLP)
//  MOSS   mode 0, moss/hexagon/mega/blk.c:234-259 (RMS-mod, LoRA-A, QKV+RMS+RoPE, joint attention,
//         O + gate, RMS-mod, up_gate + SiTU, down + gate)
// Fusions relative to the reference: q/k RMS+RoPE run in the QKV GEMM epilogue (blk.c:159-160 ran a
// separate pass), residual+gate in the O/CO/M2 epilogues, GELU in M1, SiTU in up_gate; q|k|v and
// ck|cv are one GEMM each; the K=8192 down projection runs as one K loop (blk.c:172-174 split it).
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <vector>

#include "../../include/hxdit.h"
#include "hx_internal.h"
#include "hx_sp.h"

using namespace hx;

namespace {

constexpr size_t kAnimaPackF16 = 138416128u;  // W_TOTAL, hexagon/mega/blk_wlayout.h:15
constexpr size_t kAnimaModW = 125833216u;     // W_MODW
constexpr size_t kAnimaGain = 125829120u;     // W_GAIN
inline size_t wq(size_t x) { return x / 2048u * 1152u; }  // WQ(), blk_wlayout.h:17
constexpr size_t kMossPack = 135397376u;      // W_TOTAL, moss/hexagon/mega/blk_meta.h:17

struct Weights {
  int model = 0, D = 0, F = 0, Cd = 0, H = 0, lora = 0;
  int proj = 0;  // MOSS text projection weights (MODE 2 only): W_O = [D][Cd + 128], Cd = text width
  DevMat mats[HX_NMATS];
  bool has[HX_NMATS] = {};
  const float* gain = nullptr;
  const __half* modA = nullptr;
  const __half* modB = nullptr;
  std::vector<void*> owned;  // device allocations owned by the handle
};

struct Buf {
  void* ptr = nullptr;
  size_t bytes = 0;
};

struct Glue {
  int D = 0;
  __half *t_norm = nullptr, *t_lin1 = nullptr, *t_lin2 = nullptr, *x_emb = nullptr /* [D][128], K padded */,
         *f_modA = nullptr, *f_modB = nullptr, *f_lin = nullptr;
  std::vector<void*> owned;
};

// Device scratch of the sampler, grown on demand (never inside a graph capture).
struct MossGlue {
  int D = 0;
  __half *t_lin0 = nullptr, *t_lin2 = nullptr, *mod_w = nullptr, *head_w = nullptr, *fin_w = nullptr,
         *emb = nullptr /* [D][192]: video_embedder with the bias in column 128 */;
  float *t_b0 = nullptr, *t_b2 = nullptr, *mod_b = nullptr, *head_b = nullptr, *fin_norm = nullptr, *Q = nullptr;
  std::vector<void*> owned;
};
constexpr int kMossEmbK = 192;  // 128 latent channels + the bias column, padded to the GEMM's K step

// Device scratch of the MOSS sampler, grown on demand (never inside a graph capture).
struct MossScratch {
  int D = 0;
  size_t rows = 0;
  float *e = nullptr, *a = nullptr, *tm = nullptr, *mod = nullptr, *head = nullptr, *v = nullptr;
  __half* xin = nullptr;
  void release() {
    for (void* p : {(void*)e, (void*)a, (void*)tm, (void*)mod, (void*)head, (void*)v, (void*)xin}) cudaFree(p);
    *this = MossScratch();
  }
};

struct SampleScratch {
  int S = 0, D = 0;
  size_t rows = 0;
  float *tp = nullptr, *emb = nullptr, *tmp = nullptr, *lora = nullptr, *h256 = nullptr, *fmod = nullptr,
        *y = nullptr;
  __half* P = nullptr;
  __half* ckv = nullptr;  // cross-attention k|v of every block, computed once per sample
  size_t ckv_elems = 0;
  const __half** modtab = nullptr;  // device: the blocks' AdaLN A weights, then their B weights
  std::vector<const __half*> modtab_host;
  float* se = nullptr;              // silu(emb) of the current step
  void release() {
    for (void* p : {(void*)tp, (void*)emb, (void*)tmp, (void*)lora, (void*)h256, (void*)fmod, (void*)y, (void*)P,
                    (void*)ckv, (void*)modtab, (void*)se})
      cudaFree(p);
    *this = SampleScratch();
  }
};

struct ChainGraph {
  std::vector<int64_t> key;
  cudaGraphExec_t exec = nullptr;
  uint64_t last_use = 0;
};
constexpr size_t kMaxGraphs = 16;  // e.g. one per denoising step of a sampler

}  // namespace

struct Adapter {
  AdapterWeights w;
  std::vector<void*> owned;
};

struct hx_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = true;
  int* status = nullptr;  // device word
  std::map<int, Buf> bufs;
  std::map<int, std::unique_ptr<Weights>> weights;
  int next_fd = 1;
  float* modscratch = nullptr;  // chain modulation vectors
  size_t modscratch_floats = 0;
  __half* wexp = nullptr;  // fp16 expansion of one quantised matrix before its GEMM (stream-ordered)
  size_t wexp_bytes = 0;
  // expansions issued ahead of their GEMMs (Anima chain): two fp16 buffers used in turn, filled on a side
  // stream that forks from and joins back into `stream` through the events below
  __half* xbuf[2] = {nullptr, nullptr};
  size_t xbuf_bytes = 0;
  cudaStream_t xstream = nullptr;
  cudaEvent_t xev_fork = nullptr, xev_read[2] = {nullptr, nullptr}, xev_ready[2] = {nullptr, nullptr};
  cudaEvent_t ev[34] = {};
  cudaEvent_t spev[4] = {};  // Ulysses attention parts of the last timed block (times[17..19])
  bool spev_used = false;
  std::vector<ChainGraph> graphs;
  uint64_t graph_clock = 0;
  std::map<int, std::unique_ptr<Glue>> glues;
  SampleScratch ss;
  std::map<int, std::unique_ptr<MossGlue>> moss_glues;
  std::map<int, std::unique_ptr<Adapter>> adapters;
  MossScratch ms;
  hx::SpState sp;
  std::mutex mu;
  void drop_graphs() {
    for (auto& g : graphs)
      if (g.exec) cudaGraphExecDestroy(g.exec);
    graphs.clear();
  }
};

namespace {

#define CK(call)                                  \
  do {                                            \
    cudaError_t e_ = (call);                      \
    if (e_ != cudaSuccess) {                      \
      if (getenv("HX_DEBUG"))                     \
        fprintf(stderr, "hxdit: %s:%d %s -> %s\n", __FILE__, __LINE__, #call, cudaGetErrorString(e_)); \
      return HX_E_CUDA;                           \
    }                                             \
  } while (0)

struct DevGuard {
  int prev = -1;
  explicit DevGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DevGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

DevMat to_devmat(const hx_mat& m) {
  DevMat d;
  d.fmt = m.fmt;
  d.N = m.n;
  d.K = m.k;
  d.group = m.group ? m.group : (m.fmt == HX_FMT_F16 ? 64 : 32);
  d.w = m.w;
  d.scale = static_cast<__half*>(m.scale);
  d.minv = static_cast<__half*>(m.minv);
  return d;
}

bool valid_mat(const hx_mat& m) {
  if (!m.w || m.n <= 0 || m.k <= 0) return false;
  if (m.fmt != HX_FMT_F16 && !m.scale) return false;
  if (m.fmt == HX_FMT_Q4A && !m.minv) return false;
  return m.fmt >= 0 && m.fmt <= 3;
}

// ---------------------------------------------------------------- pack loading
int alloc_mat(Weights& W, int slot, int fmt, int N, int K, int group) {
  DevMat& d = W.mats[slot];
  d.fmt = fmt;
  d.N = N;
  d.K = K;
  d.group = group;
  const size_t wbytes = fmt == HX_FMT_F16 ? static_cast<size_t>(N) * K * 2 : static_cast<size_t>(N) * K;
  void* p = nullptr;
  CK(cudaMalloc(&p, wbytes));
  W.owned.push_back(p);
  d.w = p;
  if (fmt == HX_FMT_Q8) {
    void* s = nullptr;
    CK(cudaMalloc(&s, static_cast<size_t>(K / group) * N * 2));
    W.owned.push_back(s);
    d.scale = static_cast<__half*>(s);
  }
  W.has[slot] = true;
  return HX_OK;
}

// copy `bytes` of the pack at `off` into device staging, then repack `nb x kb` tiles into slot rows
int repack_into(Weights& W, int slot, const uint8_t* dpack, size_t off, int nb, int kb, bool q8, int row0, int mode,
                cudaStream_t s) {
  DevMat& d = W.mats[slot];
  CK(repack_tiles_launch(dpack + off, nb, kb, q8, d.w, d.scale, row0, d.N, mode, s));
  return HX_OK;
}

int load_anima(hx_ctx* h, const uint8_t* pack, size_t bytes, Weights& W) {
  const bool q8 = bytes == wq(kAnimaGain) + 4096 + (kAnimaPackF16 - kAnimaModW);
  if (!q8 && bytes != kAnimaPackF16) return HX_E_FORMAT;
  const int D = 2048, Cd = 1024, F = 8192;
  W.model = HX_MODEL_ANIMA;
  W.D = D;
  W.F = F;
  W.Cd = Cd;
  W.H = 16;
  const int fmt = q8 ? HX_FMT_Q8 : HX_FMT_F16;
  int rc;
  if ((rc = alloc_mat(W, HX_W_QKV, fmt, 3 * D, D, 32)) || (rc = alloc_mat(W, HX_W_O, fmt, D, D, 32)) ||
      (rc = alloc_mat(W, HX_W_CQ, fmt, D, D, 32)) || (rc = alloc_mat(W, HX_W_CKV, fmt, 2 * D, Cd, 32)) ||
      (rc = alloc_mat(W, HX_W_CO, fmt, D, D, 32)) || (rc = alloc_mat(W, HX_W_M1, fmt, F, D, 32)) ||
      (rc = alloc_mat(W, HX_W_M2, fmt, D, F, 32)))
    return rc;
  uint8_t* dpack = nullptr;
  CK(cudaMalloc(&dpack, bytes));
  CK(cudaMemcpyAsync(dpack, pack, bytes, cudaMemcpyHostToDevice, h->stream));
  // order of export_all.py:9 and offsets of blk_wlayout.h:3-12 (fp16) / WQ() (q8)
  struct M { size_t off; int slot, nb, kb, row0; };
  const size_t f16off[10] = {0u, 8388608u, 16777216u, 25165824u, 33554432u, 41943040u, 46137344u, 50331648u,
                             58720256u, 92274688u};
  auto O = [&](int i) { return q8 ? wq(f16off[i]) : f16off[i]; };
  const M list[10] = {{O(0), HX_W_QKV, 64, 64, 0},      {O(1), HX_W_QKV, 64, 64, D},  {O(2), HX_W_QKV, 64, 64, 2 * D},
                      {O(3), HX_W_O, 64, 64, 0},        {O(4), HX_W_CQ, 64, 64, 0},   {O(5), HX_W_CKV, 64, 32, 0},
                      {O(6), HX_W_CKV, 64, 32, D},      {O(7), HX_W_CO, 64, 64, 0},   {O(8), HX_W_M1, 256, 64, 0},
                      {O(9), HX_W_M2, 64, 256, 0}};
  for (const M& m : list) {
    if ((rc = repack_into(W, m.slot, dpack, m.off, m.nb, m.kb, q8, m.row0, 0, h->stream))) {
      cudaFree(dpack);
      return rc;
    }
  }
  const size_t goff = q8 ? wq(kAnimaGain) : kAnimaGain, moff = q8 ? wq(kAnimaGain) + 4096 : kAnimaModW;
  float* gain = nullptr;
  __half *mA = nullptr, *mB = nullptr;
  CK(cudaMalloc(&gain, 512 * 4));
  CK(cudaMalloc(&mA, 3ull * 256 * D * 2));
  CK(cudaMalloc(&mB, 3ull * 6144 * 256 * 2));
  W.owned.push_back(gain);
  W.owned.push_back(mA);
  W.owned.push_back(mB);
  CK(cudaMemcpyAsync(gain, dpack + goff, 512 * 4, cudaMemcpyDeviceToDevice, h->stream));
  const size_t sa = 256ull * D * 2, sb = 6144ull * 256 * 2;
  for (int site = 0; site < 3; ++site) {  // per site: a[256][2048] then b[6144][256] (export_all.py:34-36)
    CK(cudaMemcpyAsync(reinterpret_cast<uint8_t*>(mA) + site * sa, dpack + moff + site * (sa + sb), sa,
                       cudaMemcpyDeviceToDevice, h->stream));
    CK(cudaMemcpyAsync(reinterpret_cast<uint8_t*>(mB) + site * sb, dpack + moff + site * (sa + sb) + sa, sb,
                       cudaMemcpyDeviceToDevice, h->stream));
  }
  W.gain = gain;
  W.modA = mA;
  W.modB = mB;
  CK(cudaStreamSynchronize(h->stream));
  CK(cudaFree(dpack));
  return HX_OK;
}

int load_moss(hx_ctx* h, const uint8_t* pack, size_t bytes, Weights& W) {
  if (bytes != kMossPack) return HX_E_FORMAT;
  const int D = 3072, F = 8192;
  W.model = HX_MODEL_MOSS;
  W.D = D;
  W.F = F;
  W.H = 24;
  W.lora = 1;
  int rc;
  const int K1 = D + 128;
  if ((rc = alloc_mat(W, HX_W_Q, HX_FMT_Q8, D, K1, 32)) || (rc = alloc_mat(W, HX_W_K, HX_FMT_Q8, D, K1, 32)) ||
      (rc = alloc_mat(W, HX_W_V, HX_FMT_Q8, D, K1, 32)) || (rc = alloc_mat(W, HX_W_O, HX_FMT_Q8, D, K1, 32)) ||
      (rc = alloc_mat(W, HX_W_M1, HX_FMT_Q8, 2 * F, K1, 32)) ||
      (rc = alloc_mat(W, HX_W_M2, HX_FMT_Q8, D, F + 128, 32)) ||
      (rc = alloc_mat(W, HX_W_AQKV, HX_FMT_Q8, 384, D, 32)) || (rc = alloc_mat(W, HX_W_AO, HX_FMT_Q8, 128, D, 32)) ||
      (rc = alloc_mat(W, HX_W_AUG, HX_FMT_Q8, 128, D, 32)) || (rc = alloc_mat(W, HX_W_ADN, HX_FMT_Q8, 128, F, 32)))
    return rc;
  uint8_t* dpack = nullptr;
  CK(cudaMalloc(&dpack, bytes));
  CK(cudaMemcpyAsync(dpack, pack, bytes, cudaMemcpyHostToDevice, h->stream));
  // offsets of moss/hexagon/mega/blk_meta.h:6-16
  struct M { size_t off; int slot, nb, kb, mode; };
  const M list[10] = {{0u, HX_W_Q, 96, 100, 0},          {11059200u, HX_W_K, 96, 100, 0},
                      {22118400u, HX_W_V, 96, 100, 0},   {33177600u, HX_W_O, 96, 100, 0},
                      {44236800u, HX_W_M1, 512, 100, 1}, {103219200u, HX_W_M2, 96, 260, 0},
                      {131973120u, HX_W_AQKV, 12, 96, 0}, {133300224u, HX_W_AO, 4, 96, 0},
                      {133742592u, HX_W_AUG, 4, 96, 0},  {134184960u, HX_W_ADN, 4, 256, 0}};
  for (const M& m : list) {
    if ((rc = repack_into(W, m.slot, dpack, m.off, m.nb, m.kb, true, 0, m.mode, h->stream))) {
      cudaFree(dpack);
      return rc;
    }
  }
  float* gain = nullptr;
  CK(cudaMalloc(&gain, (256 + 2 * D) * 4));
  W.owned.push_back(gain);
  CK(cudaMemcpyAsync(gain, dpack + 135364608u, (256 + 2 * D) * 4, cudaMemcpyDeviceToDevice, h->stream));
  W.gain = gain;
  CK(cudaStreamSynchronize(h->stream));
  CK(cudaFree(dpack));
  return HX_OK;
}

// MOSS text projection pack (export_moss.py:61-65 `pack_proj`): [96 nb][132 kb] q8 tiles of
// [Wp^T ; bias row, 127 zero rows] at offset 0, padded with zeros to the block-pack size.
int load_moss_proj(hx_ctx* h, const uint8_t* pack, size_t bytes, Weights& W) {
  const int D = 3072, TW = 4096;
  const size_t need = static_cast<size_t>(D / 32) * ((TW + 128) / 32) * 1152;
  if (bytes != kMossPack && bytes != need) return HX_E_FORMAT;
  W.model = HX_MODEL_MOSS;
  W.proj = 1;
  W.D = D;
  W.F = 8192;
  W.Cd = TW;
  W.H = 24;
  W.lora = 1;
  int rc;
  if ((rc = alloc_mat(W, HX_W_O, HX_FMT_Q8, D, TW + 128, 32))) return rc;
  uint8_t* dpack = nullptr;
  CK(cudaMalloc(&dpack, need));
  CK(cudaMemcpyAsync(dpack, pack, need, cudaMemcpyHostToDevice, h->stream));
  rc = repack_into(W, HX_W_O, dpack, 0, D / 32, (TW + 128) / 32, true, 0, 0, h->stream);
  cudaStreamSynchronize(h->stream);
  cudaFree(dpack);
  return rc;
}

// ---------------------------------------------------------------- block orchestration
class Lookahead;

struct Stage {
  hx_ctx* h;
  int ntimes;
  int ti = 0;
  int stop;
  bool stopped = false;
  const __half* ckv_pre = nullptr;  // Anima: this block's cross-attention k|v already computed (sampler cache)
  Lookahead* xa = nullptr;          // Anima chain: weight expansions issued ahead (nullptr: one per block)
  const Weights* next = nullptr;    // Anima chain: the next block, whose q|k|v expansion the last GEMM issues
  // returns true when the caller must stop (meta STOP reached)
  bool tick() {
    if (ntimes > 0 && ti < 32) cudaEventRecord(h->ev[ti + 1], h->stream);
    ++ti;
    if (stop && ti >= stop) stopped = true;
    return stopped;
  }
};

inline const float* fptr(const uint8_t* blob, int off) { return reinterpret_cast<const float*>(blob + off); }
inline __half* hptr(uint8_t* blob, int off) { return reinterpret_cast<__half*>(blob + off); }

#define CKL(call)                                   \
  do {                                              \
    cudaError_t e_ = (call);                        \
    if (e_ != cudaSuccess) {                        \
      if (getenv("HX_DEBUG"))                       \
        fprintf(stderr, "hxdit: %s:%d %s -> %s\n", __FILE__, __LINE__, #call, cudaGetErrorString(e_)); \
      return e_ == cudaErrorInvalidValue ? HX_E_ARG : HX_E_CUDA; \
    }                                               \
  } while (0)

GemmArgs gargs(hx_ctx* h, const __half* A, int lda, int M, const DevMat* W, int epi) {
  GemmArgs g;
  g.wexp = h->wexp;
  g.wexp_bytes = h->wexp_bytes;
  g.A = A;
  g.lda = lda;
  g.M = M;
  g.K1 = W->K;
  g.W = W;
  g.epi = epi;
  g.status = h->status;
  return g;
}

// Grow the weight-expansion scratch to `bytes` (outside graph capture only; captured graphs hold the old
// pointer and are dropped). A failed allocation leaves no scratch: the GEMMs then dequantise in-kernel.
void reserve_wexp(hx_ctx* h, size_t bytes) {
  if (bytes <= h->wexp_bytes) return;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(h->stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return;
  cudaStreamSynchronize(h->stream);
  h->drop_graphs();
  cudaFree(h->wexp);
  h->wexp = nullptr;
  h->wexp_bytes = 0;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  h->wexp = static_cast<__half*>(p);
  h->wexp_bytes = bytes;
}

// Grow the two look-ahead expansion buffers to `bytes` each (outside graph capture; drops captured
// graphs). On failure there are none and the chain expands in line.
void reserve_xbuf(hx_ctx* h, size_t bytes) {
  if (bytes <= h->xbuf_bytes || !h->xstream) return;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(h->stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return;
  cudaStreamSynchronize(h->stream);
  cudaStreamSynchronize(h->xstream);
  h->drop_graphs();
  for (auto& b : h->xbuf) {
    cudaFree(b);
    b = nullptr;
  }
  h->xbuf_bytes = 0;
  void* p0 = nullptr;
  void* p1 = nullptr;
  if (cudaMalloc(&p0, bytes) != cudaSuccess || cudaMalloc(&p1, bytes) != cudaSuccess) {
    cudaFree(p0);
    cudaGetLastError();
    return;
  }
  h->xbuf[0] = static_cast<__half*>(p0);
  h->xbuf[1] = static_cast<__half*>(p1);
  h->xbuf_bytes = bytes;
}

// Quantised weights expanded to fp16 ahead of their GEMMs. The expansion for a GEMM runs on the handle's
// side stream into one of two buffers used in turn; it is issued as soon as the GEMM before has been
// enqueued and waits only for the GEMM that last read its buffer (two GEMMs back), so it runs under the
// kernels in between (the norm, the attention) instead of in front of its own GEMM. The GEMM waits for it
// through an event. The same policy as the in-line expansion of gemm_launch decides which GEMMs expand.
class Lookahead {
 public:
  explicit Lookahead(hx_ctx* h) : h_(h) {}
  Lookahead(const Lookahead&) = delete;
  Lookahead& operator=(const Lookahead&) = delete;
  ~Lookahead() { finish(); }
  // issue the expansion of W for a GEMM of M rows (a no-op when it is already issued or does not apply)
  cudaError_t issue(const DevMat& W, int M) {
    if (armed_ && src_ == &W) return cudaSuccess;
    if (armed_) {  // an expansion nobody consumed: join it before reusing the state
      cudaError_t e = finish();
      if (e != cudaSuccess) return e;
    }
    const size_t need = static_cast<size_t>(W.N) * W.K * 2;
    if (W.fmt == WF_F16 || M < expand_min_rows() || !h_->xstream || !h_->xbuf[1] || h_->xbuf_bytes < need)
      return cudaSuccess;
    cudaError_t e;
    if (!started_) {  // fork: the side stream follows everything enqueued on the main stream so far
      if ((e = cudaEventRecord(h_->xev_fork, h_->stream)) != cudaSuccess) return e;
      if ((e = cudaStreamWaitEvent(h_->xstream, h_->xev_fork, 0)) != cudaSuccess) return e;
      started_ = true;
    }
    const int b = next_;
    next_ ^= 1;
    if (read_[b] && (e = cudaStreamWaitEvent(h_->xstream, h_->xev_read[b], 0)) != cudaSuccess) return e;
    if ((e = expand_launch(W, h_->xbuf[b], h_->xstream)) != cudaSuccess) return e;
    if ((e = cudaEventRecord(h_->xev_ready[b], h_->xstream)) != cudaSuccess) return e;
    armed_ = true;
    src_ = &W;
    buf_ = b;
    view_ = DevMat();
    view_.fmt = WF_F16;
    view_.N = W.N;
    view_.K = W.K;
    view_.group = 64;
    view_.w = h_->xbuf[b];
    return cudaSuccess;
  }
  // the GEMM g on the main stream, on the expansion issued for g.W if there is one
  cudaError_t gemm(GemmArgs g) {
    const bool use = armed_ && src_ == g.W;
    cudaError_t e;
    if (use) {
      if ((e = cudaStreamWaitEvent(h_->stream, h_->xev_ready[buf_], 0)) != cudaSuccess) return e;
      g.W = &view_;
    }
    if ((e = gemm_launch(g, h_->stream)) != cudaSuccess) return e;
    if (use) {
      if ((e = cudaEventRecord(h_->xev_read[buf_], h_->stream)) != cudaSuccess) return e;
      read_[buf_] = true;
      armed_ = false;
    }
    return cudaSuccess;
  }
  // join an expansion that no GEMM consumed (the side stream must end joined, e.g. inside a capture)
  cudaError_t finish() {
    if (!armed_) return cudaSuccess;
    armed_ = false;
    return cudaStreamWaitEvent(h_->stream, h_->xev_ready[buf_], 0);
  }

 private:
  hx_ctx* h_;
  bool started_ = false, armed_ = false;
  bool read_[2] = {false, false};  // a GEMM reading buffer b was enqueued after the fork
  int next_ = 0, buf_ = 0;
  const DevMat* src_ = nullptr;
  DevMat view_;
};

// the scratch a weight set needs: its largest quantised matrix as fp16
size_t wexp_need(const Weights& W) {
  size_t need = 0;
  for (int i = 0; i < HX_NMATS; ++i)
    if (W.has[i] && W.mats[i].fmt != WF_F16)
      need = std::max(need, static_cast<size_t>(W.mats[i].N) * W.mats[i].K * 2);
  return need;
}

// cross-attention k|v of one Anima block: [rows][2D] fp16, k RMS-normalised with the ck gain
cudaError_t ckv_launch(hx_ctx* h, const Weights& W, const __half* ctx, int rows, __half* out) {
  GemmArgs gk = gargs(h, ctx, W.Cd, rows, &W.mats[HX_W_CKV], EPI_RMS);
  gk.out = out;
  gk.ldo = 2 * W.D;
  gk.gain0 = W.gain + 384;
  gk.seg1 = gk.seg2 = W.D;
  return gemm_launch(gk, h->stream);
}

int anima_block(hx_ctx* h, const Weights& W, const int32_t* meta, uint8_t* blob, const float* mod, Stage& st) {
  const int D = W.D, F = W.F, Cd = W.Cd, H = W.H;
  const int T = meta[HX_A_NTOK], C = meta[HX_A_NCTX];
  const int B = meta[HX_A_BATCH] > 0 ? meta[HX_A_BATCH] : 1;
  const int rows = B * T;
  cudaStream_t s = h->stream;
  float* x = reinterpret_cast<float*>(blob + meta[HX_A_X]);
  __half* hbuf = hptr(blob, meta[HX_A_H]);
  __half* qkv = hptr(blob, meta[HX_A_Q]);
  __half* obuf = hptr(blob, meta[HX_A_O]);
  __half* mid = hptr(blob, meta[HX_A_MID]);
  __half* ckv = hptr(blob, meta[HX_A_CK]);
  const __half* ctx = hptr(blob, meta[HX_A_CTX]);
  const float* cosT = fptr(blob, meta[HX_A_COS]);
  const float* sinT = fptr(blob, meta[HX_A_SIN]);
  const float* gain = W.gain;
  Lookahead local(h);
  Lookahead& X = st.xa ? *st.xa : local;
  CKL(X.issue(W.mats[HX_W_QKV], rows));
  for (int site = 0; site < 3; ++site) {
    const float* sh = mod + (site * 3 + 0) * D;
    const float* sc = mod + (site * 3 + 1) * D;
    const float* gt = mod + (site * 3 + 2) * D;
    CKL(lnmod_launch(x, hbuf, rows, D, sh, sc, 0, T, 1e-6f, s));
    if (st.tick()) return HX_OK;
    if (site == 0) {
      GemmArgs g = gargs(h, hbuf, D, rows, &W.mats[HX_W_QKV], EPI_RMS);
      g.out = qkv;
      g.ldo = 3 * D;
      g.gain0 = gain;
      g.gain1 = gain + 128;
      g.seg1 = D;
      g.seg2 = 2 * D;
      g.rope0 = g.rope1 = 1;
      g.cosT = cosT;
      g.sinT = sinT;
      g.rows_per_img = T;
      CKL(X.gemm(g));
      CKL(X.issue(W.mats[HX_W_O], rows));
      if (st.tick()) return HX_OK;
      if (st.tick()) return HX_OK;  // rope slot: fused into the QKV epilogue
      AttnArgs a;
      a.q = qkv; a.ldq = 3 * D; a.q_col0 = 0;
      a.k = qkv; a.ldk = 3 * D; a.k_col0 = D;
      a.v = qkv; a.ldv = 3 * D; a.v_col0 = 2 * D;
      a.o = obuf; a.ldo = D;
      a.B = B; a.H = H; a.Tq = T; a.Tk = T;
      a.status = h->status;
      CKL(attn_launch(a, s));
      if (st.tick()) return HX_OK;
      GemmArgs go = gargs(h, obuf, D, rows, &W.mats[HX_W_O], EPI_RESID);
      go.x = x;
      go.ldx = D;
      go.gate = gt;
      CKL(X.gemm(go));
      CKL(X.issue(W.mats[HX_W_CQ], rows));
      if (st.tick()) return HX_OK;
    } else if (site == 1) {
      GemmArgs gq = gargs(h, hbuf, D, rows, &W.mats[HX_W_CQ], EPI_RMS);
      gq.out = qkv;
      gq.ldo = 3 * D;
      gq.gain0 = gain + 256;
      gq.seg1 = gq.seg2 = D;
      CKL(X.gemm(gq));
      CKL(X.issue(W.mats[HX_W_CO], rows));
      if (st.ckv_pre) {
        ckv = const_cast<__half*>(st.ckv_pre);
      } else {
        CKL(ckv_launch(h, W, ctx, B * C, ckv));
      }
      if (st.tick()) return HX_OK;
      if (st.tick()) return HX_OK;  // rms slot: fused into the two GEMMs above
      AttnArgs a;
      a.q = qkv; a.ldq = 3 * D; a.q_col0 = 0;
      a.k = ckv; a.ldk = 2 * D; a.k_col0 = 0;
      a.v = ckv; a.ldv = 2 * D; a.v_col0 = D;
      a.o = obuf; a.ldo = D;
      a.B = B; a.H = H; a.Tq = T; a.Tk = C;
      a.status = h->status;
      CKL(attn_launch(a, s));
      if (st.tick()) return HX_OK;
      GemmArgs go = gargs(h, obuf, D, rows, &W.mats[HX_W_CO], EPI_RESID);
      go.x = x;
      go.ldx = D;
      go.gate = gt;
      CKL(X.gemm(go));
      CKL(X.issue(W.mats[HX_W_M1], rows));
      if (st.tick()) return HX_OK;
    } else {
      GemmArgs g1 = gargs(h, hbuf, D, rows, &W.mats[HX_W_M1], EPI_GELU);
      g1.out = mid;
      g1.ldo = F;
      CKL(X.gemm(g1));
      CKL(X.issue(W.mats[HX_W_M2], rows));
      if (st.tick()) return HX_OK;
      GemmArgs g2 = gargs(h, mid, F, rows, &W.mats[HX_W_M2], EPI_RESID);
      g2.x = x;
      g2.ldx = D;
      g2.gate = gt;
      CKL(X.gemm(g2));
      if (st.next) CKL(X.issue(st.next->mats[HX_W_QKV], rows));
      if (st.tick()) return HX_OK;
    }
  }
  return HX_OK;
}

int moss_block(hx_ctx* h, const Weights& W, const int32_t* meta, uint8_t* blob, const float* mod, Stage& st) {
  const int D = W.D, F = W.F, H = W.H;
  const int T = meta[HX_S_NTOK];
  const int nvalid = meta[HX_S_NVALID] > 0 ? meta[HX_S_NVALID] : T * (meta[HX_S_SP] > 1 ? meta[HX_S_SP] : 1);
  const int B = meta[HX_S_BATCH] > 0 ? meta[HX_S_BATCH] : 1;
  const int mode = meta[HX_S_MODE];  // 0 DiT block, 1 text refiner (no LoRA-A GEMMs), 2 text projection
  const int rows = B * T;
  cudaStream_t s = h->stream;
  float* x = reinterpret_cast<float*>(blob + meta[HX_S_X]);
  __half* hbuf = hptr(blob, meta[HX_S_H]);
  __half* qkv = hptr(blob, meta[HX_S_Q]);
  __half* obuf = hptr(blob, meta[HX_S_O]);
  __half* mid = hptr(blob, meta[HX_S_MID]);
  const float* cosT = fptr(blob, meta[HX_S_COS]);
  const float* sinT = fptr(blob, meta[HX_S_SIN]);
  const float* gain = W.gain;
  const float *sh_a = mod, *sc_a = mod + D, *gt_a = mod + 2 * D, *sh_f = mod + 3 * D, *sc_f = mod + 4 * D,
              *gt_f = mod + 5 * D;
  const bool lora = W.lora != 0;
  __half *lq = nullptr, *lo = nullptr, *lu = nullptr, *ld = nullptr;
  if (lora) {
    lq = hptr(blob, meta[HX_S_LQ]);
    lo = hptr(blob, meta[HX_S_LO]);
    lu = hptr(blob, meta[HX_S_LU]);
    ld = hptr(blob, meta[HX_S_LD]);
  }
  if (mode == 2) {  // x += gate_a * (text . Wp + bias)   (moss/hexagon/mega/blk.c:229-233)
    GemmArgs g = gargs(h, hbuf, W.Cd, rows, &W.mats[HX_W_O], EPI_RESID);
    g.K1 = W.Cd;
    g.A2 = lq;
    g.lda2 = 384;
    g.x = x;
    g.ldx = D;
    g.gate = gt_a;
    g.vec_bstride = 0;
    CKL(gemm_launch(g, s));
    st.tick();
    return HX_OK;
  }
  const bool run_a = lora && mode == 0;  // MODE 1: the L buffers hold the host's bias selector
  // ---- attention half
  CKL(rmsmod_launch(x, hbuf, rows, D, gain + 256, sh_a, sc_a, 0, T, 1e-6f, s));
  if (st.tick()) return HX_OK;
  if (run_a) {
    GemmArgs ga = gargs(h, hbuf, D, rows, &W.mats[HX_W_AQKV], EPI_STORE);
    ga.out = lq;
    ga.ldo = 384;
    CKL(gemm_launch(ga, s));
  }
  if (st.tick()) return HX_OK;
  if (lora) {
    const int slots[3] = {HX_W_Q, HX_W_K, HX_W_V};
    for (int j = 0; j < 3; ++j) {
      GemmArgs g = gargs(h, hbuf, D, rows, &W.mats[slots[j]], j < 2 ? EPI_RMS : EPI_STORE);
      g.K1 = D;
      g.A2 = lq + 128 * j;
      g.lda2 = 384;
      g.out = qkv + j * D;
      g.ldo = 3 * D;
      g.gain0 = gain + 128 * j;
      g.seg1 = g.seg2 = D;
      g.rope0 = 1;
      g.cosT = cosT;
      g.sinT = sinT;
      g.rows_per_img = T;
      CKL(gemm_launch(g, s));
    }
  } else {
    GemmArgs g = gargs(h, hbuf, D, rows, &W.mats[HX_W_QKV], EPI_RMS);
    g.out = qkv;
    g.ldo = 3 * D;
    g.gain0 = gain;
    g.gain1 = gain + 128;
    g.seg1 = D;
    g.seg2 = 2 * D;
    g.rope0 = g.rope1 = 1;
    g.cosT = cosT;
    g.sinT = sinT;
    g.rows_per_img = T;
    CKL(gemm_launch(g, s));
  }
  if (st.tick()) return HX_OK;
  const int sp = meta[HX_S_SP];
  if (sp > 1) {  // Ulysses: token shards -> head shards -> full-sequence attention -> back
    h->spev_used = st.ntimes > 19;
    CKL(hx::sp_attention(h->sp, qkv, obuf, D, T, D, H, nvalid, h->status, s, h->spev_used ? h->spev : nullptr));
  } else {
    AttnArgs a;
    a.q = qkv; a.ldq = 3 * D; a.q_col0 = 0;
    a.k = qkv; a.ldk = 3 * D; a.k_col0 = D;
    a.v = qkv; a.ldv = 3 * D; a.v_col0 = 2 * D;
    a.o = obuf; a.ldo = D;
    a.B = B; a.H = H; a.Tq = T; a.Tk = T; a.nvalid = nvalid;
    a.status = h->status;
    CKL(attn_launch(a, s));
  }
  if (st.tick()) return HX_OK;
  {
    if (run_a) {
      GemmArgs ga = gargs(h, obuf, D, rows, &W.mats[HX_W_AO], EPI_STORE);
      ga.out = lo;
      ga.ldo = 128;
      CKL(gemm_launch(ga, s));
    }
    GemmArgs g = gargs(h, obuf, D, rows, &W.mats[HX_W_O], EPI_RESID);
    if (lora) {
      g.K1 = D;
      g.A2 = lo;
      g.lda2 = 128;
    }
    g.x = x;
    g.ldx = D;
    g.gate = gt_a;
    CKL(gemm_launch(g, s));
  }
  if (st.tick()) return HX_OK;
  // ---- FFN half
  CKL(rmsmod_launch(x, hbuf, rows, D, gain + 256 + D, sh_f, sc_f, 0, T, 1e-6f, s));
  if (st.tick()) return HX_OK;
  {
    if (run_a) {
      GemmArgs ga = gargs(h, hbuf, D, rows, &W.mats[HX_W_AUG], EPI_STORE);
      ga.out = lu;
      ga.ldo = 128;
      CKL(gemm_launch(ga, s));
    }
    GemmArgs g = gargs(h, hbuf, D, rows, &W.mats[HX_W_M1], EPI_SITU);
    if (lora) {
      g.K1 = D;
      g.A2 = lu;
      g.lda2 = 128;
    }
    g.out = mid;
    g.ldo = F;
    CKL(gemm_launch(g, s));
  }
  if (st.tick()) return HX_OK;
  {
    if (run_a) {
      GemmArgs ga = gargs(h, mid, F, rows, &W.mats[HX_W_ADN], EPI_STORE);
      ga.out = ld;
      ga.ldo = 128;
      CKL(gemm_launch(ga, s));
    }
    GemmArgs g = gargs(h, mid, F, rows, &W.mats[HX_W_M2], EPI_RESID);
    if (lora) {
      g.K1 = F;
      g.A2 = ld;
      g.lda2 = 128;
    }
    g.x = x;
    g.ldx = D;
    g.gate = gt_f;
    CKL(gemm_launch(g, s));
  }
  st.tick();
  return HX_OK;
}

// bytes the block reads/writes through meta offsets; checks they stay inside the blob
int check_meta(const Weights& W, const int32_t* meta, int nmeta, size_t blob_bytes) {
  auto in = [&](int off, size_t bytes) {
    return off >= 0 && static_cast<size_t>(off) <= blob_bytes && bytes <= blob_bytes - off;
  };
  if (W.model == HX_MODEL_ANIMA) {
    if (nmeta < HX_A_NMETA) return HX_E_ARG;
    const size_t T = meta[HX_A_NTOK], C = meta[HX_A_NCTX];
    const size_t B = (nmeta > HX_A_BATCH && meta[HX_A_BATCH] > 0) ? meta[HX_A_BATCH] : 1;
    if (T == 0 || T % 32 || C == 0 || C % 32) return HX_E_ARG;
    const size_t D = W.D, F = W.F, R = B * T;
    if (!in(meta[HX_A_X], R * D * 4) || !in(meta[HX_A_CTX], B * C * W.Cd * 2) || !in(meta[HX_A_COS], T * 256) ||
        !in(meta[HX_A_SIN], T * 256) || !in(meta[HX_A_H], R * D * 2) || !in(meta[HX_A_Q], R * 3 * D * 2) ||
        !in(meta[HX_A_O], R * D * 2) || !in(meta[HX_A_MID], R * F * 2) || !in(meta[HX_A_CK], B * C * 2 * D * 2))
      return HX_E_RANGE;
    for (int slot : {HX_A_X, HX_A_CTX, HX_A_COS, HX_A_SIN, HX_A_H, HX_A_Q, HX_A_O, HX_A_MID, HX_A_CK})
      if (meta[slot] % 256) return HX_E_RANGE;
  } else {
    if (nmeta < HX_S_NMETA) return HX_E_ARG;
    const size_t T = meta[HX_S_NTOK];
    const size_t B = (nmeta > HX_S_BATCH && meta[HX_S_BATCH] > 0) ? meta[HX_S_BATCH] : 1;
    if (T == 0 || T % 32) return HX_E_ARG;
    const int sp = nmeta > HX_S_SP ? meta[HX_S_SP] : 0;
    if (sp > 1 && B != 1) return HX_E_ARG;
    if (meta[HX_S_NVALID] < 0 || static_cast<size_t>(meta[HX_S_NVALID]) > T * (sp > 1 ? sp : 1)) return HX_E_ARG;
    const size_t D = W.D, F = W.F, R = B * T;
    const int mode = meta[HX_S_MODE];
    if (mode < 0 || mode > 2 || (mode == 2) != (W.proj != 0) || (mode == 1 && !W.lora)) return HX_E_ARG;
    if (W.proj) {  // MODE 2 reads H [R][Cd] and the LQ bias selector, adds into X
      if (!in(meta[HX_S_X], R * D * 4) || !in(meta[HX_S_H], R * W.Cd * 2) || !in(meta[HX_S_LQ], R * 384 * 2))
        return HX_E_RANGE;
      for (int slot : {HX_S_X, HX_S_H, HX_S_LQ})
        if (meta[slot] % 256) return HX_E_RANGE;
      return HX_OK;
    }
    if (!in(meta[HX_S_X], R * D * 4) || !in(meta[HX_S_COS], T * 256) || !in(meta[HX_S_SIN], T * 256) ||
        !in(meta[HX_S_H], R * D * 2) || !in(meta[HX_S_Q], R * 3 * D * 2) || !in(meta[HX_S_O], R * D * 2) ||
        !in(meta[HX_S_MID], R * F * 2))
      return HX_E_RANGE;
    if (W.lora && (!in(meta[HX_S_LQ], R * 384 * 2) || !in(meta[HX_S_LO], R * 256) || !in(meta[HX_S_LU], R * 256) ||
                   !in(meta[HX_S_LD], R * 256)))
      return HX_E_RANGE;
    for (int slot : {HX_S_X, HX_S_COS, HX_S_SIN, HX_S_H, HX_S_Q, HX_S_O, HX_S_MID})
      if (meta[slot] % 256) return HX_E_RANGE;
  }
  return HX_OK;
}

int run_block(hx_ctx* h, const Weights& W, const int32_t* meta, uint8_t* blob, const float* mod_dev, Stage& st) {
  return W.model == HX_MODEL_ANIMA ? anima_block(h, W, meta, blob, mod_dev, st)
                                   : moss_block(h, W, meta, blob, mod_dev, st);
}

// per-block modulation vectors in h->modscratch (allocated by the caller before any capture)
constexpr size_t kModStride(int D) { return 9ull * D + 3 * 256; }

// mods_dev: per-block device mod vectors, block k at mods_dev + k * mod_stride (stride 0: one shared vector,
// as MOSS blocks use); NULL computes them from emb / lora with each block's AdaLN weights.
int chain_body(hx_ctx* h, const std::vector<const Weights*>& ws, const int32_t* m, uint8_t* blob, const float* mods_dev,
               const float* emb_dev, const float* lora_dev, uint32_t skipmask, size_t mod_stride,
               const __half* ckv_cache = nullptr, size_t ckv_stride = 0) {
  const int model = ws[0]->model, D = ws[0]->D;
  const size_t per = model == HX_MODEL_ANIMA ? kModStride(D) : 6ull * D;
  Lookahead xa(h);  // Anima: each block's last GEMM issues the next block's q|k|v expansion
  for (size_t k = 0; k < ws.size(); ++k) {
    if ((skipmask >> k) & 1) continue;
    const float* md;
    if (mods_dev) {
      md = mods_dev + k * mod_stride;
    } else {
      float* out = h->modscratch + per * k;
      if (modulation_launch(ws[k]->modA, ws[k]->modB, emb_dev, lora_dev, out, 3, D, 256, 3 * D, h->stream) !=
          cudaSuccess)
        return HX_E_CUDA;
      md = out;
    }
    Stage st{h, 0, 0, 0};
    if (ckv_cache) st.ckv_pre = ckv_cache + k * ckv_stride;
    if (model == HX_MODEL_ANIMA) {
      st.xa = &xa;
      for (size_t k2 = k + 1; k2 < ws.size(); ++k2)
        if (!((skipmask >> k2) & 1)) {
          st.next = ws[k2];
          break;
        }
    }
    if (int r = run_block(h, *ws[k], m, blob, md, st)) return r;
  }
  return xa.finish() == cudaSuccess ? HX_OK : HX_E_CUDA;
}

int ensure_modscratch(hx_ctx* h, size_t floats) {
  if (h->modscratch_floats >= floats) return HX_OK;
  cudaStreamSynchronize(h->stream);
  cudaFree(h->modscratch);
  h->modscratch = nullptr;
  h->modscratch_floats = 0;
  if (cudaMalloc(&h->modscratch, floats * 4) != cudaSuccess) return HX_E_CUDA;
  h->modscratch_floats = floats;
  h->drop_graphs();
  return HX_OK;
}

// run `body` directly, or captured once per key and replayed
template <class F>
int run_graphed(hx_ctx* h, std::vector<int64_t> key, F&& body, bool use_graph) {
  if (!use_graph) return body();
  key.push_back(reinterpret_cast<int64_t>(h->stream));
  ChainGraph* hit = nullptr;
  for (auto& g : h->graphs)
    if (g.key == key) hit = &g;
  if (!hit) {
    cudaGraph_t graph = nullptr;
    if (cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeRelaxed) != cudaSuccess) return HX_E_CUDA;
    int r = body();
    cudaError_t ce = cudaStreamEndCapture(h->stream, &graph);
    if (r || ce != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      return r ? r : HX_E_CUDA;
    }
    cudaGraphExec_t exec = nullptr;
    cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) return HX_E_CUDA;
    if (h->graphs.size() >= kMaxGraphs) {  // evict the least recently used
      auto lru = std::min_element(h->graphs.begin(), h->graphs.end(),
                                  [](const ChainGraph& a, const ChainGraph& b) { return a.last_use < b.last_use; });
      cudaGraphExecDestroy(lru->exec);
      h->graphs.erase(lru);
    }
    h->graphs.push_back(ChainGraph{key, exec, 0});
    hit = &h->graphs.back();
  }
  hit->last_use = ++h->graph_clock;
  return cudaGraphLaunch(hit->exec, h->stream) == cudaSuccess ? HX_OK : HX_E_CUDA;
}

std::vector<int32_t> full_meta(const int32_t* meta, int nmeta, int model) {
  const int n = model == HX_MODEL_ANIMA ? HX_A_NMETA_EXT : HX_S_NMETA_EXT;
  std::vector<int32_t> m(std::max(n, nmeta), 0);
  std::copy(meta, meta + nmeta, m.begin());
  return m;
}

hx_ctx* H(hx_handle h) { return reinterpret_cast<hx_ctx*>(h); }

}  // namespace

// ====================================================================== C ABI
extern "C" {

const char* hx_version(void) { return "hxdit 0.1 (sm_100a)"; }

int hx_open(int device, hx_handle* out) {
  if (!out) return HX_E_ARG;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return HX_E_ARG;
  DevGuard g(device);
  auto* h = new hx_ctx();
  h->device = device;
  if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&h->status, sizeof(int)) != cudaSuccess || cudaMemset(h->status, 0, sizeof(int)) != cudaSuccess) {
    delete h;
    return HX_E_CUDA;
  }
  for (auto& e : h->ev) cudaEventCreate(&e);
  for (auto& e : h->spev) cudaEventCreate(&e);
  // side stream and events of the look-ahead weight expansion (without them the chain expands in line)
  if (cudaStreamCreateWithFlags(&h->xstream, cudaStreamNonBlocking) != cudaSuccess) {
    h->xstream = nullptr;
    cudaGetLastError();
  }
  cudaEventCreateWithFlags(&h->xev_fork, cudaEventDisableTiming);
  for (int b = 0; b < 2; ++b) {
    cudaEventCreateWithFlags(&h->xev_read[b], cudaEventDisableTiming);
    cudaEventCreateWithFlags(&h->xev_ready[b], cudaEventDisableTiming);
  }
  *out = reinterpret_cast<hx_handle>(h);
  return HX_OK;
}

int hx_close(hx_handle hh) {
  hx_ctx* h = H(hh);
  if (!h) return HX_E_ARG;
  {
    DevGuard g(h->device);
    cudaStreamSynchronize(h->stream);
    h->drop_graphs();  // graphs holding NCCL calls go before the communicator
    hx::sp_comm_destroy(h->sp);
    for (auto& kv : h->bufs) cudaFree(kv.second.ptr);
    for (auto& kv : h->weights)
      for (void* p : kv.second->owned) cudaFree(p);
    cudaFree(h->modscratch);
    cudaFree(h->wexp);
    if (h->xstream) cudaStreamSynchronize(h->xstream);
    for (auto b : h->xbuf) cudaFree(b);
    if (h->xstream) cudaStreamDestroy(h->xstream);
    cudaEventDestroy(h->xev_fork);
    for (int b = 0; b < 2; ++b) {
      cudaEventDestroy(h->xev_read[b]);
      cudaEventDestroy(h->xev_ready[b]);
    }
    for (auto& kv : h->glues)
      for (void* p : kv.second->owned) cudaFree(p);
    for (auto& kv : h->moss_glues)
      for (void* p : kv.second->owned) cudaFree(p);
    for (auto& kv : h->adapters)
      for (void* p : kv.second->owned) cudaFree(p);
    h->ss.release();
    h->ms.release();
    cudaFree(h->status);
    for (auto& e : h->ev) cudaEventDestroy(e);
    for (auto& e : h->spev) cudaEventDestroy(e);
    if (h->own_stream) cudaStreamDestroy(h->stream);
  }
  delete h;
  return HX_OK;
}

int hx_get_stream(hx_handle hh, void** stream) {
  if (!hh || !stream) return HX_E_ARG;
  *stream = H(hh)->stream;
  return HX_OK;
}

int hx_set_stream(hx_handle hh, void* stream) {
  hx_ctx* h = H(hh);
  if (!h) return HX_E_ARG;
  std::lock_guard<std::mutex> lk(h->mu);
  DevGuard g(h->device);
  cudaStreamSynchronize(h->stream);
  if (h->own_stream) cudaStreamDestroy(h->stream);
  h->stream = static_cast<cudaStream_t>(stream);
  h->own_stream = false;
  h->drop_graphs();
  return HX_OK;
}

int hx_sync(hx_handle hh) {
  hx_ctx* h = H(hh);
  if (!h) return HX_E_ARG;
  DevGuard g(h->device);
  CK(cudaStreamSynchronize(h->stream));
  return HX_OK;
}

int hx_status(hx_handle hh, int* status) {
  hx_ctx* h = H(hh);
  if (!h || !status) return HX_E_ARG;
  DevGuard g(h->device);
  CK(cudaStreamSynchronize(h->stream));
  CK(cudaMemcpy(status, h->status, sizeof(int), cudaMemcpyDeviceToHost));
  CK(cudaMemset(h->status, 0, sizeof(int)));
  return HX_OK;
}

int hx_wait_selftest(hx_handle hh, int64_t limit_ns, int arrive, int32_t* rc) {
  hx_ctx* h = H(hh);
  // 1 us .. 2 s (the pipelines' own limit)
  if (!h || !rc || limit_ns < 1000 || limit_ns > 2000000000LL) return HX_E_ARG;
  std::lock_guard<std::mutex> lk(h->mu);
  DevGuard g(h->device);
  *rc = HX_OK;
  CK(cudaStreamSynchronize(h->stream));
  CK(cudaMemsetAsync(h->status, 0, sizeof(int), h->stream));
  CK(hx::wait_selftest_launch(h->status, static_cast<unsigned long long>(limit_ns), arrive ? 1 : 0, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  int stv = 0;
  CK(cudaMemcpy(&stv, h->status, sizeof(int), cudaMemcpyDeviceToHost));
  if (stv) {
    CK(cudaMemset(h->status, 0, sizeof(int)));
    *rc = HX_E_TIMEOUT;
  }
  return HX_OK;
}

int hx_status_ptr(hx_handle hh, int** status_dev) {
  if (!hh || !status_dev) return HX_E_ARG;
  *status_dev = H(hh)->status;
  return HX_OK;
}

// ---------------------------------------------------------------- buffers
int hx_buf_alloc(hx_handle hh, size_t bytes, int* fd) {
  hx_ctx* h = H(hh);
  if (!h || !fd || !bytes) return HX_E_ARG;
  std::lock_guard<std::mutex> lk(h->mu);
  DevGuard g(h->device);
  void* p = nullptr;
  CK(cudaMalloc(&p, bytes));
  CK(cudaMemsetAsync(p, 0, bytes, h->stream));
  *fd = h->next_fd++;
  h->bufs[*fd] = Buf{p, bytes};
  return HX_OK;
}

int hx_buf_free(hx_handle hh, int fd) {
  hx_ctx* h = H(hh);
  if (!h) return HX_E_ARG;
  std::lock_guard<std::mutex> lk(h->mu);
  auto it = h->bufs.find(fd);
  if (it == h->bufs.end()) return HX_E_ARG;
  DevGuard g(h->device);
  cudaStreamSynchronize(h->stream);
  cudaFree(it->second.ptr);
  h->bufs.erase(it);
  h->drop_graphs();
  return HX_OK;
}

int hx_buf_ptr(hx_handle hh, int fd, void** dev) {
  hx_ctx* h = H(hh);
  if (!h || !dev) return HX_E_ARG;
  auto it = h->bufs.find(fd);
  if (it == h->bufs.end()) return HX_E_ARG;
  *dev = it->second.ptr;
  return HX_OK;
}

int hx_buf_write(hx_handle hh, int fd, size_t off, const void* src, size_t bytes) {
  hx_ctx* h = H(hh);
  if (!h || (!src && bytes)) return HX_E_ARG;
  auto it = h->bufs.find(fd);
  if (it == h->bufs.end() || off > it->second.bytes || bytes > it->second.bytes - off) return HX_E_ARG;
  DevGuard g(h->device);
  CK(cudaMemcpyAsync(static_cast<uint8_t*>(it->second.ptr) + off, src, bytes, cudaMemcpyHostToDevice, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  return HX_OK;
}

int hx_buf_read(hx_handle hh, int fd, size_t off, void* dst, size_t bytes) {
  hx_ctx* h = H(hh);
  if (!h || (!dst && bytes)) return HX_E_ARG;
  auto it = h->bufs.find(fd);
  if (it == h->bufs.end() || off > it->second.bytes || bytes > it->second.bytes - off) return HX_E_ARG;
  DevGuard g(h->device);
  CK(cudaMemcpyAsync(dst, static_cast<uint8_t*>(it->second.ptr) + off, bytes, cudaMemcpyDeviceToHost, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  return HX_OK;
}

// ---------------------------------------------------------------- weights
int hx_weights_load(hx_handle hh, int model, const void* pack, size_t bytes, int* wfd) {
  hx_ctx* h = H(hh);
  if (!h || !pack || !wfd) return HX_E_ARG;
  std::lock_guard<std::mutex> lk(h->mu);
  DevGuard g(h->device);
  auto W = std::make_unique<Weights>();
  int rc = model == HX_MODEL_ANIMA ? load_anima(h, static_cast<const uint8_t*>(pack), bytes, *W)
           : model == HX_MODEL_MOSS ? load_moss(h, static_cast<const uint8_t*>(pack), bytes, *W)
           : model == HX_MODEL_MOSS_PROJ ? load_moss_proj(h, static_cast<const uint8_t*>(pack), bytes, *W)
                                         : HX_E_ARG;
  if (rc) {
    for (void* p : W->owned) cudaFree(p);
    return rc;
  }
  reserve_wexp(h, wexp_need(*W));
  reserve_xbuf(h, wexp_need(*W));
  *wfd = h->next_fd++;
  h->weights[*wfd] = std::move(W);
  return HX_OK;
}

int hx_weights_bind(hx_handle hh, const hx_weight_desc* d, int* wfd) {
  hx_ctx* h = H(hh);
  if (!h || !d || !wfd) return HX_E_ARG;
  auto W = std::make_unique<Weights>();
  W->model = d->model;
  W->D = d->D;
  W->F = d->F;
  W->Cd = d->Cd;
  W->H = d->H > 0 ? d->H : d->D / 128;
  W->lora = d->lora;
  W->gain = d->gain;
  W->modA = static_cast<const __half*>(d->modA);
  W->modB = static_cast<const __half*>(d->modB);
  std::vector<int> need;
  if (d->model == HX_MODEL_MOSS_PROJ) {  // text projection: W_O [D][Cd + 128] only
    W->model = HX_MODEL_MOSS;
    W->proj = 1;
    W->lora = 1;
    if (W->D <= 0 || W->D % 128 || W->Cd <= 0 || W->Cd % 64 || W->H * 128 != W->D) return HX_E_ARG;
    if (!valid_mat(d->mats[HX_W_O]) || d->mats[HX_W_O].n != W->D || d->mats[HX_W_O].k != W->Cd + 128) return HX_E_ARG;
    W->mats[HX_W_O] = to_devmat(d->mats[HX_W_O]);
    W->has[HX_W_O] = true;
    std::lock_guard<std::mutex> lk(h->mu);
    DevGuard g(h->device);
    reserve_wexp(h, wexp_need(*W));
    reserve_xbuf(h, wexp_need(*W));
    *wfd = h->next_fd++;
    h->weights[*wfd] = std::move(W);
    return HX_OK;
  }
  if (W->D <= 0 || W->D % 128 || W->F <= 0 || W->F % 256 || W->H * 128 != W->D || !W->gain) return HX_E_ARG;
  if (d->model == HX_MODEL_ANIMA) {
    need = {HX_W_QKV, HX_W_O, HX_W_CQ, HX_W_CKV, HX_W_CO, HX_W_M1, HX_W_M2};
    if (W->Cd <= 0 || W->Cd % 64) return HX_E_ARG;
  } else if (d->model == HX_MODEL_MOSS) {
    need = d->lora ? std::vector<int>{HX_W_Q, HX_W_K, HX_W_V, HX_W_O, HX_W_M1, HX_W_M2, HX_W_AQKV, HX_W_AO, HX_W_AUG,
                                      HX_W_ADN}
                   : std::vector<int>{HX_W_QKV, HX_W_O, HX_W_M1, HX_W_M2};
  } else {
    return HX_E_ARG;
  }
  for (int slot : need) {
    if (!valid_mat(d->mats[slot])) return HX_E_ARG;
    W->mats[slot] = to_devmat(d->mats[slot]);
    W->has[slot] = true;
  }
  std::lock_guard<std::mutex> lk(h->mu);
  DevGuard g(h->device);
  reserve_wexp(h, wexp_need(*W));
  reserve_xbuf(h, wexp_need(*W));
  *wfd = h->next_fd++;
  h->weights[*wfd] = std::move(W);
  return HX_OK;
}

int hx_weights_free(hx_handle hh, int wfd) {
  hx_ctx* h = H(hh);
  if (!h) return HX_E_ARG;
  std::lock_guard<std::mutex> lk(h->mu);
  auto it = h->weights.find(wfd);
  if (it == h->weights.end()) return HX_E_NOWEIGHTS;
  DevGuard g(h->device);
  cudaStreamSynchronize(h->stream);
  for (void* p : it->second->owned) cudaFree(p);
  h->weights.erase(it);
  h->drop_graphs();
  return HX_OK;
}

int hx_lora_fold(hx_handle hh, int wfd, int slot, const float* B, const float* A, int rank, float scale) {
  hx_ctx* h = H(hh);
  if (!h || !B || !A || slot < 0 || slot >= HX_NMATS || rank < 1 || rank > 128) return HX_E_ARG;
  std::lock_guard<std::mutex> lk(h->mu);
  auto it = h->weights.find(wfd);
  if (it == h->weights.end()) return HX_E_NOWEIGHTS;
  const Weights& W = *it->second;
  if (!W.has[slot]) return HX_E_ARG;
  const DevMat& M = W.mats[slot];
  if (M.fmt != HX_FMT_Q8) return HX_E_FORMAT;
  const bool lora_rows = W.model == HX_MODEL_MOSS && W.lora &&
                         (slot == HX_W_Q || slot == HX_W_K || slot == HX_W_V || slot == HX_W_O || slot == HX_W_M1 ||
                          slot == HX_W_M2);
  const int k_base = M.K - (lora_rows ? 128 : 0);
  const int row_mode = (W.model == HX_MODEL_MOSS && slot == HX_W_M1) ? 1 : 0;
  const int floor_mode = W.model == HX_MODEL_ANIMA ? 1 : 0;
  DevGuard g(h->device);
  const cudaError_t e = lora_fold_launch(M, k_base, B, A, rank, scale, row_mode, floor_mode, h->stream);
  return e == cudaSuccess ? HX_OK : e == cudaErrorInvalidValue ? HX_E_ARG : HX_E_CUDA;
}

int hx_lora_fold_slots(hx_handle hh, int wfd, int proj, const float* B, const float* A, int rank, float scale) {
  hx_ctx* h = H(hh);
  if (!h || !B || !A || proj < HX_LORA_Q || proj > HX_LORA_DN || rank < 1 || rank > 128) return HX_E_ARG;
  std::lock_guard<std::mutex> lk(h->mu);
  auto it = h->weights.find(wfd);
  if (it == h->weights.end()) return HX_E_NOWEIGHTS;
  const Weights& W = *it->second;
  if (W.model != HX_MODEL_MOSS || !W.lora) return HX_E_FORMAT;
  static const int kSlot[6] = {HX_W_Q, HX_W_K, HX_W_V, HX_W_O, HX_W_M1, HX_W_M2};
  static const int kA[6] = {HX_W_AQKV, HX_W_AQKV, HX_W_AQKV, HX_W_AO, HX_W_AUG, HX_W_ADN};
  static const int kRow0[6] = {0, 128, 256, 0, 0, 0};
  const int slot = kSlot[proj], aslot = kA[proj];
  if (!W.has[slot] || !W.has[aslot]) return HX_E_ARG;
  const DevMat& M = W.mats[slot];
  const DevMat& Am = W.mats[aslot];
  if (M.fmt != HX_FMT_Q8 || Am.fmt != HX_FMT_Q8) return HX_E_FORMAT;
  DevGuard g(h->device);
  const cudaError_t e = lora_fold_slots(M, M.K - 128, proj == HX_LORA_UG ? 1 : 0, Am, kRow0[proj], B, A, rank, scale,
                                        h->stream);
  return e == cudaSuccess ? HX_OK : e == cudaErrorInvalidValue ? HX_E_ARG : HX_E_CUDA;
}

int hx_pack_apply_overlay(void* pack, size_t pack_bytes, const void* ovl, size_t ovl_bytes) {
  if (!pack || !ovl || ovl_bytes < 4) return HX_E_ARG;
  const uint8_t* o = static_cast<const uint8_t*>(ovl);
  uint32_t n;
  std::memcpy(&n, o, 4);
  // pass 1: every record inside both buffers
  size_t pos = 4;
  for (uint32_t i = 0; i < n; ++i) {
    if (ovl_bytes - pos < 12) return HX_E_FORMAT;
    uint64_t off;
    uint32_t len;
    std::memcpy(&off, o + pos, 8);
    std::memcpy(&len, o + pos + 8, 4);
    pos += 12;
    if (ovl_bytes - pos < len || off > pack_bytes || pack_bytes - off < len) return HX_E_FORMAT;
    pos += len;
  }
  if (pos != ovl_bytes) return HX_E_FORMAT;
  // pass 2: apply in file order
  pos = 4;
  for (uint32_t i = 0; i < n; ++i) {
    uint64_t off;
    uint32_t len;
    std::memcpy(&off, o + pos, 8);
    std::memcpy(&len, o + pos + 8, 4);
    std::memcpy(static_cast<uint8_t*>(pack) + off, o + pos + 12, len);
    pos += 12 + len;
  }
  return HX_OK;
}

// ---------------------------------------------------------------- blob layout
int hx_blob_layout(int model, int ntok, int nctx, int batch, int D, int F, int Cd, int32_t* meta, int nmeta,
                   size_t* total) {
  if (!meta || !total || ntok <= 0 || ntok % 32 || batch <= 0 || D <= 0 || F <= 0) return HX_E_ARG;
  auto up = [](size_t v) { return (v + 4095) & ~size_t(4095); };
  size_t off = 0;
  const size_t R = static_cast<size_t>(batch) * ntok;
  auto place = [&](int slot, size_t bytes) {
    meta[slot] = static_cast<int32_t>(off);
    off += up(bytes);
  };
  if (model == HX_MODEL_ANIMA) {
    if (nmeta < HX_A_NMETA_EXT || nctx <= 0 || nctx % 32 || Cd <= 0) return HX_E_ARG;
    std::fill(meta, meta + nmeta, 0);
    place(HX_A_X, R * D * 4);
    place(HX_A_CTX, static_cast<size_t>(batch) * nctx * Cd * 2);
    place(HX_A_MOD, (9ull * D + 3 * 256) * 4);
    place(HX_A_COS, static_cast<size_t>(ntok) * 64 * 4);
    place(HX_A_SIN, static_cast<size_t>(ntok) * 64 * 4);
    place(HX_A_H, R * D * 2);
    place(HX_A_Q, R * 3 * D * 2);
    meta[HX_A_K] = meta[HX_A_Q];
    meta[HX_A_V] = meta[HX_A_Q];
    place(HX_A_O, R * D * 2);
    meta[HX_A_T] = meta[HX_A_O];
    place(HX_A_MID, R * F * 2);
    place(HX_A_CK, static_cast<size_t>(batch) * nctx * 2 * D * 2);
    meta[HX_A_CV] = meta[HX_A_CK];
    meta[HX_A_NTOK] = ntok;
    meta[HX_A_NCTX] = nctx;
    meta[HX_A_REL] = 1;
    meta[HX_A_FIRST] = 1;
    meta[HX_A_BATCH] = batch;
  } else if (model == HX_MODEL_MOSS) {
    if (nmeta < HX_S_NMETA_EXT) return HX_E_ARG;
    std::fill(meta, meta + nmeta, 0);
    place(HX_S_X, R * D * 4);
    place(HX_S_COS, static_cast<size_t>(ntok) * 64 * 4);
    place(HX_S_SIN, static_cast<size_t>(ntok) * 64 * 4);
    place(HX_S_CS, 6ull * D * 4);  // mod vectors when the call passes none
    place(HX_S_H, R * static_cast<size_t>(Cd > D ? Cd : D) * 2);  // MODE 2 reads text rows of width Cd
    place(HX_S_Q, R * 3 * D * 2);
    meta[HX_S_K] = meta[HX_S_Q];
    meta[HX_S_V] = meta[HX_S_Q];
    place(HX_S_O, R * D * 2);
    meta[HX_S_T] = meta[HX_S_O];
    place(HX_S_MID, R * F * 2);
    place(HX_S_LQ, R * 384 * 2);
    place(HX_S_LO, R * 128 * 2);
    place(HX_S_LU, R * 128 * 2);
    place(HX_S_LD, R * 128 * 2);
    meta[HX_S_NTOK] = ntok;
    meta[HX_S_NVALID] = ntok;
    meta[HX_S_REL] = 1;
    meta[HX_S_FIRST] = 1;
    meta[HX_S_NCB] = D / 32;
    meta[HX_S_BATCH] = batch;
  } else {
    return HX_E_ARG;
  }
  if (off > 0x7FFFFFFFull) return HX_E_RANGE;  // meta slots are int32 byte offsets, as in the reference
  *total = off;
  return HX_OK;
}

// ---------------------------------------------------------------- per-block operator
int hx_mega_block(hx_handle hh, const int32_t* meta, int nmeta, int wfd, int bfd, const uint8_t* mod, int modlen,
                  int32_t* times, int ntimes, int32_t* rc) {
  hx_ctx* h = H(hh);
  if (!h || !rc) return HX_E_ARG;
  const auto t_entry = std::chrono::steady_clock::now();
  *rc = HX_OK;
  if (times)
    for (int i = 0; i < ntimes; ++i) times[i] = 0;
  if (!meta) return (*rc = HX_E_ARG);
  std::lock_guard<std::mutex> lk(h->mu);
  auto wi = h->weights.find(wfd);
  if (wi == h->weights.end()) return (*rc = HX_E_NOWEIGHTS);
  auto bi = h->bufs.find(bfd);
  if (bi == h->bufs.end()) return (*rc = HX_E_NOBLOB);
  const Weights& W = *wi->second;
  std::vector<int32_t> m = full_meta(meta, nmeta, W.model);
  if (int r = check_meta(W, m.data(), static_cast<int>(m.size()), bi->second.bytes)) return (*rc = r);
  DevGuard g(h->device);
  uint8_t* blob = static_cast<uint8_t*>(bi->second.ptr);
  const int D = W.D;
  const bool anima = W.model == HX_MODEL_ANIMA;
  const int nmod = anima ? 9 * D : 6 * D;
  const int modslot = anima ? HX_A_MOD : HX_S_CS;
  if (anima && m[HX_A_STOP] == 99) return HX_OK;  // reference probe: map weights, do nothing
  float* mod_dev = reinterpret_cast<float*>(blob + m[modslot]);
  if (static_cast<size_t>(m[modslot]) + static_cast<size_t>(nmod) * 4 > bi->second.bytes) return (*rc = HX_E_RANGE);
  if (mod) {
    if (modlen < nmod * 4) return (*rc = HX_E_ARG);
    if (cudaMemcpyAsync(mod_dev, mod, static_cast<size_t>(nmod) * 4, cudaMemcpyHostToDevice, h->stream) != cudaSuccess)
      return (*rc = HX_E_CUDA);
  }
  if (!anima && m[HX_S_SP] > 1) {
    if (!h->sp.comm || h->sp.nranks != m[HX_S_SP]) return (*rc = HX_E_ARG);
    if (hx::sp_reserve(h->sp, m[HX_S_NTOK], D)) return (*rc = HX_E_CUDA);
  }
  Stage st{h, times ? ntimes : 0, 0, anima ? m[HX_A_STOP] : m[HX_S_STOP]};
  if (st.ntimes > 0) cudaEventRecord(h->ev[0], h->stream);
  if (times && ntimes > 24)
    times[24] = static_cast<int32_t>(
        std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - t_entry).count());
  int r = run_block(h, W, m.data(), blob, mod_dev, st);
  if (r) return (*rc = r);
  if (st.ntimes > 0) {
    if (cudaStreamSynchronize(h->stream) != cudaSuccess) return (*rc = HX_E_CUDA);
    for (int i = 0; i < st.ti && i < ntimes && i < 24; ++i) {
      float ms = 0.f;
      cudaEventElapsedTime(&ms, h->ev[i], h->ev[i + 1]);
      times[i] = static_cast<int32_t>(ms * 1000.f);
    }
    if (h->spev_used) {  // Ulysses attention stage: pack + q|k|v exchange, attention, o exchange + unpack
      for (int i = 0; i < 3; ++i) {
        float ms = 0.f;
        cudaEventElapsedTime(&ms, h->spev[i], h->spev[i + 1]);
        times[17 + i] = static_cast<int32_t>(ms * 1000.f);
      }
      h->spev_used = false;
    }
    int stv = 0;
    cudaMemcpy(&stv, h->status, sizeof(int), cudaMemcpyDeviceToHost);
    if (stv) {
      cudaMemset(h->status, 0, sizeof(int));
      return (*rc = HX_E_TIMEOUT);
    }
  }
  if (cudaPeekAtLastError() != cudaSuccess) return (*rc = HX_E_CUDA);
  return HX_OK;
}

int hx_sp_unique_id(void* id128) { return hx::sp_unique_id(id128) == 0 ? HX_OK : HX_E_CUDA; }

int hx_sp_init(hx_handle hh, int nranks, int rank, const void* id128) {
  hx_ctx* h = H(hh);
  if (!h || !id128 || nranks < 2 || rank < 0 || rank >= nranks) return HX_E_ARG;
  std::lock_guard<std::mutex> lk(h->mu);
  if (h->sp.comm) return HX_E_ARG;
  DevGuard g(h->device);
  return hx::sp_comm_init(h->sp, nranks, rank, id128) == 0 ? HX_OK : HX_E_CUDA;
}

int hx_modulation(hx_handle hh, int wfd, const float* emb_dev, const float* lora_dev, float* mod_dev) {
  hx_ctx* h = H(hh);
  if (!h || !emb_dev || !mod_dev) return HX_E_ARG;
  auto wi = h->weights.find(wfd);
  if (wi == h->weights.end()) return HX_E_NOWEIGHTS;
  const Weights& W = *wi->second;
  if (W.model != HX_MODEL_ANIMA || !W.modA || !W.modB) return HX_E_ARG;
  DevGuard g(h->device);
  CK(modulation_launch(W.modA, W.modB, emb_dev, lora_dev, mod_dev, 3, W.D, 256, 3 * W.D, h->stream));
  return HX_OK;
}

int hx_chain(hx_handle hh, const int32_t* meta, int nmeta, const int* wfds, int count, int bfd, const float* mods_dev,
             const float* emb_dev, const float* lora_dev, uint32_t skipmask, int use_graph, int32_t* rc) {
  hx_ctx* h = H(hh);
  if (!h || !rc || !meta || !wfds || count <= 0) return HX_E_ARG;
  *rc = HX_OK;
  std::lock_guard<std::mutex> lk(h->mu);
  auto bi = h->bufs.find(bfd);
  if (bi == h->bufs.end()) return (*rc = HX_E_NOBLOB);
  std::vector<const Weights*> ws(count);
  for (int k = 0; k < count; ++k) {
    auto wi = h->weights.find(wfds[k]);
    if (wi == h->weights.end()) return (*rc = HX_E_NOWEIGHTS);
    ws[k] = wi->second.get();
    if (ws[k]->model != ws[0]->model || ws[k]->D != ws[0]->D) return (*rc = HX_E_ARG);
  }
  const int model = ws[0]->model, D = ws[0]->D;
  std::vector<int32_t> m = full_meta(meta, nmeta, model);
  for (int k = 0; k < count; ++k)
    if (int r = check_meta(*ws[k], m.data(), static_cast<int>(m.size()), bi->second.bytes)) return (*rc = r);
  if (!mods_dev) {
    if (model != HX_MODEL_ANIMA || !emb_dev) return (*rc = HX_E_ARG);
    for (int k = 0; k < count; ++k)
      if (!ws[k]->modA || !ws[k]->modB) return (*rc = HX_E_ARG);
  }
  DevGuard g(h->device);
  if (!mods_dev)
    if (int r = ensure_modscratch(h, kModStride(D) * count)) return (*rc = r);
  if (model == HX_MODEL_MOSS && m[HX_S_SP] > 1) {
    if (!h->sp.comm || h->sp.nranks != m[HX_S_SP]) return (*rc = HX_E_ARG);
    if (hx::sp_reserve(h->sp, m[HX_S_NTOK], D)) return (*rc = HX_E_CUDA);
  }
  uint8_t* blob = static_cast<uint8_t*>(bi->second.ptr);
  std::vector<int64_t> key(m.begin(), m.end());
  for (int k = 0; k < count; ++k) key.push_back(wfds[k]);
  for (int64_t v : {int64_t(1), int64_t(bfd), reinterpret_cast<int64_t>(mods_dev), reinterpret_cast<int64_t>(emb_dev),
                    reinterpret_cast<int64_t>(lora_dev), int64_t(skipmask)})
    key.push_back(v);
  const int r = run_graphed(
      h, key,
      [&] {
        return chain_body(h, ws, m.data(), blob, mods_dev, emb_dev, lora_dev, skipmask,
                          ws[0]->model == HX_MODEL_ANIMA ? 9ull * ws[0]->D : 6ull * ws[0]->D);
      },
      use_graph != 0);
  return (*rc = r);
}

// ---------------------------------------------------------------- glue + sampler
int hx_adapter_load(hx_handle hh, const hx_anima_adapter_desc* d, int* afd) {
  hx_ctx* h = H(hh);
  if (!h || !d || !afd || !d->embed || d->vocab <= 0 || !d->out_w || !d->out_b || !d->norm) return HX_E_ARG;
  for (const hx_adapter_block_desc& b : d->blocks) {
    const void* p[] = {b.norm_sa, b.sa_q, b.sa_k, b.sa_v, b.sa_o, b.sa_qn, b.sa_kn, b.norm_ca, b.ca_q, b.ca_k,
                       b.ca_v, b.ca_o, b.ca_qn, b.ca_kn, b.norm_mlp, b.mlp0_w, b.mlp0_b, b.mlp2_w, b.mlp2_b};
    for (const void* q : p)
      if (!q) return HX_E_ARG;
  }
  std::lock_guard<std::mutex> lk(h->mu);
  DevGuard g(h->device);
  auto A = std::make_unique<Adapter>();
  bool ok = true;
  auto copy = [&](const void* src, size_t elems) -> const __half* {
    void* p = nullptr;
    if (!ok || cudaMalloc(&p, elems * 2) != cudaSuccess) {
      ok = false;
      return nullptr;
    }
    A->owned.push_back(p);
    if (cudaMemcpyAsync(p, src, elems * 2, cudaMemcpyDeviceToDevice, h->stream) != cudaSuccess) ok = false;
    return static_cast<const __half*>(p);
  };
  const size_t D = 1024, F = 4096;
  A->w.vocab = d->vocab;
  A->w.embed = copy(d->embed, static_cast<size_t>(d->vocab) * D);
  for (int i = 0; i < 6; ++i) {
    const hx_adapter_block_desc& b = d->blocks[i];
    AdapterWeights::Block& o = A->w.blocks[i];
    o.norm_sa = copy(b.norm_sa, D);
    o.sa_q = copy(b.sa_q, D * D);
    o.sa_k = copy(b.sa_k, D * D);
    o.sa_v = copy(b.sa_v, D * D);
    o.sa_o = copy(b.sa_o, D * D);
    o.sa_qn = copy(b.sa_qn, 64);
    o.sa_kn = copy(b.sa_kn, 64);
    o.norm_ca = copy(b.norm_ca, D);
    o.ca_q = copy(b.ca_q, D * D);
    o.ca_k = copy(b.ca_k, D * D);
    o.ca_v = copy(b.ca_v, D * D);
    o.ca_o = copy(b.ca_o, D * D);
    o.ca_qn = copy(b.ca_qn, 64);
    o.ca_kn = copy(b.ca_kn, 64);
    o.norm_mlp = copy(b.norm_mlp, D);
    o.mlp0_w = copy(b.mlp0_w, F * D);
    o.mlp0_b = copy(b.mlp0_b, F);
    o.mlp2_w = copy(b.mlp2_w, D * F);
    o.mlp2_b = copy(b.mlp2_b, D);
  }
  A->w.out_w = copy(d->out_w, D * D);
  A->w.out_b = copy(d->out_b, D);
  A->w.norm = copy(d->norm, D);
  if (!ok || cudaStreamSynchronize(h->stream) != cudaSuccess) {
    for (void* p : A->owned) cudaFree(p);
    return HX_E_CUDA;
  }
  *afd = h->next_fd++;
  h->adapters[*afd] = std::move(A);
  return HX_OK;
}

int hx_anima_adapter(hx_handle hh, int afd, const float* hidden, int S, const int32_t* ids, const float* wts, int L,
                     float* out) {
  hx_ctx* h = H(hh);
  if (!h || !hidden || !ids || !wts || !out) return HX_E_ARG;
  std::lock_guard<std::mutex> lk(h->mu);
  auto it = h->adapters.find(afd);
  if (it == h->adapters.end()) return HX_E_ARG;
  DevGuard g(h->device);
  const cudaError_t e = adapter_run(it->second->w, hidden, S, ids, wts, L, out, h->status, h->stream);
  return e == cudaSuccess ? HX_OK : e == cudaErrorInvalidValue ? HX_E_ARG : HX_E_CUDA;
}

int hx_glue_load(hx_handle hh, const hx_anima_glue_desc* d, int* gfd) {
  hx_ctx* h = H(hh);
  if (!h || !d || !gfd || d->D <= 0 || d->D % 256) return HX_E_ARG;
  if (!d->t_norm || !d->t_lin1 || !d->t_lin2 || !d->x_emb || !d->f_modA || !d->f_modB || !d->f_lin) return HX_E_ARG;
  std::lock_guard<std::mutex> lk(h->mu);
  DevGuard g(h->device);
  auto G = std::make_unique<Glue>();
  const size_t D = d->D;
  auto copy = [&](const void* src, size_t elems, __half** dst) -> int {
    void* p = nullptr;
    CK(cudaMalloc(&p, elems * 2));
    G->owned.push_back(p);
    CK(cudaMemcpyAsync(p, src, elems * 2, cudaMemcpyDeviceToDevice, h->stream));
    *dst = static_cast<__half*>(p);
    return HX_OK;
  };
  int r;
  if ((r = copy(d->t_norm, D, &G->t_norm)) || (r = copy(d->t_lin1, D * D, &G->t_lin1)) ||
      (r = copy(d->t_lin2, 3 * D * D, &G->t_lin2)) || (r = copy(d->f_modA, 256 * D, &G->f_modA)) ||
      (r = copy(d->f_modB, 2 * D * 256, &G->f_modB)) || (r = copy(d->f_lin, 64 * D, &G->f_lin))) {
    for (void* p : G->owned) cudaFree(p);
    return r;
  }
  void* xe = nullptr;
  if (cudaMalloc(&xe, D * 128 * 2) != cudaSuccess) {
    for (void* p : G->owned) cudaFree(p);
    return HX_E_CUDA;
  }
  G->owned.push_back(xe);
  G->x_emb = static_cast<__half*>(xe);
  if (pad_cols_launch(static_cast<const __half*>(d->x_emb), G->x_emb, static_cast<int>(D), 68, 128, h->stream) !=
          cudaSuccess ||
      cudaStreamSynchronize(h->stream) != cudaSuccess) {
    for (void* p : G->owned) cudaFree(p);
    return HX_E_CUDA;
  }
  G->D = d->D;
  *gfd = h->next_fd++;
  h->glues[*gfd] = std::move(G);
  return HX_OK;
}

int hx_anima_sample(hx_handle hh, int gfd, const int32_t* meta, int nmeta, const int* wfds, int nblk, int bfd,
                    float* latent, int lat_h, int lat_w, int nsteps, const float* sigmas, int use_graph,
                    int32_t* rc) {
  hx_ctx* h = H(hh);
  if (!h || !rc || !meta || !wfds || nblk <= 0 || !latent) return HX_E_ARG;
  *rc = HX_OK;
  if (nsteps <= 0 || nsteps > 8 || lat_h % 2 || lat_w % 2) return (*rc = HX_E_ARG);
  std::lock_guard<std::mutex> lk(h->mu);
  auto gi = h->glues.find(gfd);
  if (gi == h->glues.end()) return (*rc = HX_E_ARG);
  const Glue& G = *gi->second;
  auto bi = h->bufs.find(bfd);
  if (bi == h->bufs.end()) return (*rc = HX_E_NOBLOB);
  std::vector<const Weights*> ws(nblk);
  for (int k = 0; k < nblk; ++k) {
    auto wi = h->weights.find(wfds[k]);
    if (wi == h->weights.end()) return (*rc = HX_E_NOWEIGHTS);
    ws[k] = wi->second.get();
    if (ws[k]->model != HX_MODEL_ANIMA || ws[k]->D != G.D || !ws[k]->modA || !ws[k]->modB) return (*rc = HX_E_ARG);
  }
  std::vector<int32_t> m = full_meta(meta, nmeta, HX_MODEL_ANIMA);
  for (int k = 0; k < nblk; ++k)
    if (int r = check_meta(*ws[k], m.data(), static_cast<int>(m.size()), bi->second.bytes)) return (*rc = r);
  const int D = G.D, T = m[HX_A_NTOK], B = m[HX_A_BATCH] > 0 ? m[HX_A_BATCH] : 1;
  if ((lat_h / 2) * (lat_w / 2) != T) return (*rc = HX_E_ARG);
  Sigmas sg{};
  float sig[9];
  for (int i = 0; i <= nsteps; ++i) {
    if (sigmas) {
      sig[i] = sigmas[i];
    } else if (i == nsteps) {
      sig[i] = 0.f;
    } else {  // animad.cpp:397-399
      const double sv = nsteps > 1 ? 1.0 - (1.0 - 0.001) * i / (nsteps - 1) : 1.0;
      sig[i] = static_cast<float>(3 * sv / (1 + 2 * sv));
    }
  }
  for (int i = 0; i < nsteps; ++i) sg.s[i] = sig[i];
  DevGuard g(h->device);
  const size_t rows = static_cast<size_t>(B) * T;
  const int C = m[HX_A_NCTX];
  const size_t ckv_stride = static_cast<size_t>(B) * C * 2 * D, ckv_need = ckv_stride * nblk;
  SampleScratch& sc = h->ss;
  if (sc.S < nsteps || sc.D != D || sc.rows < rows || sc.ckv_elems < ckv_need ||
      sc.modtab_host.size() < 2 * static_cast<size_t>(nblk)) {
    cudaStreamSynchronize(h->stream);
    h->drop_graphs();
    sc.release();
    const size_t S = 8;
    bool ok = cudaMalloc(&sc.tp, S * D * 4) == cudaSuccess && cudaMalloc(&sc.emb, S * D * 4) == cudaSuccess &&
              cudaMalloc(&sc.tmp, S * D * 4) == cudaSuccess && cudaMalloc(&sc.lora, S * 3 * D * 4) == cudaSuccess &&
              cudaMalloc(&sc.h256, S * 256 * 4) == cudaSuccess && cudaMalloc(&sc.fmod, S * 2 * D * 4) == cudaSuccess &&
              cudaMalloc(&sc.y, rows * 64 * 4) == cudaSuccess && cudaMalloc(&sc.P, rows * 128 * 2) == cudaSuccess &&
              cudaMalloc(&sc.ckv, ckv_need * 2) == cudaSuccess &&
              cudaMalloc(&sc.modtab, 2 * static_cast<size_t>(nblk) * sizeof(void*)) == cudaSuccess &&
              cudaMalloc(&sc.se, static_cast<size_t>(D) * 4) == cudaSuccess;
    if (!ok) {
      sc.release();
      return (*rc = HX_E_CUDA);
    }
    sc.S = static_cast<int>(S);
    sc.D = D;
    sc.rows = rows;
    sc.ckv_elems = ckv_need;
    sc.modtab_host.assign(2 * static_cast<size_t>(nblk), nullptr);
  }
  {  // the blocks' AdaLN weights for the batched modulation (uploaded when they change)
    std::vector<const __half*> tab(sc.modtab_host.size(), nullptr);
    for (int k = 0; k < nblk; ++k) {
      tab[k] = ws[k]->modA;
      tab[nblk + k] = ws[k]->modB;
    }
    if (tab != sc.modtab_host) {
      if (cudaMemcpyAsync(sc.modtab, tab.data(), tab.size() * sizeof(void*), cudaMemcpyHostToDevice, h->stream) !=
          cudaSuccess)
        return (*rc = HX_E_CUDA);
      sc.modtab_host = tab;
    }
  }
  if (int r = ensure_modscratch(h, kModStride(D) * nblk)) return (*rc = r);
  uint8_t* blob = static_cast<uint8_t*>(bi->second.ptr);
  float* x = reinterpret_cast<float*>(blob + m[HX_A_X]);
  const __half* ctxp = hptr(blob, m[HX_A_CTX]);
  __half* hbuf = hptr(blob, m[HX_A_H]);
  cudaStream_t s = h->stream;
  auto body = [&]() -> int {
    const int S = nsteps;
    CKL(temb_launch(sg, S, D, G.t_norm, sc.tp, sc.emb, s));
    CKL(gemv_rows_launch(G.t_lin1, sc.tp, sc.tmp, S, D, D, 0, nullptr, 0, D, s));
    CKL(gemv_rows_launch(G.t_lin2, sc.tmp, sc.lora, S, D, 3 * D, 1, nullptr, 0, 3 * D, s));
    CKL(gemv_rows_launch(G.f_modA, sc.emb, sc.h256, S, D, 256, 1, nullptr, 0, 256, s));
    CKL(gemv_rows_launch(G.f_modB, sc.h256, sc.fmod, S, 256, 2 * D, 0, sc.lora, 3 * D, 2 * D, s));
    // the cross-attention k|v of each block depend only on the context: once per sample, not per step
    for (int k = 0; k < nblk; ++k) CKL(ckv_launch(h, *ws[k], ctxp, B * C, sc.ckv + k * ckv_stride));
    DevMat xe, fl;
    xe.fmt = WF_F16; xe.N = D; xe.K = 128; xe.w = G.x_emb;
    fl.fmt = WF_F16; fl.N = 64; fl.K = D; fl.w = G.f_lin;
    for (int i = 0; i < S; ++i) {
      CKL(patchify_launch(latent, sc.P, B, 16, lat_h, lat_w, 128, s));
      GemmArgs ge = gargs(h, sc.P, 128, static_cast<int>(rows), &xe, EPI_STORE32);
      ge.x = x;
      ge.ldx = D;
      CKL(gemm_launch(ge, s));
      // the 36 blocks' modulation vectors of this step in one pair of launches
      const size_t per = kModStride(D);
      CKL(modulation_batch_launch(sc.modtab, sc.modtab + nblk, nblk, sc.emb + static_cast<size_t>(i) * D,
                                  sc.lora + static_cast<size_t>(i) * 3 * D, h->modscratch, per, sc.se, 3, D, 256,
                                  3 * D, s));
      if (int r = chain_body(h, ws, m.data(), blob, h->modscratch, nullptr, nullptr, 0, per, sc.ckv, ckv_stride))
        return r;
      const float* fm = sc.fmod + static_cast<size_t>(i) * 2 * D;
      CKL(lnmod_launch(x, hbuf, static_cast<int>(rows), D, fm, fm + D, 0, T, 1e-6f, s));
      GemmArgs gf = gargs(h, hbuf, D, static_cast<int>(rows), &fl, EPI_STORE32);
      gf.x = sc.y;
      gf.ldx = 64;
      CKL(gemm_launch(gf, s));
      CKL(unpatch_euler_launch(sc.y, latent, B, 16, lat_h, lat_w, 64, sig[i + 1] - sig[i], s));
    }
    return HX_OK;
  };
  std::vector<int64_t> key(m.begin(), m.end());
  for (int k = 0; k < nblk; ++k) key.push_back(wfds[k]);
  for (int64_t v : {int64_t(2), int64_t(gfd), int64_t(bfd), reinterpret_cast<int64_t>(latent), int64_t(lat_h),
                    int64_t(lat_w), int64_t(nsteps)})
    key.push_back(v);
  for (int i = 0; i <= nsteps; ++i) {
    int32_t bits;
    std::memcpy(&bits, &sig[i], 4);
    key.push_back(bits);
  }
  return (*rc = run_graphed(h, key, body, use_graph != 0));
}

// ---------------------------------------------------------------- MOSS sampler
int hx_moss_glue_load(hx_handle hh, const hx_moss_glue_desc* d, int* gfd) {
  hx_ctx* h = H(hh);
  if (!h || !d || !gfd || d->D <= 0 || d->D % 256) return HX_E_ARG;
  if (!d->t_lin0 || !d->t_b0 || !d->t_lin2 || !d->t_b2 || !d->mod_w || !d->mod_b || !d->head_w || !d->head_b ||
      !d->emb_w || !d->emb_b || !d->fin_norm || !d->fin_w || !d->mix_q)
    return HX_E_ARG;
  std::lock_guard<std::mutex> lk(h->mu);
  DevGuard g(h->device);
  auto G = std::make_unique<MossGlue>();
  const size_t D = d->D;
  auto fail = [&](int r) {
    cudaStreamSynchronize(h->stream);
    for (void* p : G->owned) cudaFree(p);
    return r;
  };
  auto copy = [&](const void* src, size_t bytes, void** dst) -> bool {
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return false;
    G->owned.push_back(p);
    *dst = p;
    return cudaMemcpyAsync(p, src, bytes, cudaMemcpyDeviceToDevice, h->stream) == cudaSuccess;
  };
  void* ptr[12] = {};
  const bool ok = copy(d->t_lin0, D * 256 * 2, &ptr[0]) && copy(d->t_lin2, D * D * 2, &ptr[1]) &&
                  copy(d->mod_w, 6 * D * D * 2, &ptr[2]) && copy(d->head_w, 2 * D * D * 2, &ptr[3]) &&
                  copy(d->fin_w, 128 * D * 2, &ptr[4]) && copy(d->t_b0, D * 4, &ptr[5]) && copy(d->t_b2, D * 4, &ptr[6]) &&
                  copy(d->mod_b, 6 * D * 4, &ptr[7]) && copy(d->head_b, 2 * D * 4, &ptr[8]) &&
                  copy(d->fin_norm, D * 4, &ptr[9]) && copy(d->mix_q, 128 * 128 * 4, &ptr[10]);
  if (!ok) return fail(HX_E_CUDA);
  G->t_lin0 = static_cast<__half*>(ptr[0]);
  G->t_lin2 = static_cast<__half*>(ptr[1]);
  G->mod_w = static_cast<__half*>(ptr[2]);
  G->head_w = static_cast<__half*>(ptr[3]);
  G->fin_w = static_cast<__half*>(ptr[4]);
  G->t_b0 = static_cast<float*>(ptr[5]);
  G->t_b2 = static_cast<float*>(ptr[6]);
  G->mod_b = static_cast<float*>(ptr[7]);
  G->head_b = static_cast<float*>(ptr[8]);
  G->fin_norm = static_cast<float*>(ptr[9]);
  G->Q = static_cast<float*>(ptr[10]);
  if (cudaMalloc(&ptr[11], D * kMossEmbK * 2) != cudaSuccess) return fail(HX_E_CUDA);
  G->owned.push_back(ptr[11]);
  G->emb = static_cast<__half*>(ptr[11]);
  if (moss_emb_pad_launch(static_cast<const __half*>(d->emb_w), d->emb_b, G->emb, static_cast<int>(D), kMossEmbK,
                          h->stream) != cudaSuccess ||
      cudaStreamSynchronize(h->stream) != cudaSuccess)
    return fail(HX_E_CUDA);
  G->D = d->D;
  *gfd = h->next_fd++;
  h->moss_glues[*gfd] = std::move(G);
  return HX_OK;
}

namespace {
struct Mgl1Entry {
  char name[41];
  int32_t dtype, nd, dims[3];
  int64_t off, bytes;
};
// parse and validate every entry of an MGL1 file (export_glue.py layout, little endian, 76-byte entries)
int mgl1_entries(const uint8_t* b, size_t size, std::vector<Mgl1Entry>& out) {
  constexpr size_t kEnt = 40 + 4 + 4 + 12 + 8 + 8;
  if (!b || size < 8 || std::memcmp(b, "MGL1", 4) != 0) return HX_E_FORMAT;
  int32_t n;
  std::memcpy(&n, b + 4, 4);
  if (n < 0 || static_cast<size_t>(n) > (size - 8) / kEnt) return HX_E_FORMAT;
  out.resize(n);
  for (int i = 0; i < n; ++i) {
    const uint8_t* e = b + 8 + static_cast<size_t>(i) * kEnt;
    Mgl1Entry& m = out[i];
    std::memcpy(m.name, e, 40);
    m.name[40] = 0;
    std::memcpy(&m.dtype, e + 40, 4);
    std::memcpy(&m.nd, e + 44, 4);
    std::memcpy(m.dims, e + 48, 12);
    std::memcpy(&m.off, e + 60, 8);
    std::memcpy(&m.bytes, e + 68, 8);
    if ((m.dtype != 0 && m.dtype != 1) || m.nd < 0 || m.nd > 3 || m.off < 0 || m.bytes < 0) return HX_E_FORMAT;
    if (static_cast<uint64_t>(m.off) > size || static_cast<uint64_t>(m.bytes) > size - m.off) return HX_E_FORMAT;
    int64_t elems = 1;
    for (int d = 0; d < 3; ++d) {
      if (m.dims[d] < 0) return HX_E_FORMAT;
      elems *= m.dims[d];
    }
    if (elems * (m.dtype ? 2 : 4) != m.bytes) return HX_E_FORMAT;
  }
  return HX_OK;
}
}  // namespace

int hx_mgl1_tensor(const void* file, size_t bytes, const char* name, int* dtype, int* nd, int32_t dims[3],
                   const void** data, size_t* nbytes) {
  if (!name) return HX_E_ARG;
  std::vector<Mgl1Entry> es;
  if (int r = mgl1_entries(static_cast<const uint8_t*>(file), bytes, es)) return r;
  for (const Mgl1Entry& e : es) {
    if (std::strncmp(e.name, name, 40) != 0) continue;
    if (dtype) *dtype = e.dtype;
    if (nd) *nd = e.nd;
    if (dims) std::memcpy(dims, e.dims, 12);
    if (data) *data = static_cast<const uint8_t*>(file) + e.off;
    if (nbytes) *nbytes = static_cast<size_t>(e.bytes);
    return HX_OK;
  }
  return HX_E_RANGE;
}

int hx_moss_glue_load_mgl1(hx_handle hh, const void* file, size_t bytes, int* gfd) {
  hx_ctx* h = H(hh);
  if (!h || !file || !gfd) return HX_E_ARG;
  std::vector<Mgl1Entry> es;
  if (int r = mgl1_entries(static_cast<const uint8_t*>(file), bytes, es)) return r;
  const uint8_t* base = static_cast<const uint8_t*>(file);
  auto find = [&](const char* n) -> const Mgl1Entry* {
    for (const Mgl1Entry& e : es)
      if (std::strncmp(e.name, n, 40) == 0) return &e;
    return nullptr;
  };
  const Mgl1Entry* emb = find("video_embedder.weight");
  if (!emb || emb->nd != 2) return HX_E_FORMAT;
  const int64_t D = emb->dims[0];
  // name, rows, cols (cols 1 for vectors), device dtype (1 fp16, 0 fp32)
  struct Need { const char* name; int64_t r, c; int f16; };
  const Need need[13] = {{"time_embedding.0.weight", D, 256, 1}, {"time_embedding.0.bias", D, 1, 0},
                         {"time_embedding.2.weight", D, D, 1},  {"time_embedding.2.bias", D, 1, 0},
                         {"shared_block_modulation.weight", 6 * D, D, 1}, {"shared_block_modulation.bias", 6 * D, 1, 0},
                         {"video_head_modulation.weight", 2 * D, D, 1}, {"video_head_modulation.bias", 2 * D, 1, 0},
                         {"video_embedder.weight", D, 128, 1},  {"video_embedder.bias", D, 1, 0},
                         {"final_norm_video.weight", D, 1, 0},  {"final_linear_video.weight", 128, D, 1},
                         {"latent_mix.Q", 128, 128, 0}};
  std::vector<void*> tmp;
  auto cleanup = [&](int r) {
    for (void* p : tmp) cudaFree(p);
    return r;
  };
  void* dptr[13] = {};
  for (int i = 0; i < 13; ++i) {
    const Mgl1Entry* e = find(need[i].name);
    if (!e) return cleanup(HX_E_FORMAT);
    const int64_t n = need[i].r * need[i].c;
    if (static_cast<int64_t>(e->dims[0]) * std::max(1, e->dims[1]) * std::max(1, e->dims[2]) != n) return cleanup(HX_E_FORMAT);
    std::vector<uint16_t> h16;
    std::vector<float> f32;
    const void* src = base + e->off;
    size_t nb;
    if (need[i].f16) {
      if (e->dtype == 1) {
        nb = n * 2;
      } else {
        h16.resize(n);
        for (int64_t k = 0; k < n; ++k) {
          float v;
          std::memcpy(&v, base + e->off + 4 * k, 4);
          h16[k] = __half_as_ushort(__float2half_rn(v));
        }
        src = h16.data();
        nb = n * 2;
      }
    } else {
      if (e->dtype == 0) {
        nb = n * 4;
      } else {
        f32.resize(n);
        for (int64_t k = 0; k < n; ++k) {
          uint16_t u;
          std::memcpy(&u, base + e->off + 2 * k, 2);
          f32[k] = __half2float(__ushort_as_half(u));
        }
        src = f32.data();
        nb = n * 4;
      }
    }
    DevGuard g(h->device);
    if (cudaMalloc(&dptr[i], nb) != cudaSuccess) return cleanup(HX_E_CUDA);
    tmp.push_back(dptr[i]);
    if (cudaMemcpy(dptr[i], src, nb, cudaMemcpyHostToDevice) != cudaSuccess) return cleanup(HX_E_CUDA);
  }
  hx_moss_glue_desc d;
  d.D = static_cast<int>(D);
  d.t_lin0 = dptr[0];
  d.t_b0 = static_cast<const float*>(dptr[1]);
  d.t_lin2 = dptr[2];
  d.t_b2 = static_cast<const float*>(dptr[3]);
  d.mod_w = dptr[4];
  d.mod_b = static_cast<const float*>(dptr[5]);
  d.head_w = dptr[6];
  d.head_b = static_cast<const float*>(dptr[7]);
  d.emb_w = dptr[8];
  d.emb_b = static_cast<const float*>(dptr[9]);
  d.fin_norm = static_cast<const float*>(dptr[10]);
  d.fin_w = dptr[11];
  d.mix_q = static_cast<const float*>(dptr[12]);
  const int r = hx_moss_glue_load(hh, &d, gfd);
  return cleanup(r);
}

int hx_moss_sample(hx_handle hh, int gfd, const int32_t* meta, int nmeta, const int* wfds, int nblk, int bfd,
                   const float* z, float* x0, int lat_h, int lat_w, const float* text, int ntext, int nsteps,
                   const float* codes, int use_graph, int32_t* rc) {
  hx_ctx* h = H(hh);
  if (!h || !rc || !meta || !wfds || nblk <= 0 || !z || !x0 || !codes) return HX_E_ARG;
  *rc = HX_OK;
  if (nsteps <= 0 || nsteps > 8 || lat_h <= 0 || lat_w <= 0 || ntext < 0 || (ntext > 0 && !text))
    return (*rc = HX_E_ARG);
  std::lock_guard<std::mutex> lk(h->mu);
  auto gi = h->moss_glues.find(gfd);
  if (gi == h->moss_glues.end()) return (*rc = HX_E_ARG);
  const MossGlue& G = *gi->second;
  auto bi = h->bufs.find(bfd);
  if (bi == h->bufs.end()) return (*rc = HX_E_NOBLOB);
  std::vector<const Weights*> ws(nblk);
  for (int k = 0; k < nblk; ++k) {
    auto wi = h->weights.find(wfds[k]);
    if (wi == h->weights.end()) return (*rc = HX_E_NOWEIGHTS);
    ws[k] = wi->second.get();
    if (ws[k]->model != HX_MODEL_MOSS || ws[k]->proj || ws[k]->D != G.D) return (*rc = HX_E_ARG);
  }
  std::vector<int32_t> m = full_meta(meta, nmeta, HX_MODEL_MOSS);
  const int D = G.D, ntok = m[HX_S_NTOK], B = m[HX_S_BATCH] > 0 ? m[HX_S_BATCH] : 1, Ni = lat_h * lat_w;
  if (Ni + ntext > ntok || m[HX_S_SP] > 1) return (*rc = HX_E_ARG);
  m[HX_S_NVALID] = Ni + ntext;
  m[HX_S_MODE] = 0;
  for (int k = 0; k < nblk; ++k)
    if (int r = check_meta(*ws[k], m.data(), static_cast<int>(m.size()), bi->second.bytes)) return (*rc = r);
  Sigmas cd{};
  for (int i = 0; i < nsteps; ++i) cd.s[i] = codes[i];
  DevGuard g(h->device);
  const size_t rows = static_cast<size_t>(B) * ntok;
  MossScratch& sc = h->ms;
  if (sc.D != D || sc.rows < rows) {
    cudaStreamSynchronize(h->stream);
    h->drop_graphs();
    sc.release();
    const size_t S = 8;
    bool ok = cudaMalloc(&sc.e, S * 256 * 4) == cudaSuccess && cudaMalloc(&sc.a, S * D * 4) == cudaSuccess &&
              cudaMalloc(&sc.tm, S * D * 4) == cudaSuccess && cudaMalloc(&sc.mod, S * 6 * D * 4) == cudaSuccess &&
              cudaMalloc(&sc.head, S * 2 * D * 4) == cudaSuccess && cudaMalloc(&sc.v, rows * 128 * 4) == cudaSuccess &&
              cudaMalloc(&sc.xin, rows * kMossEmbK * 2) == cudaSuccess;
    if (!ok) {
      sc.release();
      return (*rc = HX_E_CUDA);
    }
    sc.D = D;
    sc.rows = rows;
  }
  uint8_t* blob = static_cast<uint8_t*>(bi->second.ptr);
  float* x = reinterpret_cast<float*>(blob + m[HX_S_X]);
  __half* hbuf = hptr(blob, m[HX_S_H]);
  cudaStream_t s = h->stream;
  auto body = [&]() -> int {
    const int S = nsteps;
    // time vectors of every step (moss_ref.py:96-105)
    CKL(moss_temb_launch(cd, S, sc.e, s));
    CKL(gemv_rows_launch(G.t_lin0, sc.e, sc.a, S, 256, D, 0, G.t_b0, 0, D, s));
    CKL(gemv_rows_launch(G.t_lin2, sc.a, sc.tm, S, D, D, 1, G.t_b2, 0, D, s));
    CKL(gemv_rows_launch(G.mod_w, sc.tm, sc.mod, S, D, 6 * D, 0, G.mod_b, 0, 6 * D, s));
    CKL(gemv_rows_launch(G.head_w, sc.tm, sc.head, S, D, 2 * D, 0, G.head_b, 0, 2 * D, s));
    DevMat we, wf;
    we.fmt = WF_F16; we.N = D; we.K = kMossEmbK; we.w = G.emb;
    wf.fmt = WF_F16; wf.N = 128; wf.K = D; wf.w = G.fin_w;
    for (int i = 0; i < S; ++i) {
      // rows = [video_embedder(z + Q x0) ; text ; 0]
      CKL(moss_mix_launch(z, x0, G.Q, sc.xin, B, Ni, ntok, kMossEmbK, s));
      GemmArgs ge = gargs(h, sc.xin, kMossEmbK, static_cast<int>(rows), &we, EPI_STORE32);
      ge.x = x;
      ge.ldx = D;
      CKL(gemm_launch(ge, s));
      for (int b = 0; b < B && ntext > 0; ++b)
        CKL(cudaMemcpyAsync(x + (static_cast<size_t>(b) * ntok + Ni) * D, text, static_cast<size_t>(ntext) * D * 4,
                            cudaMemcpyDeviceToDevice, s));
      if (int r = chain_body(h, ws, m.data(), blob, sc.mod + static_cast<size_t>(i) * 6 * D, nullptr, nullptr, 0, 0))
        return r;
      // v = final_linear(rms(x) * norm * (1 + head1) + head0), x0 = z - v
      const float* hd = sc.head + static_cast<size_t>(i) * 2 * D;
      CKL(rmsmod_launch(x, hbuf, static_cast<int>(rows), D, G.fin_norm, hd, hd + D, 0, ntok, 1e-6f, s));
      GemmArgs gf = gargs(h, hbuf, D, static_cast<int>(rows), &wf, EPI_STORE32);
      gf.x = sc.v;
      gf.ldx = 128;
      CKL(gemm_launch(gf, s));
      CKL(moss_x0_launch(z, sc.v, x0, B, Ni, ntok, 128, s));
    }
    return HX_OK;
  };
  std::vector<int64_t> key(m.begin(), m.end());
  for (int k = 0; k < nblk; ++k) key.push_back(wfds[k]);
  for (int64_t v : {int64_t(3), int64_t(gfd), int64_t(bfd), reinterpret_cast<int64_t>(z), reinterpret_cast<int64_t>(x0),
                    reinterpret_cast<int64_t>(text), int64_t(lat_h), int64_t(lat_w), int64_t(ntext), int64_t(nsteps)})
    key.push_back(v);
  for (int i = 0; i < nsteps; ++i) {
    int32_t bits;
    std::memcpy(&bits, &codes[i], 4);
    key.push_back(bits);
  }
  return (*rc = run_graphed(h, key, body, use_graph != 0));
}

// ---------------------------------------------------------------- operator level
// the operator descriptor as the launcher's arguments (W is the caller's copy of d->w)
static void gemm_args_from_desc(const hx_gemm_desc* d, const DevMat& W, GemmArgs& a) {
  a.A = static_cast<const __half*>(d->a);
  a.lda = d->lda;
  a.A2 = static_cast<const __half*>(d->a2);
  a.lda2 = d->lda2;
  a.M = d->m;
  a.K1 = d->k1 > 0 ? d->k1 : W.K;
  a.W = &W;
  a.epi = d->epi;
  a.out = static_cast<__half*>(d->out);
  a.ldo = d->ldo;
  a.x = d->x;
  a.ldx = d->ldx;
  a.gate = d->gate;
  a.vec_bstride = d->vec_bstride;
  a.rows_per_img = d->rows_per_img > 0 ? d->rows_per_img : (1 << 30);
  a.gain0 = d->gain0;
  a.gain1 = d->gain1;
  a.seg1 = d->seg1;
  a.seg2 = d->seg2;
  a.rope0 = d->rope0;
  a.rope1 = d->rope1;
  a.cosT = d->cos_t;
  a.sinT = d->sin_t;
  a.eps = d->eps > 0.f ? d->eps : 1e-6f;
  a.tile = d->tile;
}

int hx_gemm(hx_handle hh, const hx_gemm_desc* d) {
  hx_ctx* h = H(hh);
  if (!h || !d || !valid_mat(d->w)) return HX_E_ARG;
  DevGuard g(h->device);
  DevMat W = to_devmat(d->w);
  GemmArgs a;
  gemm_args_from_desc(d, W, a);
  a.status = h->status;
  if (W.fmt != WF_F16 && (a.tile == 4 || (a.tile == 0 && a.M >= expand_min_rows())))
    reserve_wexp(h, static_cast<size_t>(W.N) * W.K * 2);
  a.wexp = h->wexp;
  a.wexp_bytes = h->wexp_bytes;
  cudaError_t e = gemm_launch(a, h->stream);
  return e == cudaSuccess ? HX_OK : (e == cudaErrorInvalidValue ? HX_E_ARG : HX_E_CUDA);
}

int hx_gemm_query(const hx_gemm_desc* d, int sm_count, hx_gemm_plan* out) {
  if (!d || !out || !valid_mat(d->w)) return HX_E_ARG;
  DevMat W = to_devmat(d->w);
  GemmArgs a;
  gemm_args_from_desc(d, W, a);
  GemmChoice c;
  if (gemm_choose(a, sm_count, true, c) != cudaSuccess) return HX_E_ARG;
  int expand = 0;
  DevMat f;
  if (c.expand) {  // the fp16 GEMM on the expanded weights (scratch of the handle, as hx_gemm reserves it)
    expand = 1;
    f.fmt = WF_F16;
    f.N = W.N;
    f.K = W.K;
    f.group = 64;
    f.w = W.w;
    a.W = &f;
    a.tile = 0;
    if (gemm_choose(a, sm_count, false, c) != cudaSuccess) return HX_E_ARG;
  }
  out->kernel = c.kernel;
  out->expand = expand;
  out->tile_m = c.kernel == 1 ? 128 : 256;
  out->tile_n = c.kernel == 2 ? c.tile_n : 256;
  out->tiles = c.kernel == 3 ? gemm_wt_tiles(a) : c.tiles;
  out->streamk = c.streamk;
  return HX_OK;
}

static void attn_args_from_desc(const hx_attn_desc* d, AttnArgs& a) {
  a.q = static_cast<const __half*>(d->q);
  a.ldq = d->ldq;
  a.q_col0 = d->q_col0;
  a.k = static_cast<const __half*>(d->k);
  a.ldk = d->ldk;
  a.k_col0 = d->k_col0;
  a.v = static_cast<const __half*>(d->v);
  a.ldv = d->ldv;
  a.v_col0 = d->v_col0;
  a.o = static_cast<__half*>(d->o);
  a.ldo = d->ldo;
  a.B = d->batch;
  a.H = d->heads;
  a.Tq = d->tq;
  a.Tk = d->tk;
  a.nvalid = d->nvalid;
  a.scale = d->scale;
  a.kernel = d->kernel;
}

int hx_attention(hx_handle hh, const hx_attn_desc* d) {
  hx_ctx* h = H(hh);
  if (!h || !d) return HX_E_ARG;
  DevGuard g(h->device);
  AttnArgs a;
  attn_args_from_desc(d, a);
  a.status = h->status;
  cudaError_t e = attn_launch(a, h->stream);
  return e == cudaSuccess ? HX_OK : (e == cudaErrorInvalidValue ? HX_E_ARG : HX_E_CUDA);
}

int hx_attention_query(const hx_attn_desc* d, int sm_count, int32_t* kernel) {
  if (!d || !kernel) return HX_E_ARG;
  AttnArgs a;
  attn_args_from_desc(d, a);
  const int k = attn_choose(a, sm_count);
  if (k < 0) return HX_E_ARG;
  *kernel = k;
  return HX_OK;
}

int hx_lnmod(hx_handle hh, const float* x, void* h16, int rows, int D, const float* shift, const float* scale,
             long vec_bstride, int rows_per_img, float eps) {
  hx_ctx* h = H(hh);
  if (!h || !x || !h16 || !shift || !scale) return HX_E_ARG;
  DevGuard g(h->device);
  cudaError_t e = lnmod_launch(x, static_cast<__half*>(h16), rows, D, shift, scale, vec_bstride, rows_per_img, eps,
                               h->stream);
  return e == cudaSuccess ? HX_OK : (e == cudaErrorInvalidValue ? HX_E_ARG : HX_E_CUDA);
}

int hx_rmsmod(hx_handle hh, const float* x, void* h16, int rows, int D, const float* w, const float* shift,
              const float* scale, long vec_bstride, int rows_per_img, float eps) {
  hx_ctx* h = H(hh);
  if (!h || !x || !h16 || !shift || !scale) return HX_E_ARG;
  DevGuard g(h->device);
  cudaError_t e = rmsmod_launch(x, static_cast<__half*>(h16), rows, D, w, shift, scale, vec_bstride, rows_per_img,
                                eps, h->stream);
  return e == cudaSuccess ? HX_OK : (e == cudaErrorInvalidValue ? HX_E_ARG : HX_E_CUDA);
}

// ---------------------------------------------------------------- rope tables (host)
int hx_rope_anima(int gh, int gw, double theta, int ntok, float* cs, float* sn) {
  if (gh <= 0 || gw <= 0 || ntok < gh * gw || !cs || !sn || theta <= 0) return HX_E_ARG;
  const int dim_h = 128 / 6 * 2, dim_t = 128 - 2 * dim_h, nt = dim_t / 2, nh = dim_h / 2;
  std::vector<double> fh(nh);
  for (int i = 0; i < nh; ++i) fh[i] = 1.0 / std::pow(theta, (2.0 * i) / dim_h);
  std::memset(cs, 0, sizeof(float) * 64 * ntok);
  std::memset(sn, 0, sizeof(float) * 64 * ntok);
  for (int tk = 0; tk < gh * gw; ++tk) {
    const int hh = tk / gw, ww = tk % gw;
    for (int d = 0; d < 64; ++d) {
      const double ang = d < nt ? 0.0 : d < nt + nh ? hh * fh[d - nt] : ww * fh[d - nt - nh];
      cs[tk * 64 + d] = static_cast<float>(std::cos(ang));
      sn[tk * 64 + d] = static_cast<float>(std::sin(ang));
    }
  }
  return HX_OK;
}

int hx_rope_moss(int Hh, int Ww, int T, const float* bands, int ntok, float* cs, float* sn) {
  if (Hh < 0 || Ww < 0 || T < 0 || !bands || !cs || !sn || ntok < Hh * Ww + T) return HX_E_ARG;
  const int Nimg = Hh * Ww, N = Nimg + T;
  std::memset(cs, 0, sizeof(float) * 64 * ntok);
  std::memset(sn, 0, sizeof(float) * 64 * ntok);
  for (int tk = 0; tk < N; ++tk) {
    double c[4] = {0, 0, 0, 0};
    if (tk < Nimg) {
      c[1] = T;
      c[2] = tk / Ww - (Hh - 1) / 2.0;
      c[3] = tk % Ww - (Ww - 1) / 2.0;
    } else {
      c[1] = tk - Nimg;
    }
    for (int d = 0; d < 64; ++d) {
      const double a = c[d / 16] * static_cast<double>(bands[d % 16]);
      cs[tk * 64 + d] = static_cast<float>(std::cos(a));
      sn[tk * 64 + d] = static_cast<float>(std::sin(a));
    }
  }
  return HX_OK;
}

}  // extern "C"

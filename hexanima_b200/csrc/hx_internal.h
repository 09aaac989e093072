// Internal host-side declarations shared by the kernel files and the C-ABI layer.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

namespace hx {

// Weight storage formats on the device (the layouts are described in gemm.cu).
enum WFmt : int { WF_F16 = 0, WF_Q8 = 1, WF_Q4A = 2, WF_Q4 = 3 };

// GEMM epilogues. They follow the flush modes of the reference GEMM engine
// (hexagon/mega/gemm2.c:58-82, moss/hexagon/mega/gemm2.c:89-123).
enum Epi : int {
  EPI_STORE = 0,  // out16 = acc
  EPI_RESID = 1,  // x32 += gate[n] * acc                      (mode 1; mode 4 is the same with full K)
  EPI_GELU = 2,   // out16 = gelu_erf(acc)                      (mode 2)
  EPI_RMS = 3,    // per 128-col head: rms * gain (+ rope)      (mode 3)
  EPI_SITU = 5,   // tile cols [0,128) up, [128,256) gate -> 128 outputs   (mode 5)
  EPI_STORE32 = 6,  // x32 = acc (fp32 output in the x / ldx fields; glue GEMMs)
};

// A weight matrix W[N][K] in device memory, in one of the WFmt layouts.
struct DevMat {
  int fmt = WF_F16;
  int N = 0, K = 0;       // output features, reduction length (K includes appended LoRA rows)
  int group = 32;         // quantisation group along K (q8: 32 or 64; q4/q4a: 32)
  void* w = nullptr;      // fp16 [N][K] | u8 [N][K] (offset binary) | u8 [N][K/2] (packed nibbles)
  __half* scale = nullptr;  // [K/group][N]
  __half* minv = nullptr;   // [K/group][N] (q4a only)
};

struct GemmArgs {
  // A: fp16 row-major [M][lda]; columns [0, K1) come from A, [K1, K) from A2 (row-major [M][lda2]).
  const __half* A = nullptr;
  int lda = 0;
  const __half* A2 = nullptr;
  int lda2 = 0;
  int M = 0, K1 = 0;
  const DevMat* W = nullptr;
  int epi = EPI_STORE;
  // outputs
  __half* out = nullptr;  // fp16 [M][ldo]
  int ldo = 0;
  float* x = nullptr;     // fp32 residual [M][ldx]
  int ldx = 0;
  // per-column vectors; for row m the image is m / rows_per_img and the vector is vec + img * vec_bstride
  const float* gate = nullptr;
  long vec_bstride = 0;
  int rows_per_img = 1 << 30;
  // EPI_RMS: columns < seg1 use gain0 (rope if rope0), < seg2 gain1 (rope if rope1), others are stored plain
  const float* gain0 = nullptr;
  const float* gain1 = nullptr;
  int seg1 = 0, seg2 = 0, rope0 = 0, rope1 = 0;
  const float* cosT = nullptr;  // [rows_per_img][64]
  const float* sinT = nullptr;
  float eps = 1e-6f;
  int* status = nullptr;
  int max_ctas = 0;  // 0 = one CTA per SM
  // 0 auto, 1 single-CTA 128x256 tiles, 2 CTA-pair 256x256 tiles, 3 q8 weights in TMEM, 4 quantised
  // weights expanded to fp16 in wexp first (auto does so from expand_min_rows() rows up), 5 CTA-pair
  // 256x224 tiles (GELU or store epilogue, fp16 or q8 weights)
  int tile = 0;
  // scratch for the expanded weights (fp16 [N][K]); nullptr or too small: dequantise inside the GEMM
  __half* wexp = nullptr;
  size_t wexp_bytes = 0;
};

struct AttnArgs {
  // Q rows [B][Tq][ldq] fp16, head h at column q_col0 + 128 h; likewise K and V.
  const __half* q = nullptr;
  int ldq = 0, q_col0 = 0;
  const __half* k = nullptr;
  int ldk = 0, k_col0 = 0;
  const __half* v = nullptr;
  int ldv = 0, v_col0 = 0;
  __half* o = nullptr;  // [B][Tq][ldo], head h at column 128 h
  int ldo = 0;
  int B = 1, H = 1, Tq = 0, Tk = 0;
  int nvalid = 0;       // keys with index >= nvalid get probability 0 (0 = all Tk keys valid)
  float scale = 1.0f;   // logits are q.k * scale
  int* status = nullptr;
  // 0 auto (the short-key kernel for 128 < Tk <= 256 with at most six 128-query tiles per SM), 1 the general
  // online-softmax kernel, 2 the short-key kernel (Tk <= 256)
  int kernel = 0;
};

cudaError_t gemm_launch(const GemmArgs& a, cudaStream_t s);
cudaError_t attn_short_launch(const AttnArgs& a, cudaStream_t s);
int attn_choose(const AttnArgs& a, int sms);
// q8 GEMM with the dequantised weights in TMEM (gemm_wt.cu): STORE / GELU / RESID / RMS epilogues,
// N a multiple of 256; gemm_launch picks it for the RMS epilogue when its tiles fill the GPU (tile 3
// forces it)
// what gemm_launch runs for a GEMM: kernel 1 single-CTA 128x256 tiles, 2 CTA pairs (256 x tile_n per
// pair, stream-K tail when streamk), 3 q8 weights in TMEM; expand: quantised weights go to fp16 first and
// the fp16 GEMM that follows is chosen for tile 0 (tiles / tile_n then belong to that GEMM)
struct GemmChoice {
  int kernel = 0;
  bool expand = false;
  int tile_n = 256;
  int streamk = 0;
  int tiles = 0;
};
cudaError_t gemm_choose(const GemmArgs& a, int sms, bool have_scratch, GemmChoice& c);
bool gemm_wt_eligible(const GemmArgs& a);
int gemm_wt_tiles(const GemmArgs& a);
cudaError_t gemm_wt_launch(const GemmArgs& a, cudaStream_t s);
cudaError_t attn_launch(const AttnArgs& a, cudaStream_t s);
// quantised W -> fp16 [N][K] at dst (expand.cu), bit-identical to the GEMMs' own dequantisers
cudaError_t expand_launch(const DevMat& W, __half* dst, cudaStream_t s);
// GEMMs with at least this many rows expand quantised weights first when a scratch is given
// (default 3072 = two 1536-token images; environment HX_EXPAND_ROWS overrides, read once)
int expand_min_rows();

// memory-bound kernels (elem.cu)
cudaError_t lnmod_launch(const float* x, __half* h, int rows, int D, const float* shift, const float* scale,
                         long vec_bstride, int rows_per_img, float eps, cudaStream_t s);
cudaError_t rmsmod_launch(const float* x, __half* h, int rows, int D, const float* w, const float* shift,
                          const float* scale, long vec_bstride, int rows_per_img, float eps, cudaStream_t s);
cudaError_t modulation_batch_launch(const __half* const* Atab, const __half* const* Btab, int nblk, const float* emb,
                                    const float* lora, float* out, size_t out_stride, float* se, int nsite, int D,
                                    int R, int O, cudaStream_t s);
cudaError_t modulation_launch(const __half* Aw, const __half* Bw, const float* emb, const float* lora, float* out,
                              int nsite, int D, int R, int O, cudaStream_t s);
cudaError_t f32_to_f16_launch(const float* src, __half* dst, size_t n, cudaStream_t s);
// one CTA whose thread 0 waits with a run-time limit on an mbarrier that is arrived on only if `arrive`
cudaError_t wait_selftest_launch(int* status, unsigned long long limit_ns, int arrive, cudaStream_t s);

// per-step glue (glue.cu)
struct Sigmas {
  float s[8];
};
cudaError_t temb_launch(Sigmas sig, int S, int D, const __half* w_norm, float* tp, float* emb, cudaStream_t s);
cudaError_t gemv_rows_launch(const __half* W, const float* X, float* Y, int S, int K, int O, int silu_in,
                             const float* add, int add_ld, int y_ld, cudaStream_t s);
cudaError_t patchify_launch(const float* lat, __half* P, int B, int C, int H, int W, int kpad, cudaStream_t s);
cudaError_t unpatch_euler_launch(const float* y, float* lat, int B, int C, int H, int W, int ldy, float dt,
                                 cudaStream_t s);
cudaError_t pad_cols_launch(const __half* src, __half* dst, int rows, int cols, int ld_dst, cudaStream_t s);
// MOSS sampler glue (glue.cu)
cudaError_t moss_temb_launch(Sigmas codes, int S, float* e, cudaStream_t s);
cudaError_t moss_mix_launch(const float* z, const float* x0, const float* Q, __half* xin, int B, int Ni, int ntok,
                            int kp, cudaStream_t s);
cudaError_t moss_x0_launch(const float* z, const float* v, float* x0, int B, int Ni, int ntok, int ldv,
                           cudaStream_t s);
cudaError_t moss_emb_pad_launch(const __half* W, const float* bias, __half* Wp, int D, int kp, cudaStream_t s);

// weight repacking from the reference pack records (repack.cu)
cudaError_t repack_tiles_launch(const uint8_t* rec, int nb, int kb, bool q8, void* dst, __half* scale, int row0,
                                int nrows_total, int mode, cudaStream_t s);
// scale * B * A folded into the base columns [0, k_base) of a q8 matrix, requantised per group
// (lora.cu). row_mode 1: MOSS up_gate device row order; floor_mode 0 MOSS, 1 Anima scale floor.
cudaError_t lora_fold_launch(const DevMat& W, int k_base, const float* B, const float* A, int rank, float lscale,
                             int row_mode, int floor_mode, cudaStream_t s);
// The Anima LLM adapter (adapter.cu): fp16 device weights, 6 blocks.
struct AdapterWeights {
  const __half* embed = nullptr;  // [vocab][1024]
  int vocab = 0;
  struct Block {
    const __half *norm_sa, *sa_q, *sa_k, *sa_v, *sa_o, *sa_qn, *sa_kn;
    const __half *norm_ca, *ca_q, *ca_k, *ca_v, *ca_o, *ca_qn, *ca_kn;
    const __half *norm_mlp, *mlp0_w, *mlp0_b, *mlp2_w, *mlp2_b;
  } blocks[6];
  const __half *out_w = nullptr, *out_b = nullptr, *norm = nullptr;
};
// hidden fp32 [S][1024] on the device, ids / wts on the host ([L], L <= 512), out fp32 [512][1024] on the
// device; synchronous on s
cudaError_t adapter_run(const AdapterWeights& W, const float* hidden, int S, const int32_t* ids_host,
                        const float* wts_host, int L, float* out, int* status, cudaStream_t s);
// the rank-128 LoRA slot fold (lorasvd.cu): W the LoRA-carrying matrix (K = k_base + 128), A the
// LoRA-A matrix whose rows a_row0 .. +127 are the slots; synchronous on s
cudaError_t lora_fold_slots(const DevMat& W, int k_base, int row_mode, const DevMat& A, int a_row0, const float* Bu,
                            const float* Au, int rank, float scale, cudaStream_t s);
int sm_count();

// Kernels of the block chain are launched with programmatic stream serialization: a kernel's launch and
// prologue (barrier set-up, TMEM allocation, tensor-map prefetch) overlap the tail of the kernel before
// it, and it waits in grid_dep_wait() (hx_ptx.cuh) before its first global-memory access. Every kernel
// launched through pdl_attr executes that wait. HX_PDL=0 in the environment turns it off (read once).
bool pdl_enabled();
// appends the attribute to attrs when enabled; returns the new attribute count
inline unsigned pdl_attr(cudaLaunchAttribute* attrs, unsigned n) {
  if (!pdl_enabled()) return n;
  attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[n].val.programmaticStreamSerializationAllowed = 1;
  return n + 1;
}
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  cfg.attrs = attr;
  cfg.numAttrs = pdl_attr(attr, 0);
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace hx

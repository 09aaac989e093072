/* hxdit.h — C ABI of the B200 DiT block runtime (libhxdit.so).
 *
 * Drop-in for the per-block operator the reference drives over FastRPC and the chain runner
 * around it (Herolias/hexanima):
 *   mega_open / mega_close         hexagon/mega/mega_imp.c:16-18
 *   mega_block(meta, wfd, bfd, mod, times, rc)   hexagon/mega/mega.idl:10, hexagon/mega/blk.c:186-197,
 *                                  moss/hexagon/mega/blk.c:269-281
 *   rpcmem buffers + fds           hexagon/mega/megarun.cpp:109-127
 *   per-block modulation thread    hexagon/mega/megarun.cpp:158-171
 *   chain loop over blocks         hexagon/mega/megarun.cpp:176-184
 *   gemm_run_geo / attn_run / k_*  hexagon/mega/gemm2.h:16, blk.c:54, kern.h:11-32 (operator level)
 *
 * Conventions: plain pointers and sizes, no C++ or torch types. Functions return HX_OK (0) or a
 * negative HX_E* code; no call aborts the process or traps the GPU. Device pointers ("_dev")
 * are CUDA device addresses on the handle's device; work is ordered on the handle's stream.
 * Device kernels bound their waits; a timeout is reported through hx_status / *rc = HX_E_TIMEOUT.
 */
#ifndef HXDIT_H
#define HXDIT_H
#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define HX_API __attribute__((visibility("default")))
#else
#define HX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status codes
 * rc values of hx_mega_block follow the reference's (hexagon/mega/blk.c:110-127;
 * moss/hexagon/mega/blk.c:148-155): 0 ok, negative = failure. */
#define HX_OK 0
#define HX_E_ARG (-1)       /* bad argument / handle / size */
#define HX_E_CUDA (-2)      /* CUDA runtime error (launch, copy, allocation) */
#define HX_E_NOWEIGHTS (-5) /* unknown weight handle  (reference: -5 weights map failed) */
#define HX_E_NOBLOB (-6)    /* unknown blob buffer    (reference: -6 no blob) */
#define HX_E_RANGE (-7)     /* meta offsets reach outside the blob (reference: -7 blob map) */
#define HX_E_FORMAT (-8)    /* pack bytes do not match a known pack layout */
#define HX_E_TIMEOUT (-77)  /* a device-side bounded wait expired (reference: -77 HMX self-test) */
#define HX_E_SCRATCH (-9)   /* request larger than a fixed static scratch area (hx_modulation_noalloc) */

/* ------------------------------------------------------------------ models and weight formats */
#define HX_MODEL_ANIMA 1    /* hexagon/mega: D 2048, 16 heads, self + cross attention, GELU MLP */
#define HX_MODEL_MOSS 2     /* moss/hexagon/mega: D 3072, 24 heads, joint attention, SiTU MLP, LoRA K tiles */
#define HX_MODEL_MOSS_PROJ 3 /* MOSS text projection (mode 2): text_embedder.proj 4096 -> 3072 + bias, the pack of
                               moss/export_moss.py:61-65 ([96 nb][132 kb] q8 tiles at offset 0, padded to the
                               block-pack size, or unpadded); the weight set serves only meta MODE 2 */

#define HX_FMT_F16 0        /* fp16 W[N][K] */
#define HX_FMT_Q8 1         /* u8 W[N][K] offset binary (q+128), fp16 scale[K/group][N], group 32|64 */
#define HX_FMT_Q4A 2        /* u8 W[N][K/2] nibbles (see hx_mat), fp16 scale and min [K/32][N]: nib*s+m */
#define HX_FMT_Q4 3         /* as Q4A without min: (nib-8)*s */

typedef struct hx_ctx* hx_handle;

/* ------------------------------------------------------------------ lifecycle
 * hx_open: mega_open (hexagon/mega/mega_imp.c:16). Binds CUDA device `device`, creates a stream. */
HX_API int hx_open(int device, hx_handle* out);
/* hx_close: mega_close (hexagon/mega/mega_imp.c:18). Frees every buffer and weight set of the handle. */
HX_API int hx_close(hx_handle h);
/* The CUDA stream (cudaStream_t) the handle launches on; hx_set_stream replaces it (caller-owned). */
HX_API int hx_get_stream(hx_handle h, void** stream);
HX_API int hx_set_stream(hx_handle h, void* stream);
HX_API int hx_sync(hx_handle h);
/* Device status word written by bounded waits (0 = ok, else the code of the wait that expired);
 * reading it synchronises the stream and clears it. */
HX_API int hx_status(hx_handle h, int* status);
/* Self-test of the bounded device wait, in the spirit of the reference's HMX self-test that answers
 * rc -77 when its check fails (moss/hexagon/mega/blk.c:112-118,149-155). One thread waits on a
 * shared-memory mbarrier with the given limit (1 us .. 2 s); when arrive != 0 another thread arrives on
 * it and the wait succeeds (*rc = HX_OK), otherwise the wait expires and the kernel returns with the
 * status word set, which the host reads: *rc = HX_E_TIMEOUT. Nothing else runs in that kernel. The
 * status word is cleared before and after; the handle stays usable. Synchronises the handle's stream. */
HX_API int hx_wait_selftest(hx_handle h, int64_t limit_ns, int arrive, int32_t* rc);
/* Device pointer to the status word, for callers that launch operators on their own streams. */
HX_API int hx_status_ptr(hx_handle h, int** status_dev);

/* ------------------------------------------------------------------ buffers
 * Device buffers named by small integer "fds", the analogue of the rpcmem buffers + fds that
 * megarun maps for the DSP (hexagon/mega/megarun.cpp:109-127). */
HX_API int hx_buf_alloc(hx_handle h, size_t bytes, int* fd);
HX_API int hx_buf_free(hx_handle h, int fd);
HX_API int hx_buf_ptr(hx_handle h, int fd, void** dev);
HX_API int hx_buf_write(hx_handle h, int fd, size_t off, const void* src, size_t bytes); /* host -> device, stream-ordered, returns when copied */
HX_API int hx_buf_read(hx_handle h, int fd, size_t off, void* dst, size_t bytes);        /* device -> host, synchronises */

/* ------------------------------------------------------------------ weights */
typedef struct {
  int fmt;      /* HX_FMT_* */
  int n, k;     /* W is [n][k]: n output features, k reduction length (LoRA-B rows included) */
  int group;    /* quantisation group along k */
  void* w;      /* fp16 [n][k] | u8 [n][k] | u8 [n][k/2]: in every 32-bit word (8 consecutive k),
                   k sits at nibble (k>>1) + 4*(k&1) */
  void* scale;  /* fp16 [k/group][n] */
  void* minv;   /* fp16 [k/32][n] (Q4A) */
} hx_mat;

/* matrix slots of hx_weight_desc.mats */
#define HX_W_QKV 0   /* Anima [3D][D] (q|k|v rows); MOSS [3D][D] when lora == 0 */
#define HX_W_O 1     /* self-attention output [D][D(+128)] */
#define HX_W_CQ 2    /* Anima cross-attention q [D][D] */
#define HX_W_CKV 3   /* Anima cross-attention k|v [2D][Cd] */
#define HX_W_CO 4    /* Anima cross-attention output [D][D] */
#define HX_W_M1 5    /* Anima mlp.layer1 [F][D]; MOSS up_gate [2F][D(+128)], rows grouped per 256:
                        128 up rows then the 128 gate rows of the same outputs */
#define HX_W_M2 6    /* Anima mlp.layer2 [D][F]; MOSS ffn_down [D][F(+128)] */
#define HX_W_Q 7     /* MOSS with lora: q, k, v each [D][D+128] */
#define HX_W_K 8
#define HX_W_V 9
#define HX_W_AQKV 10 /* MOSS LoRA down matrices: [384][D], [128][D], [128][D], [128][F] */
#define HX_W_AO 11
#define HX_W_AUG 12
#define HX_W_ADN 13
#define HX_NMATS 14

typedef struct {
  int model;         /* HX_MODEL_* */
  int D, F, Cd, H;   /* hidden size, FFN width, context width (Anima), heads */
  int lora;          /* MOSS: matrices carry 128 LoRA-B rows at the end of K (export_moss.py:14-27) */
  hx_mat mats[HX_NMATS];
  const float* gain; /* device fp32. Anima [512]: q*1/sqrt(128), k, cq*1/sqrt(128), ck (export_all.py:31-32).
                        MOSS [128+128+D+D]: q/sqrt(128), k, norm1, norm2 (export_moss.py:39) */
  const void* modA;  /* Anima fp16 [3][256][D]: adaln_modulation_{self_attn,cross_attn,mlp}.1 */
  const void* modB;  /* Anima fp16 [3][6144][256]: adaln_modulation_*.2 */
} hx_weight_desc;

/* Load one reference block pack (host bytes of blkNN.bin) into device memory owned by the handle.
 * Anima: fp16 (W_TOTAL = 138,416,128 B) or q8 (WQ_TOTAL) packs, recognised by size as megarun
 * does (hexagon/mega/megarun.cpp:97; layout hexagon/mega/blk_wlayout.h:3-20). MOSS: q8 pack of
 * 135,397,376 B (moss/hexagon/mega/blk_meta.h:6-17). */
HX_API int hx_weights_load(hx_handle h, int model, const void* pack, size_t bytes, int* wfd);
/* Bind caller-owned device arrays already in the device layout (no copy; they must outlive use). */
HX_API int hx_weights_bind(hx_handle h, const hx_weight_desc* desc, int* wfd);
HX_API int hx_weights_free(hx_handle h, int wfd);
/* Fold scale * B * A (a LoRA delta of rank 1..128) into the q8 matrix `slot` of weight set wfd, in
 * place: dequantise, add, and requantise every K-group with the pack rule of the reference's fold
 * tool (moss/mossrun/lorafold.cpp:138-156 `quant`; scale floor 6.2e-5 for MOSS, 0 -> 1.0 for Anima).
 * Only the base columns change: with MOSS LoRA K rows (desc.lora) the first K-128.
 *   B: device fp32 [N][rank] in the matrix's logical row order (MOSS up_gate: rows [0,F) up,
 *      [F,2F) gate; Anima fused qkv: q, k, v rows).   A: device fp32 [rank][K_base].
 * The base-tile variant of the reference's rank-128-slot fold (lorafold.cpp:200-284). Bound
 * (caller-owned) weights are modified too. Runs on the handle's stream. */
HX_API int hx_lora_fold(hx_handle h, int wfd, int slot, const float* B_dev, const float* A_dev, int rank, float scale);

/* Projections of a MOSS block that carry rank-128 LoRA slots (export_moss.py:14-27). */
#define HX_LORA_Q 0   /* slots: HX_W_Q K columns [D, D+128) and HX_W_AQKV rows [0, 128) */
#define HX_LORA_K 1   /* HX_W_K, HX_W_AQKV rows [128, 256) */
#define HX_LORA_V 2   /* HX_W_V, HX_W_AQKV rows [256, 384) */
#define HX_LORA_O 3   /* HX_W_O, HX_W_AO */
#define HX_LORA_UG 4  /* HX_W_M1 (up_gate), HX_W_AUG */
#define HX_LORA_DN 5  /* HX_W_M2 (ffn_down), HX_W_ADN */
/* Fold scale * B * A into the rank-128 LoRA slots of projection `proj` of a MOSS q8 weight set with
 * LoRA (desc.lora = 1 or a MOSS pack): the slots become the best rank-128 approximation of their
 * current delta plus scale * B * A, found by the Gram-eigen / SVD route of the reference's fold tool
 * (moss/mossrun/lorafold.cpp:200-284 `fold`, singular values on the B side), and are requantised
 * with the pack rule (lorafold.cpp:138-156). The base columns do not change.
 *   B: device fp32 [N][rank] in the projection's logical row order (up_gate: [0,F) up, [F,2F) gate).
 *   A: device fp32 [rank][K_base] (K_base = D, or F for ffn_down).   rank 1..128.
 * Synchronous on the handle's stream (host eigen-solves between device steps); returns HX_E_FORMAT
 * for a weight set without LoRA slots or with non-q8 matrices. */
HX_API int hx_lora_fold_slots(hx_handle h, int wfd, int proj, const float* B_dev, const float* A_dev, int rank,
                              float scale);

/* Apply a LoRA overlay file (blkNN.ovl written by moss/make_lora_overlay.py:54-56 and
 * moss/mossrun/lorafold.cpp:284-288: u32 n, then n records of u64 pack offset, u32 length, bytes)
 * to a block pack in host memory before hx_weights_load. All records are checked first; on a
 * truncated overlay or a record outside the pack it returns HX_E_FORMAT and leaves the pack as it was. */
HX_API int hx_pack_apply_overlay(void* pack, size_t pack_bytes, const void* ovl, size_t ovl_bytes);

/* ------------------------------------------------------------------ the per-block operator */
/* Anima meta[] slots: byte offsets into the blob buffer, then scalars.
 * Same order as hexagon/mega/blk_meta.h:3-5. Weight-offset slots are ignored (weights come from
 * wfd). Device blob layout (hx_blob_layout fills it):
 *   X   fp32 [B][NTOK][D] residual stream, updated in place
 *   CTX fp16 [B][NCTX][Cd]
 *   MOD fp32 [9][D] (shift, scale, gate per site), read when the call passes mod == NULL
 *   COS, SIN fp32 [NTOK][64]
 *   H fp16 [B*NTOK][D]; Q fp16 [B*NTOK][3D] (fused q|k|v; K and V point into it);
 *   O fp16 [B*NTOK][D]; MID fp16 [B*NTOK][F]; CK fp16 [B*NCTX][2D] (fused ck|cv) */
enum {
  HX_A_X = 0, HX_A_CTX, HX_A_MOD, HX_A_GAIN, HX_A_COS, HX_A_SIN,
  HX_A_WSQ, HX_A_WSK, HX_A_WSV, HX_A_WSO, HX_A_WCQ, HX_A_WCK, HX_A_WCV, HX_A_WCO, HX_A_WM1, HX_A_WM2,
  HX_A_H, HX_A_Q, HX_A_K, HX_A_V, HX_A_O, HX_A_T, HX_A_MID, HX_A_CK, HX_A_CV,
  HX_A_NTOK, HX_A_NCTX, HX_A_STOP, HX_A_NW, HX_A_REL, HX_A_FIRST, HX_A_Q8,
  HX_A_NMETA,               /* 32, the reference's M_NMETA */
  HX_A_BATCH = HX_A_NMETA,  /* extension: images stacked in the blob (default 1) */
  HX_A_NMETA_EXT
};
/* MOSS meta[] slots (moss/hexagon/mega/blk_meta.h:3-4). Blob layout:
 *   X fp32 [B][NTOK][D]; COS, SIN fp32 [NTOK][64]; H fp16 [B*NTOK][D]; Q fp16 [B*NTOK][3D] (fused);
 *   O fp16 [B*NTOK][D]; MID fp16 [B*NTOK][F]; LQ fp16 [B*NTOK][384]; LO, LU, LD fp16 [B*NTOK][128];
 *   mod: fp32 [6][D] (shift_a, scale_a, gate_a, shift_f, scale_f, gate_f) passed by the call or at CS.
 * MODE (moss/hexagon/mega/blk_meta.h:4, blk.c:229-237):
 *   0  DiT block.
 *   1  text-refiner block: the LoRA-A GEMMs are skipped; the host fills LQ/LO/LU/LD with the bias
 *      selector (fp16 1.0 in column 0 of every 128-column part, 0 elsewhere) so the pack's LoRA K rows
 *      (row 0 = bias, export_moss.py:43-59) add the biases; mod = (0, 0, 1, 0, 0, 1) rows.
 *   2  text projection with a HX_MODEL_MOSS_PROJ weight set: X += gate_a * (H . Wp + bias), H fp16
 *      [B*NTOK][text width] (the Cd of hx_blob_layout, 4096), the bias through the LQ selector. */
enum {
  HX_S_X = 0, HX_S_COS, HX_S_SIN, HX_S_H, HX_S_Q, HX_S_K, HX_S_V, HX_S_O, HX_S_T, HX_S_MID,
  HX_S_LQ, HX_S_LO, HX_S_LU, HX_S_LD, HX_S_NTOK, HX_S_NVALID, HX_S_STOP, HX_S_NW, HX_S_REL,
  HX_S_FIRST, HX_S_MODE, HX_S_NCB, HX_S_FMT, HX_S_ROWS, HX_S_CS, HX_S_WOFF,
  HX_S_NMETA,               /* 26, the reference's M_NMETA */
  HX_S_BATCH = HX_S_NMETA,  /* extension: images stacked in the blob (default 1) */
  HX_S_SP,                  /* extension: P > 1 runs the attention sequence-parallel over the handle's
                               communicator (hx_sp_init): NTOK is this rank's token count, NVALID the
                               image's valid token count over all P shards; batch must be 1 */
  HX_S_NMETA_EXT
};

/* Fill meta[] with a blob layout (megarun.cpp:42-57 layout()) for `batch` images; *total = bytes.
 * nmeta must be >= HX_A_NMETA_EXT (Anima) or HX_S_NMETA_EXT (MOSS). For MOSS, nctx is unused, the mod
 * vectors go to the CS slot, and a Cd above D (the text width of MODE 2) widens the H region to Cd. */
HX_API int hx_blob_layout(int model, int ntok, int nctx, int batch, int D, int F, int Cd, int32_t* meta, int nmeta,
                   size_t* total);

/* Ulysses sequence parallelism across GPUs (no counterpart in the single-device reference):
 * rank 0 creates a 128-byte id with hx_sp_unique_id and every rank passes it to hx_sp_init (a
 * collective over the P ranks). MOSS blocks with meta[HX_S_SP] = P then exchange q|k|v token shards
 * for head shards (NCCL grouped send/recv), attend over the full sequence on H/P heads and exchange
 * the outputs back. The communicator lives until hx_close. */
HX_API int hx_sp_unique_id(void* id128);
HX_API int hx_sp_init(hx_handle h, int nranks, int rank, const void* id128);

/* One DiT block forward: mega_block (hexagon/mega/mega.idl:10). mod: host fp32 modulation
 * (Anima 9*D floats, MOSS 6*D; modlen in bytes) copied per call, or NULL to read it from the blob.
 * times[0..]: per-stage microseconds when ntimes > 0 (synchronises; slot order of the reference's
 * TICKs, times[24] = entry latency). With meta SP > 1 and ntimes > 19 the attention sub-stage slots
 * (times[17..22] in the reference, blk.c:178) hold the Ulysses parts: [17] pack + q|k|v all-to-all,
 * [18] attention on the rank's heads, [19] o all-to-all + unpack. *rc: HX_OK or a negative HX_E* code. */
HX_API int hx_mega_block(hx_handle h, const int32_t* meta, int nmeta, int wfd, int bfd, const uint8_t* mod, int modlen,
                  int32_t* times, int ntimes, int32_t* rc);

/* Per-block AdaLN modulation of an Anima block (megarun.cpp:158-171):
 * for site s: mod[3s..3s+2][D] = B_s (A_s silu(emb)) + lora[0:3D]. emb [D], lora [3D], mod [9D]
 * device fp32; mod_dev must hold 9*D + 3*256 floats (the tail is scratch). */
HX_API int hx_modulation(hx_handle h, int wfd, const float* emb_dev, const float* lora_dev, float* mod_dev);

/* Allocation-free variant of hx_modulation, with no counterpart in the reference. For callers that
 * cannot call cudaMalloc: code that runs while another thread captures a CUDA graph in the global
 * capture mode, hosts that run from a fixed, pre-reserved memory pool (as the reference's DSP side runs
 * from a fixed VTCM/rpcmem region), or callers that never open a handle because hx_open allocates.
 * It needs no handle: modA [nsite][256][D] and modB [nsite][3D][256] are fp16 device arrays, both
 * 16-byte aligned (else HX_E_ARG, checked before any launch), emb [D], lora [3D] (may be NULL) and
 * mod [nsite][3D] fp32 device arrays, stream a cudaStream_t (NULL = the legacy default stream) of the
 * current device. The 256-wide hidden vectors live in a static device
 * array of 4096 floats (16 KB) that every GPU loading the library holds until the process exits, so
 * nsite * 256 must be <= 4096 (else HX_E_SCRATCH). The first call on a device looks up that array's
 * device address with the device current; make that first call before any stream capture. That address
 * is remembered per device index for the life of the process: after cudaDeviceReset on a device, do not
 * call this function on it again. Returns HX_E_CUDA if either launch is refused. All calls
 * share the array and each call overwrites the part it reads before reading it; calls whose kernels
 * overlap on the GPU (different streams without ordering) race on it. Allocates nothing. */
HX_API int hx_modulation_noalloc(const void* modA, const void* modB, const float* emb_dev, const float* lora_dev,
                                 float* mod_dev, int nsite, int D, void* stream);

/* Run `count` blocks in order on one blob: the megarun chain (megarun.cpp:176-184).
 * Anima: mods_dev NULL -> each block's modulation is computed from emb_dev/lora_dev first;
 * otherwise mods_dev holds count*9*D floats. skipmask bit k skips block k (x passes through).
 * use_graph != 0 captures the chain once in a CUDA graph and replays it while the arguments repeat. */
HX_API int hx_chain(hx_handle h, const int32_t* meta, int nmeta, const int* wfds, int count, int bfd,
             const float* mods_dev, const float* emb_dev, const float* lora_dev, uint32_t skipmask, int use_graph,
             int32_t* rc);

/* ------------------------------------------------------------------ per-step glue and the sampler
 * Anima step glue of phone/animad.cpp:423-492, on the GPU: timestep embedding (σ used directly as t,
 * [cos | sin] with frequencies 10000^(-i/(D/2)), RMSNorm * t_embedding_norm), t_embedder
 * lora = linear_2(silu(linear_1(tp))), patchify (16 latent channels + a zero 17th, feature c*4+a*2+b),
 * x_embedder 68 -> D, the block chain, final layer (LayerNorm * (1 + scale) + shift with
 * [shift | scale] = B_f (A_f silu(emb)) + lora[0:2D], linear D -> 64), unpatchify, Euler update. */
typedef struct {
  int D;                /* hidden size (2048) */
  const void* t_norm;   /* fp16 [D]       t_embedding_norm.weight */
  const void* t_lin1;   /* fp16 [D][D]    t_embedder.1.linear_1.weight */
  const void* t_lin2;   /* fp16 [3D][D]   t_embedder.1.linear_2.weight */
  const void* x_emb;    /* fp16 [D][68]   x_embedder.proj.1.weight */
  const void* f_modA;   /* fp16 [256][D]  final_layer.adaln_modulation.1.weight */
  const void* f_modB;   /* fp16 [2D][256] final_layer.adaln_modulation.2.weight */
  const void* f_lin;    /* fp16 [64][D]   final_layer.linear.weight */
} hx_anima_glue_desc;
/* Copy the glue weights (device pointers) into handle-owned memory; *gfd names them. */
HX_API int hx_glue_load(hx_handle h, const hx_anima_glue_desc* d, int* gfd);
/* Full sample on the blob of `meta` (Anima layout; CTX, COS and SIN filled by the caller):
 * latent_dev fp32 [B][16][lat_h][lat_w] is denoised in place over nsteps Euler steps
 * (nsteps <= 8). sigmas: host [nsteps + 1] or NULL for the animad schedule
 * s = linspace(1, 0.001, nsteps), sigma = 3s / (1 + 2s), sigma_nsteps = 0 (animad.cpp:397-399).
 * use_graph != 0 captures the whole sample once per argument set and replays it. */
HX_API int hx_anima_sample(hx_handle h, int gfd, const int32_t* meta, int nmeta, const int* wfds, int nblk, int bfd,
                           float* latent_dev, int lat_h, int lat_w, int nsteps, const float* sigmas, int use_graph,
                           int32_t* rc);

/* The Anima LLM adapter (phone/animad.cpp:179-218): 6 blocks (dim 1024, 16 heads x 64, MLP 4096) that turn
 * T5 token ids and the LLM's hidden states into the DiT cross-attention context. Weights: fp16 device
 * arrays, names as in the checkpoint (llm_adapter.*); copied by hx_adapter_load. */
typedef struct {
  const void* norm_sa;  /* [1024] norm_self_attn.weight */
  const void* sa_q;     /* [1024][1024] self_attn.q_proj.weight (k_proj, v_proj, o_proj alike) */
  const void* sa_k;
  const void* sa_v;
  const void* sa_o;
  const void* sa_qn;    /* [64] self_attn.q_norm.weight */
  const void* sa_kn;    /* [64] self_attn.k_norm.weight */
  const void* norm_ca;  /* [1024] norm_cross_attn.weight */
  const void* ca_q;     /* cross_attn.{q,k,v,o}_proj.weight [1024][1024] */
  const void* ca_k;
  const void* ca_v;
  const void* ca_o;
  const void* ca_qn;    /* [64] */
  const void* ca_kn;    /* [64] */
  const void* norm_mlp; /* [1024] */
  const void* mlp0_w;   /* [4096][1024] mlp.0.weight */
  const void* mlp0_b;   /* [4096] */
  const void* mlp2_w;   /* [1024][4096] mlp.2.weight */
  const void* mlp2_b;   /* [1024] */
} hx_adapter_block_desc;
typedef struct {
  const void* embed;    /* [vocab][1024] llm_adapter.embed.weight */
  int vocab;
  hx_adapter_block_desc blocks[6];
  const void* out_w;    /* [1024][1024] out_proj.weight */
  const void* out_b;    /* [1024] out_proj.bias */
  const void* norm;     /* [1024] norm.weight */
} hx_anima_adapter_desc;
HX_API int hx_adapter_load(hx_handle h, const hx_anima_adapter_desc* d, int* afd);
/* Context [512][1024] fp32 (device, rows >= L zero) from hidden fp32 [S][1024] (device), token ids
 * int32 [L] and per-token weights fp32 [L] (host; 1 <= L <= 512, 0 <= id < vocab). Synchronous. */
HX_API int hx_anima_adapter(hx_handle h, int afd, const float* hidden_dev, int S, const int32_t* ids, const float* wts,
                            int L, float* out_dev);

/* MOSS sampler glue (moss/sample_ref.py:14-20 with moss_ref.py:96-120 dit_forward; mossrun.cpp:306-333):
 * weights as device arrays (copied), fp16 matrices and fp32 vectors, moss_ref names. */
typedef struct {
  int D;                  /* 3072 (a multiple of 256) */
  const void* t_lin0;     /* fp16 [D][256]   time_embedding.0.weight */
  const float* t_b0;      /* fp32 [D]        time_embedding.0.bias */
  const void* t_lin2;     /* fp16 [D][D]     time_embedding.2.weight */
  const float* t_b2;      /* fp32 [D]        time_embedding.2.bias */
  const void* mod_w;      /* fp16 [6D][D]    shared_block_modulation.weight */
  const float* mod_b;     /* fp32 [6D] */
  const void* head_w;     /* fp16 [2D][D]    video_head_modulation.weight */
  const float* head_b;    /* fp32 [2D] */
  const void* emb_w;      /* fp16 [D][128]   video_embedder.weight */
  const float* emb_b;     /* fp32 [D]        (rounded to fp16: it rides in the GEMM's K column 128) */
  const float* fin_norm;  /* fp32 [D]        final_norm_video.weight */
  const void* fin_w;      /* fp16 [128][D]   final_linear_video.weight */
  const float* mix_q;     /* fp32 [128][128] latent_mix.Q */
} hx_moss_glue_desc;
HX_API int hx_moss_glue_load(hx_handle h, const hx_moss_glue_desc* desc, int* gfd);
/* MOSS glue file glue.bin (moss/export_glue.py:1-2,17-23): "MGL1", int32 n, n entries of
 * {char name[40]; int32 dtype (0 f32, 1 f16); int32 nd; int32 dims[3]; int64 offset; int64 bytes}, data
 * 128-byte aligned. hx_mgl1_tensor finds a tensor by name in the file bytes (host memory): HX_E_FORMAT
 * for a malformed file, HX_E_RANGE if the name is absent. hx_moss_glue_load_mgl1 builds the sampler glue
 * from such a file (fp32 matrices rounded to fp16 for the device mat-vecs and GEMMs); step_codes and
 * rope.bands stay with the caller (read them with hx_mgl1_tensor). */
HX_API int hx_mgl1_tensor(const void* file, size_t bytes, const char* name, int* dtype, int* nd, int32_t dims[3],
                          const void** data, size_t* nbytes);
HX_API int hx_moss_glue_load_mgl1(hx_handle h, const void* file, size_t bytes, int* gfd);
/* A MOSS sample over nsteps <= 8 step codes (host floats, e.g. 1000 968 926 871): per step
 *   xin = z + Q x0;  rows = [video_embedder(xin) ; text rows];  mod, head = time vectors(code);
 *   nblk blocks (MODE 0, one shared mod);  v = final_linear(rms(x) * fin_norm * (1 + head1) + head0);  x0 = z - v.
 * z_dev, x0_dev: fp32 [B][128][lat_h][lat_w] (x0 in/out: zeros for a fresh sample, the clean estimate at
 * the end); text_dev: fp32 [ntext][D] refined text rows, shared by the B = meta BATCH images. meta: a MOSS
 * blob layout with NTOK >= lat_h*lat_w + ntext; NVALID is set to lat_h*lat_w + ntext; the caller fills
 * COS/SIN with hx_rope_moss(lat_h, lat_w, ntext, bands, NTOK). The whole sample runs as one CUDA graph
 * when use_graph != 0. */
HX_API int hx_moss_sample(hx_handle h, int gfd, const int32_t* meta, int nmeta, const int* wfds, int nblk, int bfd,
                          const float* z_dev, float* x0_dev, int lat_h, int lat_w, const float* text_dev, int ntext,
                          int nsteps, const float* codes, int use_graph, int32_t* rc);

/* ------------------------------------------------------------------ operator level (device pointers) */
typedef struct {
  const void* a; int lda;       /* fp16 [m][lda], columns [0,k1) */
  const void* a2; int lda2;     /* fp16 [m][lda2]: columns [k1, w.k) (LoRA extra K tiles, gemm_geo_t.A2) */
  int m, k1;
  hx_mat w;
  int epi;                      /* HX_EPI_* */
  void* out; int ldo;           /* fp16 output */
  float* x; int ldx;            /* fp32 residual (HX_EPI_RESID) */
  const float* gate;            /* [n] (+ image * vec_bstride) */
  long vec_bstride; int rows_per_img;
  const float* gain0; const float* gain1;   /* HX_EPI_RMS: per-head gains [128] */
  int seg1, seg2, rope0, rope1;
  const float* cos_t; const float* sin_t;   /* [rows_per_img][64] */
  float eps;
  int tile;                     /* 0 auto, 1 single-CTA 128x256, 2 CTA-pair 256x256, 3 q8 weights in TMEM,
                                   4 quantised weights expanded to fp16 in the handle's scratch first (auto
                                   does so from 3072 rows up; HX_EXPAND_ROWS in the environment overrides),
                                   5 CTA-pair 256x224 (HX_EPI_GELU or HX_EPI_STORE, fp16 or q8 weights;
                                   auto picks it for GELU when it needs fewer waves, HX_PAIR_TN=256 / 224
                                   overrides) */
} hx_gemm_desc;
#define HX_EPI_STORE 0
#define HX_EPI_RESID 1
#define HX_EPI_GELU 2
#define HX_EPI_RMS 3
#define HX_EPI_SITU 5
#define HX_EPI_STORE32 6   /* fp32 output written to x / ldx */
/* O = A W^T with a fused epilogue: gemm_run_geo (hexagon/mega/gemm2.c:96-137, moss gemm2.c:145-193). */
HX_API int hx_gemm(hx_handle h, const hx_gemm_desc* d);

/* What hx_gemm runs for a descriptor on a GPU with sm_count SMs, decided on the host alone (no handle,
 * no device work; pointers are only checked for presence and alignment). The handle's expansion scratch
 * is assumed present, as hx_gemm reserves it. HX_OK, or HX_E_ARG when hx_gemm would reject d. */
typedef struct {
  int kernel;     /* 1 single-CTA tiles, 2 CTA pairs (cta_group::2), 3 q8 weights dequantised into TMEM */
  int expand;     /* 1: quantised weights expanded to fp16 first; the fields below describe the fp16 GEMM */
  int tile_m, tile_n;  /* output tile of a CTA (kernel 1) or of a CTA pair / TMEM-weight pair (2, 3) */
  int tiles;      /* tiles of the launch */
  int streamk;    /* 1: the last partial wave of CTA-pair tiles is cut into stream-K shares */
} hx_gemm_plan;
HX_API int hx_gemm_query(const hx_gemm_desc* d, int sm_count, hx_gemm_plan* out);

typedef struct {
  const void* q; int ldq, q_col0;
  const void* k; int ldk, k_col0;
  const void* v; int ldv, v_col0;
  void* o; int ldo;
  int batch, heads, tq, tk, nvalid;
  float scale;
  int kernel;                   /* 0 auto, 1 the general kernel (online softmax over 128-key tiles), 2 the
                                   short-key kernel (tk <= 256: K and V resident, one exact softmax step;
                                   auto takes it for 128 < tk <= 256 with at most six 128-query tiles per
                                   SM; HX_ATTN_SHORT=0 / 1: never / always) */
} hx_attn_desc;
/* softmax(q k^T * scale) v per head, head_dim 128: attn_run (hexagon/mega/blk.c:54-91,
 * masked moss/hexagon/mega/blk.c:54-94). Keys >= nvalid are masked (0 = none). */
HX_API int hx_attention(hx_handle h, const hx_attn_desc* d);
/* The kernel hx_attention runs for d on a GPU with sm_count SMs (host-side): *kernel = 1 general, 2
 * short-key. HX_OK, or HX_E_ARG when hx_attention would reject d. */
HX_API int hx_attention_query(const hx_attn_desc* d, int sm_count, int32_t* kernel);

/* k_lnmod_s (hexagon/mega/kern.c:31-65): h16 = LN(x) * (1 + scale) + shift, eps 1e-6 by convention. */
HX_API int hx_lnmod(hx_handle h, const float* x, void* h16, int rows, int D, const float* shift, const float* scale,
             long vec_bstride, int rows_per_img, float eps);
/* k_rmsmod_s (moss/hexagon/mega/kern.c:345-375): h16 = x rsqrt(mean x^2 + eps) w (1 + scale) + shift. */
HX_API int hx_rmsmod(hx_handle h, const float* x, void* h16, int rows, int D, const float* w, const float* shift,
              const float* scale, long vec_bstride, int rows_per_img, float eps);

/* Host-side RoPE tables [ntok][64] (angle index d of the 64 split-half pairs (d, d+64)).
 * Anima 3D split t/h/w = 22/21/21 angles, theta for h and w (make_rope, hexagon/mega/megarun.cpp:77-90);
 * theta 10000 reproduces megarun. Rows >= gh*gw are zero. */
HX_API int hx_rope_anima(int gh, int gw, double theta, int ntok, float* cos_out, float* sin_out);
/* MOSS 4D rope (rope_tables, moss/mossrun/mossrun.cpp:190-202; moss/moss_ref.py:27-35):
 * image token (y, x): coords (0, T, y-(H-1)/2, x-(W-1)/2); text token i: (0, i, 0, 0);
 * angle d = coord[d/16] * bands[d%16]. Rows >= H*W + T are zero. */
HX_API int hx_rope_moss(int H, int W, int T, const float* bands16, int ntok, float* cos_out, float* sin_out);

/* Library version string. */
HX_API const char* hx_version(void);

#ifdef __cplusplus
}
#endif
#endif /* HXDIT_H */

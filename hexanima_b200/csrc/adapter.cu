// The Anima LLM adapter on the GPU (phone/animad.cpp:179-218 `adapter`): T5 token ids [L] plus the LLM's
// hidden states [S][1024] -> the DiT cross-attention context [512][1024] (rows >= L zero).
//
//   x = embed[ids]
//   6 x { x += o_proj(attn(q, k, v))  with h = RMS(x) * norm_self_attn, q/k/v = h W^T, per-head RMS on
//                                      q and k (gains q_norm / k_norm), 1D split-half RoPE (pairs j, j+32)
//         x += o_proj(attn(...))      with queries from RMS(x) * norm_cross_attn and keys / values from the
//                                      hidden states (keys roped with their own positions 0..S-1)
//         x += W2 GELU(W1 RMS(x) * norm_mlp + b1) + b2 }
//   out = (RMS(x W_out^T + b_out) * norm) * wts[token]
// 16 heads of 64, scale 1/8, RMS eps 1e-6. The projections run through the tcgen05 GEMM (fp16 weights,
// activations rounded to fp16 as its A operand, fp32 results); norms, RoPE, attention and the residual
// stream stay in fp32 as in the reference. Attention is one warp per (query, head) with an online softmax:
// lane l holds dimensions l and l + 32, which is also a RoPE pair, so per-head RMS, RoPE and the q.k
// products need no data exchange beyond warp shuffles. The adapter runs once per prompt.
#include <cmath>
#include <vector>

#include "hx_internal.h"

namespace hx {

namespace {

constexpr int AD = 1024, AH = 16, AHD = 64, AF = 4096, ACTX = 512;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void embed_kernel(const int32_t* __restrict__ ids, const __half* __restrict__ emb, float* __restrict__ x) {
  const int t = blockIdx.x;
  const __half* e = emb + static_cast<size_t>(ids[t]) * AD;
  for (int j = threadIdx.x; j < AD; j += blockDim.x) x[static_cast<size_t>(t) * AD + j] = __half2float(e[j]);
}

// out[r] = in[r] * rsqrt(mean(in[r]^2) + eps) * gain (* row_scale[r]); one warp per row of AD elements
template <typename OutT>
__global__ void rms_rows_kernel(const float* __restrict__ in, int rows, const __half* __restrict__ gain,
                                const float* __restrict__ row_scale, OutT* __restrict__ out) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* v = in + static_cast<size_t>(row) * AD;
  float ss = 0.f;
  for (int j = lane; j < AD; j += 32) ss = fmaf(v[j], v[j], ss);
  ss = warp_sum(ss);
  float k = 1.0f / sqrtf(ss / AD + 1e-6f);
  if (row_scale) k *= row_scale[row];
  for (int j = lane; j < AD; j += 32) {
    const float y = v[j] * k * __half2float(gain[j]);
    if constexpr (sizeof(OutT) == 2) out[static_cast<size_t>(row) * AD + j] = __float2half_rn(y);
    else out[static_cast<size_t>(row) * AD + j] = y;
  }
}

// per (token, head): RMS over the 64 dims with gain, then RoPE on pairs (j, j + 32) with the token's angles
__global__ void head_rms_rope_kernel(float* __restrict__ t, int n, const __half* __restrict__ gain,
                                     const float* __restrict__ cosT, const float* __restrict__ sinT) {
  const int w = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (w >= n * AH) return;
  const int tok = w / AH;
  float* v = t + static_cast<size_t>(w) * AHD;
  const float a = v[lane], b = v[lane + 32];
  const float k = 1.0f / sqrtf(warp_sum(a * a + b * b) / AHD + 1e-6f);
  const float an = a * k * __half2float(gain[lane]), bn = b * k * __half2float(gain[lane + 32]);
  const float c = cosT[static_cast<size_t>(tok) * 32 + lane], s = sinT[static_cast<size_t>(tok) * 32 + lane];
  v[lane] = an * c - bn * s;
  v[lane + 32] = an * s + bn * c;
}

// o[t][h] = softmax_s(q[t][h] . k[s][h] / 8) v[s][h]; one warp per (t, h), online softmax over the keys
__global__ void attn64_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                              int L, int S, float* __restrict__ o) {
  const int w = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (w >= L * AH) return;
  const int t = w / AH, h = w % AH;
  const float* qq = q + static_cast<size_t>(t) * AD + h * AHD;
  const float q0 = qq[lane], q1 = qq[lane + 32];
  float m = -INFINITY, l = 0.f, a0 = 0.f, a1 = 0.f;
  for (int s = 0; s < S; ++s) {
    const float* kk = k + static_cast<size_t>(s) * AD + h * AHD;
    const float sc = warp_sum(q0 * kk[lane] + q1 * kk[lane + 32]) * 0.125f;
    const float mn = fmaxf(m, sc);
    const float corr = expf(m - mn), p = expf(sc - mn);
    const float* vv = v + static_cast<size_t>(s) * AD + h * AHD;
    l = l * corr + p;
    a0 = a0 * corr + p * vv[lane];
    a1 = a1 * corr + p * vv[lane + 32];
    m = mn;
  }
  float* oo = o + static_cast<size_t>(t) * AD + h * AHD;
  oo[lane] = a0 / l;
  oo[lane + 32] = a1 / l;
}

__global__ void to_f16_kernel(const float* __restrict__ in, __half* __restrict__ out, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += static_cast<size_t>(gridDim.x) * blockDim.x)
    out[i] = __float2half_rn(in[i]);
}

// x[r][j] += y[r][j] (+ bias[j])
__global__ void add_kernel(float* __restrict__ x, const float* __restrict__ y, const __half* __restrict__ bias,
                           size_t n, int dim) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += static_cast<size_t>(gridDim.x) * blockDim.x)
    x[i] += y[i] + (bias ? __half2float(bias[i % dim]) : 0.f);
}

// out = fp16(gelu_erf(m + bias))
__global__ void bias_gelu_kernel(const float* __restrict__ m, const __half* __restrict__ bias, __half* __restrict__ out,
                                 size_t n, int dim) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float v = m[i] + __half2float(bias[i % dim]);
    out[i] = __float2half_rn(0.5f * v * (1.0f + erff(v * 0.70710678118654752f)));
  }
}

}  // namespace

cudaError_t adapter_run(const AdapterWeights& W, const float* hidden, int S, const int32_t* ids_host,
                        const float* wts_host, int L, float* out, int* status, cudaStream_t s) {
  if (!hidden || !ids_host || !wts_host || !out || L < 1 || L > ACTX || S < 1 || S > 65536) return cudaErrorInvalidValue;
  for (int i = 0; i < L; ++i)
    if (ids_host[i] < 0 || ids_host[i] >= W.vocab) return cudaErrorInvalidValue;
  const int P = L > S ? L : S;  // rows of the RoPE tables and of k / v
  // RoPE tables (animad.cpp:130-137 rope1d): angle i / 10000^(2j/64) in double, stored as fp32
  std::vector<float> hc(static_cast<size_t>(P) * 32), hs(hc.size());
  for (int i = 0; i < P; ++i)
    for (int j = 0; j < 32; ++j) {
      const double a = i / std::pow(10000.0, (2.0 * j) / 64.0);
      hc[static_cast<size_t>(i) * 32 + j] = static_cast<float>(std::cos(a));
      hs[static_cast<size_t>(i) * 32 + j] = static_cast<float>(std::sin(a));
    }
  char* base = nullptr;
  const size_t nL = static_cast<size_t>(L) * AD, nP = static_cast<size_t>(P) * AD;
  // x, q, o, r [L][AD] fp32; k, v [P][AD] fp32; m1 [L][AF] fp32; h16 [L][AF] fp16 (also [L][AD]); hid16 [S][AD];
  // cos, sin [P][32]; ids [L] int32; wts [L] fp32
  const size_t bytes = (4 * nL + 2 * nP + static_cast<size_t>(L) * AF) * 4 + static_cast<size_t>(L) * AF * 2 +
                       static_cast<size_t>(S) * AD * 2 + 2 * hc.size() * 4 + static_cast<size_t>(L) * 8 + 16 * 256;  // + alignment
  cudaError_t e = cudaMalloc(&base, bytes);
  if (e != cudaSuccess) return e;
  size_t off = 0;
  auto take = [&](size_t n) {
    void* p = base + off;
    off += (n + 255) & ~size_t(255);
    return p;
  };
  float* x = static_cast<float*>(take(nL * 4));
  float* q = static_cast<float*>(take(nL * 4));
  float* o = static_cast<float*>(take(nL * 4));
  float* r = static_cast<float*>(take(nL * 4));
  float* k = static_cast<float*>(take(nP * 4));
  float* v = static_cast<float*>(take(nP * 4));
  float* m1 = static_cast<float*>(take(static_cast<size_t>(L) * AF * 4));
  __half* h16 = static_cast<__half*>(take(static_cast<size_t>(L) * AF * 2));
  __half* hid16 = static_cast<__half*>(take(static_cast<size_t>(S) * AD * 2));
  float* cosT = static_cast<float*>(take(hc.size() * 4));
  float* sinT = static_cast<float*>(take(hs.size() * 4));
  int32_t* ids = static_cast<int32_t*>(take(static_cast<size_t>(L) * 4));
  float* wts = static_cast<float*>(take(static_cast<size_t>(L) * 4));
  auto done = [&](cudaError_t x) {
    const cudaError_t y = cudaStreamSynchronize(s);
    cudaFree(base);
    return x != cudaSuccess ? x : y;
  };
  if ((e = cudaMemcpyAsync(cosT, hc.data(), hc.size() * 4, cudaMemcpyHostToDevice, s)) != cudaSuccess ||
      (e = cudaMemcpyAsync(sinT, hs.data(), hs.size() * 4, cudaMemcpyHostToDevice, s)) != cudaSuccess ||
      (e = cudaMemcpyAsync(ids, ids_host, static_cast<size_t>(L) * 4, cudaMemcpyHostToDevice, s)) != cudaSuccess ||
      (e = cudaMemcpyAsync(wts, wts_host, static_cast<size_t>(L) * 4, cudaMemcpyHostToDevice, s)) != cudaSuccess)
    return done(e);

  auto gemm = [&](const __half* A, int M, int K, const __half* Wt, int N, float* y) {
    DevMat dm;
    dm.fmt = WF_F16;
    dm.N = N;
    dm.K = K;
    dm.group = 64;
    dm.w = const_cast<__half*>(Wt);
    GemmArgs a;
    a.A = A;
    a.lda = K;
    a.M = M;
    a.K1 = K;
    a.W = &dm;
    a.epi = EPI_STORE32;
    a.x = y;
    a.ldx = N;
    a.status = status;
    return gemm_launch(a, s);
  };
  const int ew = 148 * 8;  // grid of the elementwise loops
  auto rms16 = [&](const float* in, int rows, const __half* g, __half* y) {
    rms_rows_kernel<__half><<<(rows + 7) / 8, 256, 0, s>>>(in, rows, g, nullptr, y);
  };
  auto heads = [&](float* t, int n, const __half* g) {
    head_rms_rope_kernel<<<(n * AH + 7) / 8, 256, 0, s>>>(t, n, g, cosT, sinT);
  };

  embed_kernel<<<L, 256, 0, s>>>(ids, W.embed, x);
  to_f16_kernel<<<ew, 256, 0, s>>>(hidden, hid16, static_cast<size_t>(S) * AD);
  for (int b = 0; b < 6 && e == cudaSuccess; ++b) {
    const AdapterWeights::Block& B = W.blocks[b];
    // self-attention
    rms16(x, L, B.norm_sa, h16);
    if ((e = gemm(h16, L, AD, B.sa_q, AD, q)) != cudaSuccess || (e = gemm(h16, L, AD, B.sa_k, AD, k)) != cudaSuccess ||
        (e = gemm(h16, L, AD, B.sa_v, AD, v)) != cudaSuccess)
      break;
    heads(q, L, B.sa_qn);
    heads(k, L, B.sa_kn);
    attn64_kernel<<<(L * AH + 7) / 8, 256, 0, s>>>(q, k, v, L, L, o);
    to_f16_kernel<<<ew, 256, 0, s>>>(o, h16, nL);
    if ((e = gemm(h16, L, AD, B.sa_o, AD, r)) != cudaSuccess) break;
    add_kernel<<<ew, 256, 0, s>>>(x, r, nullptr, nL, AD);
    // cross-attention to the hidden states
    rms16(x, L, B.norm_ca, h16);
    if ((e = gemm(h16, L, AD, B.ca_q, AD, q)) != cudaSuccess || (e = gemm(hid16, S, AD, B.ca_k, AD, k)) != cudaSuccess ||
        (e = gemm(hid16, S, AD, B.ca_v, AD, v)) != cudaSuccess)
      break;
    heads(q, L, B.ca_qn);
    heads(k, S, B.ca_kn);
    attn64_kernel<<<(L * AH + 7) / 8, 256, 0, s>>>(q, k, v, L, S, o);
    to_f16_kernel<<<ew, 256, 0, s>>>(o, h16, nL);
    if ((e = gemm(h16, L, AD, B.ca_o, AD, r)) != cudaSuccess) break;
    add_kernel<<<ew, 256, 0, s>>>(x, r, nullptr, nL, AD);
    // MLP
    rms16(x, L, B.norm_mlp, h16);
    if ((e = gemm(h16, L, AD, B.mlp0_w, AF, m1)) != cudaSuccess) break;
    bias_gelu_kernel<<<ew, 256, 0, s>>>(m1, B.mlp0_b, h16, static_cast<size_t>(L) * AF, AF);
    if ((e = gemm(h16, L, AF, B.mlp2_w, AD, r)) != cudaSuccess) break;
    add_kernel<<<ew, 256, 0, s>>>(x, r, B.mlp2_b, nL, AD);
  }
  if (e != cudaSuccess) return done(e);
  // out_proj + bias, RMS with the final gain, per-token weight; rows >= L zero
  to_f16_kernel<<<ew, 256, 0, s>>>(x, h16, nL);
  if ((e = gemm(h16, L, AD, W.out_w, AD, r)) != cudaSuccess) return done(e);
  cudaMemsetAsync(q, 0, nL * 4, s);
  add_kernel<<<ew, 256, 0, s>>>(q, r, W.out_b, nL, AD);  // q = r + b_out
  cudaMemsetAsync(out, 0, static_cast<size_t>(ACTX) * AD * 4, s);
  rms_rows_kernel<float><<<(L + 7) / 8, 256, 0, s>>>(q, L, W.norm, wts, out);
  return done(cudaGetLastError());
}

}  // namespace hx

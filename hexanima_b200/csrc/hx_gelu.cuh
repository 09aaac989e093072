// GELU with the exact-erf definition for the GEMM epilogues, two elements at a time.
//
// gelu(x) = x Phi(x) = max(x, 0) - t(|x|),  t(a) = (a / 2) erfc(a / sqrt 2) = a e^{-a^2/2} R(a),
// the same split as the reference's table GELU (hexagon/mega/kern.c `k_gelu2`: max(x, 0) minus a
// tabulated a Phi(-a)). R(a) = erfcx(a / sqrt 2) / 2 is smooth and bounded on [0, 6]; it is replaced by
// a degree-9 polynomial fitted for this kernel (least squares in a Chebyshev basis, reweighted towards
// minimax of the relative error): 4.1e-5 relative on [0, 4.3], where fp16 results are normal, looser
// above where t falls below fp16's normal range. |x| is clamped at 6, where t < 1e-8 (under half the
// smallest fp16 subnormal). The polynomial, exponent argument and products run on the packed f32x2
// pipe, e^{-a^2/2} on MUFU ex2 (one per element). Rounded to fp16, 1 % of inputs differ from the exact
// GELU by one ulp and none by more.
#pragma once
#include <cstdint>

namespace hx {
namespace gelu_detail {

__device__ __forceinline__ uint64_t pk(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void upk(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace gelu_detail

__device__ __forceinline__ void gelu_pair(float& x0, float& x1) {
  using namespace gelu_detail;
  constexpr float c[10] = {4.999796152e-01f, -3.982473016e-01f, 2.457687557e-01f, -1.223157272e-01f,
                           4.786257446e-02f, -1.397187542e-02f, 2.864922862e-03f, -3.837234108e-04f,
                           2.985421270e-05f, -1.017048476e-06f};
  const uint64_t a = pk(fminf(fabsf(x0), 6.f), fminf(fabsf(x1), 6.f));
  uint64_t p = pk(c[9], c[9]);
#pragma unroll
  for (int i = 8; i >= 0; --i) p = fma2(p, a, pk(c[i], c[i]));
  // e^{-a^2/2} = 2^{-a^2 log2(e) / 2}
  float k0, k1;
  upk(fma2(a, fma2(a, pk(-0.7213475204f, -0.7213475204f), 0ull), 0ull), k0, k1);
  const uint64_t t = fma2(fma2(a, pk(ex2f(k0), ex2f(k1)), 0ull), p, 0ull);
  float t0, t1;
  upk(t, t0, t1);
  x0 = fmaxf(x0, 0.f) - t0;
  x1 = fmaxf(x1, 0.f) - t1;
}

// v[i] = gelu(v[i]) for 32 values
__device__ __forceinline__ void gelu32(float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 32; i += 2) gelu_pair(v[i], v[i + 1]);
}

}  // namespace hx

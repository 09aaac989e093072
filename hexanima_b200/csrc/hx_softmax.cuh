// Softmax arithmetic shared by the attention kernels: MUFU and FMA-pipe 2^x, packed f32x2 operations,
// 32-key max / exp chunks over rows of S loaded from TMEM, and the warp-uniform bounded wait.
#pragma once
#include <cstdint>

#include "hx_ptx.cuh"

namespace hx {
namespace smx {


// one MUFU op: 2^x (flush-to-zero; the inputs here are <= 0 and the results feed fp16 probabilities)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
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

__device__ __forceinline__ uint64_t fadd2_rm(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rm.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// 2^x for a pair, on the FMA and integer pipes instead of MUFU (relieves the MUFU pipe, which two
// softmax warps share per SMSP). x = n + f with n = floor(x): adding 1.5*2^23 rounded toward -inf
// leaves n in the low mantissa bits of the sum, subtracting it back gives n exactly and f = x - n is
// exact. 2^f on [0, 1) is the cubic 1 + c1 f + c2 f^2 + c3 f^3 fitted for this kernel by linear-
// programming minimax of the relative error (8.6e-5 in fp32 Horner evaluation; an fp16 half-ulp is
// 4.9e-4). 2^n is added into the exponent field: the sum's bit pattern is 0x4B400000 + n, and shifted
// left by 23 it is n << 23 (mod 2^32). Inputs are clamped at -127; results below 2^-126 are far
// under the fp16 range of P anyway.
constexpr float kRoundFloor = 12582912.0f;  // 1.5 * 2^23
constexpr float kExp2C1 = 0.695116639f, kExp2C2 = 0.22764498f, kExp2C3 = 0.0770672411f;
__device__ __forceinline__ void ex2_poly2(uint64_t x2, float& e0, float& e1) {
  float x0, x1;
  f2unpack(x2, x0, x1);
  const uint64_t xc = f2pack(fmaxf(x0, -127.f), fmaxf(x1, -127.f));
  const uint64_t t = fadd2_rm(xc, f2pack(kRoundFloor, kRoundFloor));
  const uint64_t n = fadd2(t, f2pack(-kRoundFloor, -kRoundFloor));
  const uint64_t fr = ffma2(n, f2pack(-1.f, -1.f), xc);
  uint64_t q = ffma2(fr, f2pack(kExp2C3, kExp2C3), f2pack(kExp2C2, kExp2C2));
  q = ffma2(q, fr, f2pack(kExp2C1, kExp2C1));
  q = ffma2(q, fr, f2pack(1.f, 1.f));
  float q0, q1, t0, t1;
  f2unpack(q, q0, q1);
  f2unpack(t, t0, t1);
  e0 = __uint_as_float(__float_as_uint(q0) + (__float_as_uint(t0) << 23));
  e1 = __uint_as_float(__float_as_uint(q1) + (__float_as_uint(t1) << 23));
}

// which fp16 pairs of a 32-key chunk take ex2_poly2 instead of MUFU: pair index pi with
// (pi & kPolyMask) == kPolyMask (kPolyMask 3: one pair in four)
constexpr int kPolyMask = 3;

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

// p = 2^(s*scale_log2 - m) for 32 scores, fp16-packed into pk, pairwise partial sums into sum2; the pairs
// pi with (pi & POLY) == POLY take ex2_poly2
template <bool FULL, int POLY = kPolyMask>
__device__ __forceinline__ void exp32(uint32_t (&pk)[16], uint64_t (&sum2)[4], const uint32_t (&r)[32],
                                      uint64_t scale2, uint64_t negm2, int kbase, int limit) {
#pragma unroll
  for (int t = 0; t < 32; t += 2) {
    const uint64_t x2 = ffma2(f2pack(__uint_as_float(r[t]), __uint_as_float(r[t + 1])), scale2, negm2);
    float e0, e1;
    if (((t >> 1) & POLY) == POLY) {
      ex2_poly2(x2, e0, e1);
    } else {
      float x0, x1;
      f2unpack(x2, x0, x1);
      e0 = ex2(x0);
      e1 = ex2(x1);
    }
    if constexpr (!FULL) {
      if (kbase + t >= limit) e0 = 0.f;
      if (kbase + t + 1 >= limit) e1 = 0.f;
    }
    sum2[(t >> 1) & 3] = fadd2(sum2[(t >> 1) & 3], f2pack(e0, e1));
    pk[t / 2] = pack_half2(e0, e1);
  }
}

// the same exps, kept: r[t] becomes p as fp32 (for the row sum, taken after P is published); no sums here
template <bool FULL>
__device__ __forceinline__ void exp32_keep(uint32_t (&pk)[16], uint32_t (&r)[32], uint64_t scale2, uint64_t negm2,
                                           int kbase, int limit) {
#pragma unroll
  for (int t = 0; t < 32; t += 2) {
    const uint64_t x2 = ffma2(f2pack(__uint_as_float(r[t]), __uint_as_float(r[t + 1])), scale2, negm2);
    float e0, e1;
    if (((t >> 1) & kPolyMask) == kPolyMask) {
      ex2_poly2(x2, e0, e1);
    } else {
      float x0, x1;
      f2unpack(x2, x0, x1);
      e0 = ex2(x0);
      e1 = ex2(x1);
    }
    if constexpr (!FULL) {
      if (kbase + t >= limit) e0 = 0.f;
      if (kbase + t + 1 >= limit) e1 = 0.f;
    }
    r[t] = __float_as_uint(e0);
    r[t + 1] = __float_as_uint(e1);
    pk[t / 2] = pack_half2(e0, e1);
  }
}

// bounded wait whose result is the same in every lane, so the warp-collective tcgen05.ld / st that
// follow are reached by all lanes or by none
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, status, code));
}

}  // namespace smx
}  // namespace hx

// Base-2 exponentials for the softmax of the flash-attention kernels
// (attention_mma.cu, attention_tc.cu): a polynomial form on the FMA pipe and
// the SFU instruction, so a kernel can split its exponentials between the two
// pipes.
#pragma once

#include "common.cuh"

namespace c3b {

// 2^x for x <= 8 on the FMA/ALU pipes: Cody-Waite split x = n + f with
// f in [-0.5, 0.5] (round-to-nearest through the 1.5*2^23 shifter), Taylor
// polynomial of 2^f = e^(f ln 2) to degree 5 (relative error < 4e-6 in fp32
// arithmetic, far below the bf16 rounding the result goes through), and 2^n applied
// by adding n to the exponent field.  The shifter's bit pattern is
// 0x4B400000 + n, and 0x4B400000 * 2^23 wraps to 0 in 32 bits, so that add is
// one integer multiply-add of the shifter's bits.  Inputs are clamped at -126,
// so masked scores (-inf) give 2^-126 instead of 0: at most 64 * 2^-126 of a
// row sum that is at least 1.
__device__ __forceinline__ float exp2_fma(float x) {
  x = fmaxf(x, -126.0f);
  const float shifter = 12582912.0f;  // 1.5 * 2^23
  const float t = x + shifter;
  const float n = t - shifter;
  const float f = x - n;
  float p = 1.3333558146428443e-3f;        // ln2^5 / 5!
  p = fmaf(p, f, 9.6181291076284772e-3f);  // ln2^4 / 4!
  p = fmaf(p, f, 5.5504108664821580e-2f);  // ln2^3 / 3!
  p = fmaf(p, f, 2.4022650695910071e-1f);  // ln2^2 / 2!
  p = fmaf(p, f, 6.9314718055994531e-1f);  // ln2
  p = fmaf(p, f, 1.0f);
  return __int_as_float(__float_as_int(t) * (1 << 23) + __float_as_int(p));
}

// exp2_fma on a pair of values with the packed fp32 pair instructions of
// sm_100 (one FFMA2 / FADD2 does two lanes' worth of the polynomial).
__device__ __forceinline__ float2 exp2_fma2(float2 x) {
  x.x = fmaxf(x.x, -126.0f);
  x.y = fmaxf(x.y, -126.0f);
  const float shifter = 12582912.0f;  // 1.5 * 2^23
  const float2 t = __fadd2_rn(x, make_float2(shifter, shifter));
  const float2 n = __fadd2_rn(t, make_float2(-shifter, -shifter));
  const float2 f = __ffma2_rn(n, make_float2(-1.0f, -1.0f), x);
  float2 p = __ffma2_rn(make_float2(1.3333558146428443e-3f, 1.3333558146428443e-3f), f,
                        make_float2(9.6181291076284772e-3f, 9.6181291076284772e-3f));
  p = __ffma2_rn(p, f, make_float2(5.5504108664821580e-2f, 5.5504108664821580e-2f));
  p = __ffma2_rn(p, f, make_float2(2.4022650695910071e-1f, 2.4022650695910071e-1f));
  p = __ffma2_rn(p, f, make_float2(6.9314718055994531e-1f, 6.9314718055994531e-1f));
  p = __ffma2_rn(p, f, make_float2(1.0f, 1.0f));
  return make_float2(__int_as_float(__float_as_int(t.x) * (1 << 23) + __float_as_int(p.x)),
                     __int_as_float(__float_as_int(t.y) * (1 << 23) + __float_as_int(p.y)));
}

// exp2_fma2 with a degree-3 polynomial for 2^f on [-0.5, 0.5]: a
// relative-error fit computed for this kernel (iteratively reweighted least
// squares on 20001 points; max relative error 7.5e-5 in fp32 Horner form).
// Enough for a probability that is rounded to bf16 next (2^-9 relative), and
// two fused multiply-adds shorter than the degree-5 form.
__device__ __forceinline__ float2 exp2_fma2_p3(float2 x) {
  x.x = fmaxf(x.x, -126.0f);
  x.y = fmaxf(x.y, -126.0f);
  const float shifter = 12582912.0f;  // 1.5 * 2^23
  const float2 t = __fadd2_rn(x, make_float2(shifter, shifter));
  const float2 n = __fadd2_rn(t, make_float2(-shifter, -shifter));
  const float2 f = __ffma2_rn(n, make_float2(-1.0f, -1.0f), x);
  float2 p = __ffma2_rn(make_float2(0.05517132143403903f, 0.05517132143403903f), f,
                        make_float2(0.24261054228171514f, 0.24261054228171514f));
  p = __ffma2_rn(p, f, make_float2(0.6932609856052563f, 0.6932609856052563f));
  p = __ffma2_rn(p, f, make_float2(0.9999281093641528f, 0.9999281093641528f));
  return make_float2(__int_as_float(__float_as_int(t.x) * (1 << 23) + __float_as_int(p.x)),
                     __int_as_float(__float_as_int(t.y) * (1 << 23) + __float_as_int(p.y)));
}

// Three-input maximum (one sm_100 instruction).
__device__ __forceinline__ float fmax3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x on the SFU (ex2.approx, flush-to-zero); 2^-inf = 0.
__device__ __forceinline__ float exp2_sfu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace c3b

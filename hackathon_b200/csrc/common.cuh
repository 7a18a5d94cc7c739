// Shared helpers for the c3b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string>

#include "c3b200.h"

namespace c3b {

// Thread-local last error (c3b_last_error).
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);

#define C3B_CHECK_CUDA(expr)                                                    \
  do {                                                                          \
    cudaError_t _e = (expr);                                                    \
    if (_e != cudaSuccess)                                                      \
      return ::c3b::fail(C3B_E_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e)); \
  } while (0)

#define C3B_REQUIRE(cond, msg)                                                  \
  do {                                                                          \
    if (!(cond)) return ::c3b::fail(C3B_E_INVALID, msg);                        \
  } while (0)

inline int64_t numel(const c3b_tensor& t) {
  int64_t n = 1;
  for (int i = 0; i < t.ndim; ++i) n *= t.shape[i];
  return n;
}

inline size_t dtype_size(int dt) {
  switch (dt) {
    case C3B_F32: case C3B_I32: return 4;
    case C3B_BF16: case C3B_F16: return 2;
    case C3B_I64: return 8;
    case C3B_U8: return 1;
  }
  return 0;
}

// Device-side status word: set by kernels whose bounded waits expire.
extern __device__ int g_status;
// Limit of one bounded device wait in ns (2 s unless c3b_set_wait_limit_ns
// changed it; tests shorten it to make a wait expire on purpose).
extern __device__ unsigned long long g_wait_limit_ns;

__device__ __forceinline__ float load_as_f32(const void* p, int dt, int64_t i) {
  switch (dt) {
    case C3B_F32: return static_cast<const float*>(p)[i];
    case C3B_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    case C3B_F16: return __half2float(static_cast<const __half*>(p)[i]);
    case C3B_I64: return (float)static_cast<const long long*>(p)[i];
    case C3B_I32: return (float)static_cast<const int*>(p)[i];
    default: return static_cast<const unsigned char*>(p)[i];
  }
}

__device__ __forceinline__ void store_from_f32(void* p, int dt, int64_t i, float v) {
  switch (dt) {
    case C3B_F32: static_cast<float*>(p)[i] = v; break;
    case C3B_BF16: static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v); break;
    case C3B_F16: static_cast<__half*>(p)[i] = __float2half_rn(v); break;
    case C3B_I64: static_cast<long long*>(p)[i] = (long long)v; break;
    case C3B_I32: static_cast<int*>(p)[i] = (int)v; break;
    default: static_cast<unsigned char*>(p)[i] = (unsigned char)v; break;
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Exact-erf GELU, the 5-op chain x * 0.5 * (1 + erf(x / sqrt(2))).
__device__ __forceinline__ float gelu_erf(float x) {
  return (x * (1.0f + erff(x * 0.70710678118654752f))) * 0.5f;
}

__device__ __forceinline__ float apply_act(float v, int act) {
  if (act == C3B_ACT_RELU) return fmaxf(v, 0.0f);
  if (act == C3B_ACT_GELU) return gelu_erf(v);
  return v;
}

// GELU for bf16 outputs: erf from the Abramowitz & Stegun 7.1.26 rational
// approximation (|error| < 1.5e-7, the same formula the reference's unfused Erf
// uses) with the fast reciprocal and exponential — two SFU operations and a
// handful of FMAs per element instead of the full-precision erff, whose cost
// made the FFN1 epilogue slower than its MMAs.  The result is rounded to bf16.
// Written without a sign select: x Phi(x) = 0.5 x + |x| (0.5 - q) with
// q = Phi(-|x|) = 0.5 erfc(|x| / sqrt 2), and erfc(z) = t P(t) exp(-z^2),
// t = 1 / (1 + p z), from Abramowitz & Stegun 7.1.26 (|error| <= 1.5e-7).  The
// polynomial coefficients below are A&S's, multiplied by -0.5 (so the
// polynomial yields -q / exp(-z^2)), and p is divided by sqrt 2 (so t takes |x|);
// exp(-x^2 / 2) is one ex2.approx of -x^2 log2(e) / 2, 1/d one rcp.approx.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float gelu_as_fast(float x) {
  const float ax = fabsf(x);
  const float t = rcp_approx(fmaf(0.23164188826636040f, ax, 1.0f));
  float p = fmaf(t, -0.5307027145f, 0.7265760135f);
  p = fmaf(t, p, -0.7107068705f);
  p = fmaf(t, p, 0.142248368f);
  p = fmaf(t, p, -0.127414796f);
  p *= t;                                                  // -q / exp(-x^2/2)
  const float e = ex2_approx(x * x * -0.72134752044448170f);  // exp(-x^2 / 2)
  return fmaf(ax, fmaf(p, e, 0.5f), 0.5f * x);
}

// Two-wide GELU for 16-bit outputs: the same evaluation with the multiply-adds
// issued as Blackwell's packed fp32 pairs (__ffma2_rn / __fmul2_rn), which
// halves the FMA-pipe instructions of the epilogues that run it on every
// output element.
__device__ __forceinline__ float2 gelu2_as_fast(float2 x) {
  const float2 ax = make_float2(fabsf(x.x), fabsf(x.y));
  const float2 d = __ffma2_rn(make_float2(0.23164188826636040f, 0.23164188826636040f), ax, make_float2(1.0f, 1.0f));
  const float2 t = make_float2(rcp_approx(d.x), rcp_approx(d.y));
  float2 p = __ffma2_rn(t, make_float2(-0.5307027145f, -0.5307027145f), make_float2(0.7265760135f, 0.7265760135f));
  p = __ffma2_rn(t, p, make_float2(-0.7107068705f, -0.7107068705f));
  p = __ffma2_rn(t, p, make_float2(0.142248368f, 0.142248368f));
  p = __ffma2_rn(t, p, make_float2(-0.127414796f, -0.127414796f));
  p = __fmul2_rn(t, p);
  const float2 w = __fmul2_rn(__fmul2_rn(x, x), make_float2(-0.72134752044448170f, -0.72134752044448170f));
  const float2 e = make_float2(ex2_approx(w.x), ex2_approx(w.y));
  const float2 r = __ffma2_rn(p, e, make_float2(0.5f, 0.5f));  // 0.5 - q
  return __ffma2_rn(ax, r, __fmul2_rn(x, make_float2(0.5f, 0.5f)));
}

// Activation over a register array, chosen once per call (a warp-uniform
// branch): a per-element select lets the compiler evaluate every variant,
// erff included, for every element — which cost the tcgen05 GEMM epilogues a
// third of their throughput.  bf16 outputs take the fast GELU.
// 16-bit storage formats of the tensor-core paths: bf16 (bf16 profile) or
// fp16 (fp16 profile), selected per launch by `h16` (1 = fp16).
__device__ __forceinline__ float2 unpack2h(uint32_t w, bool h16) {
  if (h16) return __half22float2(*reinterpret_cast<const __half2*>(&w));
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}
__device__ __forceinline__ uint32_t pack2h(float2 v, bool h16) {
  uint32_t r;
  if (h16) {
    __half2 t = __float22half2_rn(v);
    r = *reinterpret_cast<uint32_t*>(&t);
  } else {
    __nv_bfloat162 t = __float22bfloat162_rn(v);
    r = *reinterpret_cast<uint32_t*>(&t);
  }
  return r;
}
// 8 consecutive 16-bit elements (one 16-byte word) <-> floats
__device__ __forceinline__ void unpack8h(const uint4& w, float* v, bool h16) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack2h(u[i], h16);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ uint4 pack8h(const float* v, bool h16) {
  uint4 w;
  w.x = pack2h(make_float2(v[0], v[1]), h16);
  w.y = pack2h(make_float2(v[2], v[3]), h16);
  w.z = pack2h(make_float2(v[4], v[5]), h16);
  w.w = pack2h(make_float2(v[6], v[7]), h16);
  return w;
}

template <int N>
__device__ __forceinline__ void act_inplace(float* v, int act, bool bf16_out) {
  if (act == C3B_ACT_RELU) {
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = fmaxf(v[i], 0.0f);
  } else if (act == C3B_ACT_GELU) {
    if (bf16_out) {
#pragma unroll
      for (int i = 0; i + 1 < N; i += 2) {
        const float2 g = gelu2_as_fast(make_float2(v[i], v[i + 1]));
        v[i] = g.x;
        v[i + 1] = g.y;
      }
      if (N & 1) v[N - 1] = gelu_as_fast(v[N - 1]);
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i) v[i] = gelu_erf(v[i]);
    }
  }
}

// ---- kernel entry points implemented in the .cu files (host launchers)
int launch_ew(const c3b_tensor* in, int n_in, const c3b_tensor& out, const c3b_ew_params& p, cudaStream_t s);
int launch_copy(const c3b_tensor& in, const c3b_tensor& out, const c3b_copy_params& p, cudaStream_t s);
int launch_im2col(const c3b_tensor& in, const c3b_tensor& out, const c3b_conv_geom& g, cudaStream_t s);
int launch_reduce(const c3b_tensor& in, const c3b_tensor& out, const c3b_reduce_params& p, cudaStream_t s);
int launch_layernorm(const c3b_tensor* in, int n_in, const c3b_tensor* out, int n_out,
                     const c3b_layernorm_params& p, cudaStream_t s);
int launch_softmax(const c3b_tensor& in, const c3b_tensor& out, const c3b_softmax_params& p, cudaStream_t s);
int launch_attn_scores(const c3b_tensor* in, const c3b_tensor& out, const c3b_attn_scores_params& p, cudaStream_t s);
int launch_gather(const c3b_tensor& data, const c3b_tensor& idx, const c3b_tensor& out,
                  const c3b_gather_params& p, cudaStream_t s);
int launch_embed(const c3b_tensor* in, const c3b_tensor& out, const c3b_embed_params& p, cudaStream_t s);
int launch_stem_im2col(const c3b_tensor& in, const c3b_tensor& out, const c3b_stem_params& p, cudaStream_t s);
int launch_stem_conv(const c3b_tensor* in, int n_in, const c3b_tensor& out, const c3b_stem_conv_params& p,
                     cudaStream_t s);
int launch_gap_nhwc(const c3b_tensor* in, int n_in, const c3b_tensor& out, const c3b_gap_params& p,
                    cudaStream_t s);
int launch_wait_probe(const c3b_wait_probe_params& p, cudaStream_t s);
int launch_gemm_tf32(const c3b_tensor* in, int n_in, const c3b_tensor& out, const c3b_gemm_tc_params& p, cudaStream_t s);
bool flash_tc_supported(const c3b_flash_params& p);
int launch_flash_tc(const c3b_tensor& qkv, const c3b_tensor& out, const c3b_flash_params& p, cudaStream_t s);
int launch_gemm_simt(const c3b_tensor* in, int n_in, const c3b_tensor& out, const c3b_gemm_params& p, cudaStream_t s);
int launch_conv_simt(const c3b_tensor* in, int n_in, const c3b_tensor& out, const c3b_conv_params& p, cudaStream_t s);
int launch_gemm_tc(const c3b_tensor* in, int n_in, const c3b_tensor& out, const c3b_gemm_tc_params& p, cudaStream_t s);
int launch_conv_tc(const c3b_tensor* in, int n_in, const c3b_tensor* outs, const c3b_conv_tc_params& p,
                   cudaStream_t s);
int launch_flash_attn(const c3b_tensor& qkv, const c3b_tensor& out, const c3b_flash_params& p, cudaStream_t s);
int launch_quant_e4m3(const c3b_tensor& x, const c3b_tensor& q, const c3b_tensor& scale, const c3b_quant_params& p,
                      cudaStream_t s);
int launch_gemm_fp8(const c3b_tensor* in, int n_in, const c3b_tensor& out, const c3b_gemm_tc_params& p,
                    cudaStream_t s);
int launch_quant_fp4(const c3b_tensor& x, const c3b_tensor& q, const c3b_tensor& scale, const c3b_quant_params& p,
                     cudaStream_t s);
int launch_dequant_fp4(const c3b_tensor& q, const c3b_tensor& scale, const c3b_tensor& w, const c3b_quant_params& p,
                       cudaStream_t s);
int launch_gemm_w4a16(const c3b_tensor* in, int n_in, const c3b_tensor& out, const c3b_gemm_tc_params& p,
                      cudaStream_t s);

int sm_count();
bool launch_stem_tc(const c3b_tensor* in, const c3b_tensor& out, const c3b_stem_conv_params& p, cudaStream_t s,
                    int* rc);

}  // namespace c3b

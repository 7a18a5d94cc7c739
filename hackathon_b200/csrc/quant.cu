// Rowwise E4M3 quantisation for the fp8 precision path.
//
// One warp per row: pass 1 finds max|x| with 16-byte loads, pass 2 re-reads
// the row (L1/L2-resident by then), divides by scale = amax / 448 and converts
// pairs with the hardware round-to-nearest-even, saturating E4M3 conversion.
// The division is IEEE (x / s), so a host restatement that divides in fp32 and
// rounds to E4M3 gives the same bytes.
#include <cuda_fp4.h>
#include <cuda_fp8.h>

#include "common.cuh"

namespace c3b {

namespace {

constexpr int QWARPS = 8;

template <typename T>
__device__ __forceinline__ void load8(const T* p, float* v);

template <>
__device__ __forceinline__ void load8<float>(const float* p, float* v) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float* v) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(h[i]);
}

template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float* v) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  unpack8h(u, v, true);
}

template <typename T>
__global__ void __launch_bounds__(QWARPS * 32) quant_e4m3_kernel(const T* __restrict__ x, uint8_t* __restrict__ q,
                                                                 float* __restrict__ scale, int64_t M, int64_t K) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * QWARPS + (threadIdx.x >> 5);
  if (row >= M) return;
  const T* xr = x + row * K;
  float amax = 0.f;
  for (int64_t k = (int64_t)lane * 8; k < K; k += 256) {
    float v[8];
    load8<T>(xr + k, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
  }
  amax = warp_max(amax);
  const float s = amax > 0.f ? amax / 448.0f : 1.0f;
  if (lane == 0) scale[row] = s;
  uint8_t* qr = q + row * K;
  for (int64_t k = (int64_t)lane * 8; k < K; k += 256) {
    float v[8];
    load8<T>(xr + k, v);
    __align__(8) __nv_fp8x2_storage_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      o[i] = __nv_cvt_float2_to_fp8x2(make_float2(v[2 * i] / s, v[2 * i + 1] / s), __NV_SATFINITE, __NV_E4M3);
    *reinterpret_cast<uint2*>(qr + k) = *reinterpret_cast<const uint2*>(o);
  }
}

// FP4 (E2M1) weight quantisation for the W4A16 path: one thread per (row,
// 16-element group); scale = max|x| / 6 (1 for an all-zero group), bytes =
// E2M1(x / scale) round-to-nearest-even, saturating, element 2i in the low
// nibble of byte i.  Scales are written [K/64][N][4] (the four groups of one
// row and 64-wide K block together), the layout the W4A16 GEMM loads by TMA.
template <typename T>
__global__ void quant_fp4_kernel(const T* __restrict__ x, uint8_t* __restrict__ q, float* __restrict__ scale,
                                 int64_t N, int64_t K) {
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t groups = K / 16;
  if (gid >= N * groups) return;
  const int64_t n = gid / groups, g = gid % groups;
  const T* xr = x + n * K + g * 16;
  float v[16];
  load8<T>(xr, v);
  load8<T>(xr + 8, v + 8);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const float s = amax > 0.f ? amax / 6.0f : 1.0f;
  scale[((g >> 2) * N + n) * 4 + (g & 3)] = s;
  __align__(8) __nv_fp4x2_storage_t o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    o[i] = __nv_cvt_float2_to_fp4x2(make_float2(v[2 * i] / s, v[2 * i + 1] / s), __NV_E2M1, cudaRoundNearest);
  *reinterpret_cast<uint2*>(q + n * (K / 2) + g * 8) = *reinterpret_cast<const uint2*>(o);
}

// W4A16 weights expanded once: dequant(q, scale) -> bf16 [N, K], with the same
// arithmetic as the GEMM's converter warps (E2M1 pair -> f16x2 -> f32 pair,
// times the group scale, one bf16 rounding), so both paths see identical
// weights.  One thread per (row, 16-element group).
__global__ void dequant_fp4_kernel(const uint8_t* __restrict__ q, const float* __restrict__ scale,
                                   uint16_t* __restrict__ w, int64_t N, int64_t K, int h16) {
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t groups = K / 16;
  if (gid >= N * groups) return;
  const int64_t n = gid / groups, g = gid % groups;
  const uint2 pk = __ldg(reinterpret_cast<const uint2*>(q + n * (K / 2) + g * 8));
  const float sc = __ldg(scale + ((g >> 2) * N + n) * 4 + (g & 3));
  const float2 s2 = make_float2(sc, sc);
  uint32_t o[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t word = j < 4 ? pk.x : pk.y;
    const __half2_raw h = __nv_cvt_fp4x2_to_halfraw2((__nv_fp4x2_storage_t)((word >> (8 * (j & 3))) & 0xFF), __NV_E2M1);
    o[j] = pack2h(__fmul2_rn(__half22float2(*reinterpret_cast<const __half2*>(&h)), s2), h16);
  }
  uint4* dst = reinterpret_cast<uint4*>(w + n * K + g * 16);
  dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
  dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
}

}  // namespace

int launch_dequant_fp4(const c3b_tensor& q, const c3b_tensor& scale, const c3b_tensor& w, const c3b_quant_params& p,
                       cudaStream_t s) {
  C3B_REQUIRE(q.dtype == C3B_U8 && scale.dtype == C3B_F32 && (w.dtype == C3B_BF16 || w.dtype == C3B_F16),
              "dequantize fp4: inputs u8 codes and f32 scales, output bf16 or fp16");
  C3B_REQUIRE(p.M >= 0 && p.K > 0 && p.K % 64 == 0, "dequantize fp4: K must be a positive multiple of 64");
  C3B_REQUIRE(numel(q) >= p.M * p.K / 2 && numel(scale) >= p.M * p.K / 16 && numel(w) >= p.M * p.K,
              "dequantize fp4: extents");
  C3B_REQUIRE(((uintptr_t)q.ptr & 7) == 0 && ((uintptr_t)w.ptr & 15) == 0, "dequantize fp4: alignment");
  const int64_t work = p.M * (p.K / 16);
  if (work == 0) return C3B_OK;
  dequant_fp4_kernel<<<(unsigned)((work + 255) / 256), 256, 0, s>>>((const uint8_t*)q.ptr, (const float*)scale.ptr,
                                                                   (uint16_t*)w.ptr, p.M, p.K,
                                                                   (int)(w.dtype == C3B_F16));
  C3B_CHECK_CUDA(cudaGetLastError());
  return C3B_OK;
}

int launch_quant_fp4(const c3b_tensor& x, const c3b_tensor& q, const c3b_tensor& scale, const c3b_quant_params& p,
                     cudaStream_t s) {
  C3B_REQUIRE(x.dtype == C3B_F32 || x.dtype == C3B_BF16, "quantize fp4: input f32 or bf16");
  C3B_REQUIRE(q.dtype == C3B_U8 && scale.dtype == C3B_F32, "quantize fp4: outputs u8 and f32");
  C3B_REQUIRE(p.M >= 0 && p.K > 0 && p.K % 64 == 0, "quantize fp4: K must be a positive multiple of 64");
  C3B_REQUIRE(numel(x) >= p.M * p.K && numel(q) >= p.M * p.K / 2 && numel(scale) >= p.M * p.K / 16,
              "quantize fp4: extents");
  C3B_REQUIRE(((uintptr_t)x.ptr & 15) == 0 && ((uintptr_t)q.ptr & 7) == 0, "quantize fp4: alignment");
  const int64_t work = p.M * (p.K / 16);
  if (work == 0) return C3B_OK;
  const unsigned blocks = (unsigned)((work + 255) / 256);
  if (x.dtype == C3B_F32)
    quant_fp4_kernel<float><<<blocks, 256, 0, s>>>((const float*)x.ptr, (uint8_t*)q.ptr, (float*)scale.ptr, p.M, p.K);
  else
    quant_fp4_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>((const __nv_bfloat16*)x.ptr, (uint8_t*)q.ptr,
                                                           (float*)scale.ptr, p.M, p.K);
  C3B_CHECK_CUDA(cudaGetLastError());
  return C3B_OK;
}

int launch_quant_e4m3(const c3b_tensor& x, const c3b_tensor& q, const c3b_tensor& scale, const c3b_quant_params& p,
                      cudaStream_t s) {
  C3B_REQUIRE(x.dtype == C3B_F32 || x.dtype == C3B_BF16 || x.dtype == C3B_F16,
              "quantize e4m3: input f32, bf16 or fp16");
  C3B_REQUIRE(q.dtype == C3B_U8 && scale.dtype == C3B_F32, "quantize e4m3: outputs u8 and f32");
  C3B_REQUIRE(p.M >= 0 && p.K > 0 && p.K % 16 == 0, "quantize e4m3: K must be a positive multiple of 16");
  C3B_REQUIRE(numel(x) >= p.M * p.K && numel(q) >= p.M * p.K && numel(scale) >= p.M, "quantize e4m3: extents");
  C3B_REQUIRE(((uintptr_t)x.ptr & 15) == 0 && ((uintptr_t)q.ptr & 7) == 0, "quantize e4m3: alignment");
  if (p.M == 0) return C3B_OK;
  const unsigned blocks = (unsigned)((p.M + QWARPS - 1) / QWARPS);
  if (x.dtype == C3B_F32)
    quant_e4m3_kernel<float><<<blocks, QWARPS * 32, 0, s>>>((const float*)x.ptr, (uint8_t*)q.ptr, (float*)scale.ptr,
                                                            p.M, p.K);
  else if (x.dtype == C3B_F16)
    quant_e4m3_kernel<__half><<<blocks, QWARPS * 32, 0, s>>>((const __half*)x.ptr, (uint8_t*)q.ptr,
                                                             (float*)scale.ptr, p.M, p.K);
  else
    quant_e4m3_kernel<__nv_bfloat16><<<blocks, QWARPS * 32, 0, s>>>((const __nv_bfloat16*)x.ptr, (uint8_t*)q.ptr,
                                                                    (float*)scale.ptr, p.M, p.K);
  C3B_CHECK_CUDA(cudaGetLastError());
  return C3B_OK;
}

}  // namespace c3b

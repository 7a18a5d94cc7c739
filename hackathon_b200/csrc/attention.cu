// Causal flash-style attention on a packed QKV tensor.
//
// Replaces the reference chain split -> reshape/transpose x3 ->
// fused_attention_scores_f32 (which materialises [B,H,S,S] and recomputes each
// dot product three times, c35/engine.py:1250-1380) -> matmul_f32 (P.V, cuBLAS)
// -> fused_transpose_reshape_f32 (c35/engine.py:1383-1445) with one kernel:
// it reads q/k/v straight from the QKV projection output [B,S,3,H,D] and
// writes the merged-head layout [B,S,H*D], keeping scores in registers with an
// online softmax, so the S^2 score tensor never exists.
//
// This file holds the SIMT (FP32-math) version used by the fp32 profile; four
// threads cooperate on one query row (16 of the 64 head dims each).
#include "common.cuh"

namespace c3b {

namespace fa {
constexpr int D = 64;
constexpr int QT = 32;   // queries per block
constexpr int KT = 64;   // keys per tile
constexpr int NT = QT * 4;
}  // namespace fa

template <typename T>
__global__ void __launch_bounds__(fa::NT) flash_simt_kernel(const T* __restrict__ qkv, T* __restrict__ out,
                                                            c3b_flash_params p) {
  using namespace fa;
  __shared__ float Ks[KT][D + 1];
  __shared__ float Vs[KT][D];
  const int qtiles = (p.seq + QT - 1) / QT;
  const int qt = blockIdx.x % qtiles;
  const int h = (blockIdx.x / qtiles) % p.heads;
  const int b = blockIdx.x / (qtiles * p.heads);
  const int tid = threadIdx.x;
  const int qi = tid >> 2, part = tid & 3;
  const int q_row = qt * QT + qi;
  const int64_t tok_stride = (int64_t)3 * p.heads * D;
  const int64_t base = (int64_t)b * p.seq * tok_stride;
  float q[16], o[16];
  const bool valid = q_row < p.seq;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    q[i] = valid ? load_as_f32(qkv, sizeof(T) == 4 ? C3B_F32 : C3B_BF16,
                               base + (int64_t)q_row * tok_stride + (int64_t)h * D + part * 16 + i) * p.scale
                 : 0.f;
    o[i] = 0.f;
  }
  float m_run = -INFINITY, l_run = 0.f;
  const int kv_end = p.causal ? min(p.seq, (qt + 1) * QT) : p.seq;
  for (int k0 = 0; k0 < kv_end; k0 += KT) {
    __syncthreads();
    for (int e = tid; e < KT * D; e += NT) {
      int j = e / D, d = e % D;
      int key = k0 + j;
      float kv = 0.f, vv = 0.f;
      if (key < p.seq) {
        int64_t ko = base + (int64_t)key * tok_stride + (int64_t)(p.heads + h) * D + d;
        int64_t vo = base + (int64_t)key * tok_stride + (int64_t)(2 * p.heads + h) * D + d;
        kv = load_as_f32(qkv, sizeof(T) == 4 ? C3B_F32 : C3B_BF16, ko);
        vv = load_as_f32(qkv, sizeof(T) == 4 ? C3B_F32 : C3B_BF16, vo);
      }
      Ks[j][d] = kv;
      Vs[j][d] = vv;
    }
    __syncthreads();
    float s[KT];
    float tmax = -INFINITY;
#pragma unroll
    for (int j = 0; j < KT; ++j) {
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) acc = fmaf(q[i], Ks[j][part * 16 + i], acc);
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      const int key = k0 + j;
      if (key >= p.seq || (p.causal && key > q_row)) acc = -INFINITY;
      s[j] = acc;
      tmax = fmaxf(tmax, acc);
    }
    const float m_new = fmaxf(m_run, tmax);
    if (m_new == -INFINITY) continue;  // whole tile masked for this row
    const float corr = expf(m_run - m_new);
    l_run *= corr;
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i] *= corr;
#pragma unroll
    for (int j = 0; j < KT; ++j) {
      const float pj = expf(s[j] - m_new);
      l_run += pj;
#pragma unroll
      for (int i = 0; i < 16; ++i) o[i] = fmaf(pj, Vs[j][part * 16 + i], o[i]);
    }
    m_run = m_new;
  }
  if (valid) {
    const float inv = 1.0f / l_run;
    const int64_t ob = ((int64_t)b * p.seq + q_row) * p.heads * D + (int64_t)h * D + part * 16;
#pragma unroll
    for (int i = 0; i < 16; ++i) store_from_f32(out, sizeof(T) == 4 ? C3B_F32 : C3B_BF16, ob + i, o[i] * inv);
  }
}

int launch_flash_mma(const c3b_tensor& qkv, const c3b_tensor& out, const c3b_flash_params& p, cudaStream_t s);

int launch_flash_attn(const c3b_tensor& qkv, const c3b_tensor& out, const c3b_flash_params& p, cudaStream_t s) {
  C3B_REQUIRE(p.head_dim == fa::D, "flash attention: head_dim must be 64");
  C3B_REQUIRE(qkv.dtype == out.dtype && (qkv.dtype == C3B_F32 || qkv.dtype == C3B_BF16 || qkv.dtype == C3B_F16),
              "flash attention: f32, bf16 or fp16, same dtype in and out");
  const int64_t tokens = (int64_t)p.batch * p.seq;
  C3B_REQUIRE(numel(qkv) == tokens * 3 * p.heads * fa::D, "flash attention: qkv extents");
  C3B_REQUIRE(numel(out) >= tokens * p.heads * fa::D, "flash attention: output too small");
  if (tokens == 0) return C3B_OK;
  if (qkv.dtype == C3B_F16) {
    C3B_REQUIRE(flash_tc_supported(p), "flash attention: fp16 needs head_dim 64 and a multiple of 128 keys");
    return launch_flash_tc(qkv, out, p, s);
  }
  if (qkv.dtype == C3B_BF16) {
    if (flash_tc_supported(p)) return launch_flash_tc(qkv, out, p, s);
    return launch_flash_mma(qkv, out, p, s);
  }
  const int64_t blocks = (int64_t)p.batch * p.heads * ((p.seq + fa::QT - 1) / fa::QT);
  C3B_REQUIRE(blocks < ((int64_t)1 << 31), "flash attention: grid too large");
  flash_simt_kernel<float><<<(unsigned)blocks, fa::NT, 0, s>>>((const float*)qkv.ptr, (float*)out.ptr, p);
  C3B_CHECK_CUDA(cudaGetLastError());
  return C3B_OK;
}

}  // namespace c3b

// Tensor-core stem convolution: NCHW f32 input (Cin*kh*kw <= 32) -> NHWC bf16.
//
// The ResNet stem (3 -> 64 channels, 3x3) has K = 27: too small to pay for a
// 128-byte-per-pixel patch matrix in HBM, too large for plain FP32 FMAs to be
// cheap.  Each warp computes 16 output pixels x 64 channels with
// mma.sync m16n8k16 (bf16 operands, fp32 accumulation, K padded to 32): the
// A fragments are gathered straight from the NCHW input (zero padding by
// bounds checks), the weight fragments stay in registers for the whole kernel,
// and the bias + activation epilogue is staged through shared memory so every
// warp writes its 2 KB output tile with 16-byte coalesced stores.
#include "common.cuh"

namespace c3b {

namespace {

__device__ __forceinline__ uint32_t pk_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void mma_16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

constexpr int COUT = 64;
constexpr int WARPS = 4;

// 3 blocks per SM: caps registers at 170 (no spills; uncapped it took 239 and
// left 8 warps per SM to hide the input gathers: 0.41 -> 0.35 ms at batch 4096)
__global__ void __launch_bounds__(WARPS * 32, 3) stem_mma_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                             const float* __restrict__ bias,
                                                             __nv_bfloat16* __restrict__ out, c3b_stem_params p,
                                                             int act) {
  __shared__ __align__(16) __nv_bfloat16 stage[WARPS][16][COUT + 8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int K = p.c * p.g.kh * p.g.kw;
  // Weight fragments (B is [n][k], k-contiguous pairs), kept in registers.
  uint32_t bf[8][2][2];
#pragma unroll
  for (int nb = 0; nb < 8; ++nb)
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      const int n = nb * 8 + g;
      const int k0 = ks * 16 + 2 * t;
      auto wv = [&](int k) { return k < K ? w[k * COUT + n] : 0.f; };
      bf[nb][ks][0] = pk_bf16(wv(k0), wv(k0 + 1));
      bf[nb][ks][1] = pk_bf16(wv(k0 + 8), wv(k0 + 9));
    }
  float bv[8][2];
#pragma unroll
  for (int nb = 0; nb < 8; ++nb) {
    bv[nb][0] = bias[nb * 8 + 2 * t];
    bv[nb][1] = bias[nb * 8 + 2 * t + 1];
  }
  // The 8 k values this thread feeds: {2t, 2t+1, 2t+8, 2t+9} + 16*ks; k = (c, r, s).
  int kc[8], kr[8], ks_[8];
  bool kv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int k = (i >> 2) * 16 + 2 * t + (i & 1) + ((i >> 1) & 1) * 8;
    kv[i] = k < K;
    const int kk = kv[i] ? k : 0;
    kc[i] = kk / (p.g.kh * p.g.kw);
    kr[i] = (kk / p.g.kw) % p.g.kh;
    ks_[i] = kk % p.g.kw;
  }
  const int64_t M = (int64_t)p.n * p.ho * p.wo;
  const int64_t tiles = (M + 15) / 16;
  for (int64_t tile = (int64_t)blockIdx.x * WARPS + warp; tile < tiles; tile += (int64_t)gridDim.x * WARPS) {
    float v[2][8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t m = tile * 16 + g + 8 * h;
      const bool mok = m < M;
      const int64_t mm = mok ? m : 0;
      const int ow = (int)(mm % p.wo), oh = (int)((mm / p.wo) % p.ho);
      const int n = (int)(mm / ((int64_t)p.wo * p.ho));
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int ih = oh * p.g.sh - p.g.ph0 + kr[i] * p.g.dh;
        const int iw = ow * p.g.sw - p.g.pw0 + ks_[i] * p.g.dw;
        float val = 0.f;
        if (mok && kv[i] && ih >= 0 && ih < p.h && iw >= 0 && iw < p.w)
          val = __ldg(x + (((int64_t)n * p.c + kc[i]) * p.h + ih) * p.w + iw);
        v[h][i] = val;
      }
    }
    uint32_t af[2][4];
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      af[ks][0] = pk_bf16(v[0][ks * 4 + 0], v[0][ks * 4 + 1]);  // row g,   k 2t..2t+1
      af[ks][1] = pk_bf16(v[1][ks * 4 + 0], v[1][ks * 4 + 1]);  // row g+8
      af[ks][2] = pk_bf16(v[0][ks * 4 + 2], v[0][ks * 4 + 3]);  // row g,   k 2t+8..
      af[ks][3] = pk_bf16(v[1][ks * 4 + 2], v[1][ks * 4 + 3]);  // row g+8
    }
    float acc[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      acc[nb][0] = bv[nb][0]; acc[nb][1] = bv[nb][1];
      acc[nb][2] = bv[nb][0]; acc[nb][3] = bv[nb][1];
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) mma_16816(acc[nb], af[ks], bf[nb][ks][0], bf[nb][ks][1]);
    }
    act_inplace<32>(&acc[0][0], act, true);
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      const int col = nb * 8 + 2 * t;
      *reinterpret_cast<uint32_t*>(&stage[warp][g][col]) = pk_bf16(acc[nb][0], acc[nb][1]);
      *reinterpret_cast<uint32_t*>(&stage[warp][g + 8][col]) = pk_bf16(acc[nb][2], acc[nb][3]);
    }
    __syncwarp();
    // 16 rows x 128 bytes: 128 chunks of 16 bytes, 4 per lane, consecutive in memory.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int chunk = lane + 32 * i;
      const int row = chunk >> 3, c8 = (chunk & 7) * 8;
      const int64_t m = tile * 16 + row;
      if (m < M)
        *reinterpret_cast<uint4*>(out + m * COUT + c8) = *reinterpret_cast<const uint4*>(&stage[warp][row][c8]);
    }
    __syncwarp();
  }
}

}  // namespace

bool launch_stem_mma(const c3b_tensor* in, const c3b_tensor& out, const c3b_stem_conv_params& p, cudaStream_t s) {
  const c3b_stem_params& g = p.geom;
  if (p.cout != COUT || g.c * g.g.kh * g.g.kw > 32) return false;
  const int64_t M = (int64_t)g.n * g.ho * g.wo;
  const int64_t tiles = (M + 15) / 16;
  int64_t blocks = (tiles + WARPS - 1) / WARPS;
  const int64_t cap = (int64_t)sm_count() * 16;
  if (blocks > cap) blocks = cap;
  stem_mma_kernel<<<(unsigned)blocks, WARPS * 32, 0, s>>>((const float*)in[0].ptr, (const float*)in[1].ptr,
                                                         (const float*)in[2].ptr, (__nv_bfloat16*)out.ptr, g, p.act);
  return true;
}

}  // namespace c3b

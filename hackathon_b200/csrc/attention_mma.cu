// bf16 tensor-core causal flash attention (bf16 profile).
//
// Same contract as the SIMT kernel in attention.cu: qkv [B,S,3,H,64] bf16 ->
// out [B,S,H*64] bf16, softmax(q k^T * scale, causal) v with fp32 accumulation
// and an online (running max / running sum) softmax, so the reference's
// materialised [B,H,S,S] score tensor (c35/engine.py:1250-1380) never exists.
//
// One CTA = 4 warps = 64 query rows of one (batch, head); each warp owns 16
// rows.  K/V tiles of 64 keys are double-buffered in XOR-swizzled shared memory
// with cp.async; S = Q K^T and O += P V use mma.sync m16n8k16 (bf16 in, fp32
// accumulate), P being re-packed from the S accumulators in registers.
#include "common.cuh"
#include "exp2.cuh"

namespace c3b {

namespace fam {
constexpr int D = 64;
constexpr int QB = 64;
constexpr int KB = 64;
constexpr int NT = 128;
}  // namespace fam

__device__ __forceinline__ uint32_t su32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool pred) {
  int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(su32(dst)), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N)); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Byte offset of (row, 16-byte chunk) in a 64x64 bf16 tile with XOR swizzle.
__device__ __forceinline__ uint32_t swz(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

// MINB = resident CTAs per SM the register allocation is capped for.
// PK: softmax arithmetic on packed fp32 pairs (FFMA2 / FADD2).
template <int MINB, bool PK>
__global__ void __launch_bounds__(fam::NT, MINB) flash_mma_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                            __nv_bfloat16* __restrict__ out, c3b_flash_params p) {
  using namespace fam;
  __shared__ __align__(128) uint8_t Ks[2][KB * D * 2];
  __shared__ __align__(128) uint8_t Vs[2][KB * D * 2];
  const int qblocks = (p.seq + QB - 1) / QB;
  // Heaviest (latest) query blocks first.
  const int qb = qblocks - 1 - (int)(blockIdx.x % qblocks);
  const int h = (blockIdx.x / qblocks) % p.heads;
  const int b = blockIdx.x / (qblocks * p.heads);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t tok = (int64_t)3 * p.heads * D;
  const __nv_bfloat16* base = qkv + (int64_t)b * p.seq * tok;
  const float sl2 = p.scale * 1.4426950408889634f;  // softmax in base 2

  // Q fragments for this warp's 16 rows (4 k-steps of 16 dims).
  uint32_t qa[4][4];
  {
    const int r0 = qb * QB + warp * 16 + g, r1 = r0 + 8;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const int c0 = ks * 16 + 2 * t, c1 = c0 + 8;
      auto ld = [&](int r, int c) -> uint32_t {
        if (r >= p.seq) return 0u;
        return *reinterpret_cast<const uint32_t*>(base + (int64_t)r * tok + (int64_t)h * D + c);
      };
      qa[ks][0] = ld(r0, c0);
      qa[ks][1] = ld(r1, c0);
      qa[ks][2] = ld(r0, c1);
      qa[ks][3] = ld(r1, c1);
    }
  }

  auto load_kv = [&](int buf, int k0) {
    // 64 rows x 8 chunks for K and for V: 1024 chunks over the block.
#pragma unroll
    for (int i = 0; i < 1024 / NT; ++i) {
      const int e = tid + i * NT;
      const int which = e >> 9;  // 0: K, 1: V
      const int r = (e >> 3) & 63, c = e & 7;
      const int key = k0 + r;
      const bool ok = key < p.seq;
      const __nv_bfloat16* src = base + (int64_t)(ok ? key : 0) * tok + (int64_t)((which + 1) * p.heads + h) * D + c * 8;
      uint8_t* dst = (which ? Vs[buf] : Ks[buf]) + swz(r, c);
      cp_async16(dst, src, ok);
    }
    cp_commit();
  };

  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int row0 = qb * QB + warp * 16 + g, row1 = row0 + 8;

  const int kv_tiles = (p.seq + KB - 1) / KB;
  const int ntiles = p.causal ? min(kv_tiles, ((qb + 1) * QB + KB - 1) / KB) : kv_tiles;
  const int warp_last_row = qb * QB + warp * 16 + 15;
  load_kv(0, 0);
  for (int kt = 0; kt < ntiles; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < ntiles) {
      load_kv(buf ^ 1, (kt + 1) * KB);
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (!(p.causal && warp_last_row < kt * KB)) {
    const uint32_t kbase = su32(Ks[buf]), vbase = su32(Vs[buf]);
    // S = Q K^T : 16 x 64 per warp, 8 n-blocks of 8 keys.
    float s[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 4; ks += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = nb * 8 + (lane & 7);
        const int chunk = ks * 2 + (lane >> 3);
        ldsm_x4(kbase + swz(r, chunk), b0, b1, b2, b3);
        mma16816(s[nb], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
        mma16816(s[nb], qa[ks + 1][0], qa[ks + 1][1], qa[ks + 1][2], qa[ks + 1][3], b2, b3);
      }
    }
    // Mask and running max on the raw scores; the scale (positive) is applied
    // to the maxima and folded into the exponent's FMA below.
    const int k0 = kt * KB;
    // Only the diagonal tile (causal) and the sequence tail need masking.
    const bool need_mask = (p.causal && k0 + KB > qb * QB) || (k0 + KB > p.seq);
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        if (need_mask) {
          const int key = k0 + nb * 8 + 2 * t + j;
          if (key >= p.seq || (p.causal && key > row0)) s[nb][j] = -INFINITY;
          if (key >= p.seq || (p.causal && key > row1)) s[nb][2 + j] = -INFINITY;
        }
        mx0 = fmaxf(mx0, s[nb][j]);
        mx1 = fmaxf(mx1, s[nb][2 + j]);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    // Lazy rescaling: the reference maximum m of a row only moves when the
    // tile's maximum exceeds it by more than 8 (log2 units), so P <= 2^8 and
    // most tiles skip the O / l rescale.  The decision is warp-uniform.
    const float ms0 = mx0 * sl2, ms1 = mx1 * sl2;
    if (__any_sync(0xffffffffu, ms0 > m0 + 8.0f || ms1 > m1 + 8.0f)) {
      const float mn0 = fmaxf(m0, ms0), mn1 = fmaxf(m1, ms1);
      const float c0 = mn0 == -INFINITY ? 1.f : exp2_sfu(m0 - mn0);
      const float c1 = mn1 == -INFINITY ? 1.f : exp2_sfu(m1 - mn1);
      m0 = mn0;
      m1 = mn1;
      l0 *= c0;
      l1 *= c1;
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
        o[nb][0] *= c0; o[nb][1] *= c0;
        o[nb][2] *= c1; o[nb][3] *= c1;
      }
    }
    // A row with no visible key so far keeps m = -inf; its exponent base is 0
    // then, and its (masked, -inf) scores still give ~0.
    const float nm0 = m0 == -INFINITY ? 0.f : -m0, nm1 = m1 == -INFINITY ? 0.f : -m1;
    uint32_t pa[4][4];
    if constexpr (PK) {
      const float2 sl2v = make_float2(sl2, sl2), nm0v = make_float2(nm0, nm0), nm1v = make_float2(nm1, nm1);
      float2 ls0 = make_float2(0.f, 0.f), ls1 = make_float2(0.f, 0.f);
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
        // the exponent arguments of a row pair, one FFMA2 each
        const float2 x0 = __ffma2_rn(make_float2(s[nb][0], s[nb][1]), sl2v, nm0v);
        const float2 x1 = __ffma2_rn(make_float2(s[nb][2], s[nb][3]), sl2v, nm1v);
        float2 p0, p1;
        // a quarter of the exponentials on the SFU, three quarters as the
        // packed polynomial on the FMA pipe
        if ((nb & 3) != 0) {
          p0 = exp2_fma2(x0);
          p1 = exp2_fma2(x1);
        } else {
          p0 = make_float2(exp2_sfu(x0.x), exp2_sfu(x0.y));
          p1 = make_float2(exp2_sfu(x1.x), exp2_sfu(x1.y));
        }
        ls0 = __fadd2_rn(ls0, p0);
        ls1 = __fadd2_rn(ls1, p1);
        const int kk = nb >> 1, hi = nb & 1;
        pa[kk][hi * 2 + 0] = pack_bf16(p0.x, p0.y);
        pa[kk][hi * 2 + 1] = pack_bf16(p1.x, p1.y);
      }
      l0 += ls0.x + ls0.y;
      l1 += ls1.x + ls1.y;
    } else {
      float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
        // A quarter of the exponentials on the SFU, three quarters as a
        // polynomial on the FMA pipe: the SFU is the bottleneck of this loop on
        // sm_100 (ncu: XU pipe 72% busy with all exponentials on the SFU).
        float p00, p01, p10, p11;
        if ((nb & 3) != 0) {
          p00 = exp2_fma(fmaf(s[nb][0], sl2, nm0));
          p01 = exp2_fma(fmaf(s[nb][1], sl2, nm0));
          p10 = exp2_fma(fmaf(s[nb][2], sl2, nm1));
          p11 = exp2_fma(fmaf(s[nb][3], sl2, nm1));
        } else {
          p00 = exp2_sfu(fmaf(s[nb][0], sl2, nm0));
          p01 = exp2_sfu(fmaf(s[nb][1], sl2, nm0));
          p10 = exp2_sfu(fmaf(s[nb][2], sl2, nm1));
          p11 = exp2_sfu(fmaf(s[nb][3], sl2, nm1));
        }
        ls0 += p00 + p01;
        ls1 += p10 + p11;
        const int kk = nb >> 1, hi = nb & 1;
        pa[kk][hi * 2 + 0] = pack_bf16(p00, p01);
        pa[kk][hi * 2 + 1] = pack_bf16(p10, p11);
      }
      l0 += ls0;
      l1 += ls1;
    }
    // O += P V : A = P (16 x 64 keys), B = V (64 keys x 64 dims)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int nb = 0; nb < 8; nb += 2) {
        uint32_t b0, b1, b2, b3;
        const int i = lane >> 3;
        const int r = kk * 16 + (i & 1) * 8 + (lane & 7);
        const int chunk = nb + (i >> 1);
        ldsm_x4_t(vbase + swz(r, chunk), b0, b1, b2, b3);
        mma16816(o[nb], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b0, b1);
        mma16816(o[nb + 1], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b2, b3);
      }
    }
    }  // rows of this warp see at least one key of the tile
    __syncthreads();
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float i0 = l0 > 0.f ? 1.f / l0 : 0.f, i1 = l1 > 0.f ? 1.f / l1 : 0.f;
  const int64_t ostride = (int64_t)p.heads * D;
#pragma unroll
  for (int nb = 0; nb < 8; ++nb) {
    const int col = h * D + nb * 8 + 2 * t;
    if (row0 < p.seq)
      *reinterpret_cast<uint32_t*>(out + ((int64_t)b * p.seq + row0) * ostride + col) =
          pack_bf16(o[nb][0] * i0, o[nb][1] * i0);
    if (row1 < p.seq)
      *reinterpret_cast<uint32_t*>(out + ((int64_t)b * p.seq + row1) * ostride + col) =
          pack_bf16(o[nb][2] * i1, o[nb][3] * i1);
  }
}

int launch_flash_mma(const c3b_tensor& qkv, const c3b_tensor& out, const c3b_flash_params& p, cudaStream_t s) {
  C3B_REQUIRE(((uintptr_t)qkv.ptr & 15) == 0 && ((uintptr_t)out.ptr & 3) == 0, "flash attention: alignment");
  const int64_t blocks = (int64_t)p.batch * p.heads * ((p.seq + fam::QB - 1) / fam::QB);
  C3B_REQUIRE(blocks < ((int64_t)1 << 31), "flash attention: grid too large");
  // A/B switches: C3B200_FLASH_OCC=1 selects the uncapped register allocation
  // (the default caps registers for 4 CTAs per SM); C3B200_FLASH_PACKED=0 runs
  // the softmax on scalar fp32 instead of packed pairs.
  static const int variant = [] {
    const char* e = getenv("C3B200_FLASH_OCC");
    const char* k = getenv("C3B200_FLASH_PACKED");
    return ((e && atoi(e) == 1) ? 1 : 0) | ((k && k[0] == '0') ? 2 : 0);
  }();
  const __nv_bfloat16* q = (const __nv_bfloat16*)qkv.ptr;
  __nv_bfloat16* o = (__nv_bfloat16*)out.ptr;
  switch (variant) {
    case 0: flash_mma_kernel<4, true><<<(unsigned)blocks, fam::NT, 0, s>>>(q, o, p); break;
    case 1: flash_mma_kernel<1, true><<<(unsigned)blocks, fam::NT, 0, s>>>(q, o, p); break;
    case 2: flash_mma_kernel<4, false><<<(unsigned)blocks, fam::NT, 0, s>>>(q, o, p); break;
    default: flash_mma_kernel<1, false><<<(unsigned)blocks, fam::NT, 0, s>>>(q, o, p); break;
  }
  C3B_CHECK_CUDA(cudaGetLastError());
  return C3B_OK;
}

}  // namespace c3b

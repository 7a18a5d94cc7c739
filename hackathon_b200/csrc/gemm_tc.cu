// tcgen05 / TMEM / TMA bf16 GEMM and NHWC implicit-GEMM convolution (sm_100a).
//
// Replaces, for the bf16 precision profile, the reference contractions
// c3_gemm_epilogue (c35/engine.py:722-849; fused_gemm_epilogue_f32 and
// fused_matmul_bias_f32) and the conv chain im2col_f32 -> matmul_f32 (cuBLAS) ->
// conv_reshape_f32 -> add_bias_f32 -> relu_f32 / fused_residual_relu_f32
// (c32/decompositions.py:301-378, 505-550; c32/kernel_registry.py:318-453, 654-662).
//
// Design (one persistent CTA per SM, 6 warps):
//   warp 0      TMA producer: A tile 128x64 and B tile BNx64 (bf16, 128B swizzle)
//               into a ring of shared-memory stages (mbarrier full/empty pairs).
//               For convolution A is fetched straight from the NHWC activation
//               with a 4-D tensor map per (kh,kw) tap — TMA's out-of-bounds zero
//               fill supplies the padding, so no patch matrix ever exists.
//               Stride-2 convs use four parity-split views of the input
//               (dims C, W/2, H/2, N), one per (row parity, column parity).
//   warp 1      allocates TMEM (2 accumulator buffers of BN fp32 columns) and
//               issues tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BN, K=16)
//               from one thread; tcgen05.commit releases smem stages and
//               publishes finished accumulators.
//   warps 2..5  epilogue: tcgen05.ld 32x32b -> +bias (folded BN) [+residual]
//               -> ReLU/GELU -> bf16/f32 stores.  Double-buffered accumulators
//               let the epilogue of tile i overlap the MMAs of tile i+1.
// Every mbarrier wait is bounded (globaltimer); on expiry the kernel records
// an error in the device status word, stops issuing work, frees its TMEM and
// returns, so the context stays usable.
#include <cuda.h>
#include <cuda_fp4.h>

#include "common.cuh"
#include "tc_prims.cuh"

namespace c3b {

namespace tc {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int NUM_THREADS = 192;
constexpr int HALO_THREADS = 320;  // producer, MMA, 8 epilogue warps
constexpr int HALO16_THREADS = 576;  // producer, MMA, 16 epilogue warps (tc_gemm_kernel, tc_conv_halo_kernel)

struct __align__(64) TmaMaps {
  CUtensorMap a[4];
  CUtensorMap b;
  // epilogue tiles (row-ring conv): residual load and output store, 64-byte
  // swizzled boxes of 32 channels x one warp's 32 pixels
  CUtensorMap res, out;
};

struct TcArgs {
  int64_t M, N, K;
  int n_tiles_n, n_tiles, k_blocks;
  int block_n, stages;
  // epilogue
  void* out;
  int dt_out;
  const float* bias;
  const void* res;
  int dt_res;
  int act;
  // conv geometry (conv == 0 -> plain GEMM with a 2-D A map)
  int conv, cblocks, ksz, stride, pad;
  int pix;         // Ho*Wo
  int wo, bh;      // box geometry
  int cin;
  // halo mode (3x3 stride-1 convolution, tc_conv_halo_kernel)
  int img, wt, wblocks, ho, n_img, rows, halo_bytes, hstages;
  int bres;  // 1: all weight taps resident in shared memory for the whole kernel
  // row-ring mode (tc_conv_rowring_kernel)
  int segs, seg_rows, ring, row_bytes, n_items;
  int rring;  // sliding-window kernel: residual rows staged by TMA in this many slots (0: none)
  int cg;     // tc_gemm_kernel: 1 single CTAs, 2 CTA pairs (M = 256 tiles)
  // fp8 GEMM (tc_gemm_kernel<1>): per-row scale of A, per-column scale of B
  const float* a_scale;
  const float* b_scale;
  // tc_gemm_kernel: bf16 output through per-warp shared-memory tiles and TMA
  // stores (maps.out: 16 columns x 32 rows, 32-byte swizzle)
  int tma_out;
  // 16-bit format of A, B and every 16-bit output / residual: 0 bf16, 1 fp16
  int h16;
  // optional wait counters of the row-ring kernel (C3B200_CONV_PROF=1), else null
  unsigned long long* prof;
  // (the fields below sit last: placed earlier they changed the register
  // allocation of the other tc_gemm_kernel variants into spills)
  // fused 1x1 stride-2 shortcut (tc_gemm_kernel<0, 1>, convolutions): aux_n
  // more accumulator columns per tile, fed by the centre tap's K blocks
  // [aux_kb0, aux_kb0 + cblocks) against aux_w [aux_n][cin] (resident in
  // shared memory); output aux_out [M][aux_n] = acc + aux_bias, no activation
  int aux_n, aux_kb0;
  const uint16_t* aux_w;
  const float* aux_bias;
  uint16_t* aux_out;
};

// Row-ring wait-profiler slots (cycles summed over CTAs; epilogue slots over warps).
enum { RP_PROD_TOTAL, RP_PROD_EMPTY, RP_MMA_TOTAL, RP_MMA_RFULL, RP_MMA_TEMPTY, RP_EPI_TOTAL, RP_EPI_TFULL,
       RP_EPI_RES, RP_PAIRS, RP_COUNT };

// Epilogue for 32 columns of one bf16 output row whose residual (bf16) was
// prefetched into `rv` (4 x 16 bytes): +bias -> +residual -> act -> 64-byte store.
__device__ __forceinline__ void store32_bf16(const TcArgs& a, int64_t off, int64_t col0, float* v, const uint4* rv) {
  if (a.bias) {
    const float4* bp = reinterpret_cast<const float4*>(a.bias + col0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 b = __ldg(bp + i);
      v[4 * i] += b.x; v[4 * i + 1] += b.y; v[4 * i + 2] += b.z; v[4 * i + 3] += b.w;
    }
  }
  if (rv) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float rr[8];
      unpack8h(rv[i], rr, a.h16);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[8 * i + j] += rr[j];
    }
  }
  act_inplace<32>(v, a.act, true);
  uint4* op = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + off);
#pragma unroll
  for (int i = 0; i < 4; ++i) op[i] = pack8h(v + 8 * i, a.h16);
}

// Residual of 32 consecutive columns (bf16: 64 bytes, f32: 128 bytes) as raw words.
__device__ __forceinline__ void load_res32(const TcArgs& a, int64_t off, uint4* r) {
  if (a.dt_res != C3B_F32) {
    const uint4* rp = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.res) + off);
#pragma unroll
    for (int i = 0; i < 4; ++i) r[i] = rp[i];
  } else {
    const uint4* rp = reinterpret_cast<const uint4*>(static_cast<const float*>(a.res) + off);
#pragma unroll
    for (int i = 0; i < 8; ++i) r[i] = rp[i];
  }
}

// (x row scale x column scale) -> +bias -> +residual -> act -> store 32 columns
// of one output row (bf16 or f32).  The scales are the fp8 GEMM's dequantisation.
__device__ __forceinline__ void finish32(const TcArgs& a, int64_t off, int64_t col0, float* v, const uint4* r,
                                         float rs = 1.0f) {
  if (a.b_scale) {
    const float4* sp = reinterpret_cast<const float4*>(a.b_scale + col0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 c = __ldg(sp + i);
      v[4 * i] = v[4 * i] * rs * c.x; v[4 * i + 1] = v[4 * i + 1] * rs * c.y;
      v[4 * i + 2] = v[4 * i + 2] * rs * c.z; v[4 * i + 3] = v[4 * i + 3] * rs * c.w;
    }
  }
  if (a.bias) {
    const float4* bp = reinterpret_cast<const float4*>(a.bias + col0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 b = __ldg(bp + i);
      v[4 * i] += b.x; v[4 * i + 1] += b.y; v[4 * i + 2] += b.z; v[4 * i + 3] += b.w;
    }
  }
  if (r) {
    if (a.dt_res != C3B_F32) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float rr[8];
        unpack8h(r[i], rr, a.h16);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[8 * i + j] += rr[j];
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float* rf = reinterpret_cast<const float*>(&r[i]);
#pragma unroll
        for (int j = 0; j < 4; ++j) v[4 * i + j] += rf[j];
      }
    }
  }
  act_inplace<32>(v, a.act, a.dt_out != C3B_F32);
  if (a.dt_out != C3B_F32) {
    uint4* op = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + off);
#pragma unroll
    for (int i = 0; i < 4; ++i) op[i] = pack8h(v + 8 * i, a.h16);
  } else {
    float4* op = reinterpret_cast<float4*>(static_cast<float*>(a.out) + off);
#pragma unroll
    for (int i = 0; i < 8; ++i) op[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  }
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}
// The shared-memory source of all but the most recent committed bulk store has been read.
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }

// Residual of 16 consecutive columns (bf16: 32 bytes, f32: 64 bytes) as raw words.
__device__ __forceinline__ void load_res16(const TcArgs& a, int64_t off, uint4* r) {
  if (a.dt_res != C3B_F32) {
    const uint4* rp = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.res) + off);
    r[0] = rp[0]; r[1] = rp[1];
  } else {
    const uint4* rp = reinterpret_cast<const uint4*>(static_cast<const float*>(a.res) + off);
#pragma unroll
    for (int i = 0; i < 4; ++i) r[i] = rp[i];
  }
}

// 16 columns of one output row: (x row scale x column scale) -> +bias ->
// +residual -> act -> store (bf16 or f32).
// finish16's arithmetic without the store: (x scales) -> +bias -> +residual -> act.
// With `rtile`, the f32 residual is read as it is added from this lane's row of
// a 64-byte-swizzled shared-memory tile (16 f32 per row), so it never needs
// registers of its own.
__device__ __forceinline__ void epi16(const TcArgs& a, int64_t col0, float* v, const uint4* r, float rs,
                                      const uint8_t* rtile = nullptr, int lane = 0) {
  // pairwise (packed fp32) arithmetic: v2[i] holds columns 2i, 2i+1
  float2* v2 = reinterpret_cast<float2*>(v);
  if (a.b_scale) {
    const float4* sp = reinterpret_cast<const float4*>(a.b_scale + col0);
    const float2 rr = make_float2(rs, rs);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 c = __ldg(sp + i);
      v2[2 * i] = __fmul2_rn(v2[2 * i], __fmul2_rn(rr, make_float2(c.x, c.y)));
      v2[2 * i + 1] = __fmul2_rn(v2[2 * i + 1], __fmul2_rn(rr, make_float2(c.z, c.w)));
    }
  }
  if (a.bias) {
    const float4* bp = reinterpret_cast<const float4*>(a.bias + col0);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 b = __ldg(bp + i);
      v2[2 * i] = __fadd2_rn(v2[2 * i], make_float2(b.x, b.y));
      v2[2 * i + 1] = __fadd2_rn(v2[2 * i + 1], make_float2(b.z, b.w));
    }
  }
  if (rtile) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 q = *reinterpret_cast<const float4*>(rtile + swz64(lane, i));
      v2[2 * i] = __fadd2_rn(v2[2 * i], make_float2(q.x, q.y));
      v2[2 * i + 1] = __fadd2_rn(v2[2 * i + 1], make_float2(q.z, q.w));
    }
  } else if (r) {
    if (a.dt_res != C3B_F32) {
      const uint32_t* rb = reinterpret_cast<const uint32_t*>(r);
#pragma unroll
      for (int i = 0; i < 8; ++i) v2[i] = __fadd2_rn(v2[i], unpack2h(rb[i], a.h16));
    } else {
      const float2* rf = reinterpret_cast<const float2*>(r);
#pragma unroll
      for (int i = 0; i < 8; ++i) v2[i] = __fadd2_rn(v2[i], rf[i]);
    }
  }
  act_inplace<16>(v, a.act, a.dt_out != C3B_F32);
}

__device__ __forceinline__ void finish16(const TcArgs& a, int64_t off, int64_t col0, float* v, const uint4* r,
                                         float rs) {
  epi16(a, col0, v, r, rs);
  float2* v2 = reinterpret_cast<float2*>(v);
  if (a.dt_out != C3B_F32) {
    uint4* op = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + off);
#pragma unroll
    for (int i = 0; i < 2; ++i)
      op[i] = make_uint4(pack2h(v2[4 * i], a.h16), pack2h(v2[4 * i + 1], a.h16), pack2h(v2[4 * i + 2], a.h16),
                         pack2h(v2[4 * i + 3], a.h16));
  } else {
    float4* op = reinterpret_cast<float4*>(static_cast<float*>(a.out) + off);
#pragma unroll
    for (int i = 0; i < 4; ++i) op[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  }
}

// MODE 0: bf16 A and B (64 elements per 128-byte K block, kind::f16).
// MODE 1: e4m3 A and B (128 elements per K block, kind::f8f6f4); per-row and
//         per-column scales in the epilogue.
// MODE 2: W4A16 — bf16 A, B as packed FP4 E2M1 with an fp32 scale per 16 K
//         elements.  TMA brings the packed tile (32 bytes per row per K block)
//         and its scales; converter warps 10..17 expand them into the same
//         128-byte-swizzled bf16 stage the MMA reads (kind::f16), and warps 2..9
//         run the epilogue.
// The shared-memory layout and descriptor arithmetic of A/B are the same bytes
// in every mode.
constexpr int W4_GROUP = 16;  // K elements per FP4 scale

// CG = 2: CTA pairs (clusters of two) share each M=256 tile: every CTA loads
// its own 128 A rows and half of the tile's B columns, CTA 0 issues
// tcgen05.mma.cta_group::2 for both, and each CTA drains its own 128 rows.
// Per SM that halves the B bytes staged and read per MMA.  bf16/fp16 only.
template <int MODE, int CG = 1, bool AUX = false>
__global__ void __launch_bounds__(HALO16_THREADS, 1) tc_gemm_kernel(const __grid_constant__ TmaMaps maps, const TcArgs a) {
  constexpr bool F8 = MODE == 1, W4 = MODE == 2, TF = MODE == 3;
  static_assert(CG == 1 || MODE == 0, "CTA pairs: bf16/fp16 operands only");
  const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;
  const int cid = (int)blockIdx.x / CG, ncl = (int)gridDim.x / CG;
  constexpr int KEL = F8 ? 128 : TF ? 32 : BK;  // elements per K block (one 128-byte row)
  constexpr int EPIW = W4 ? 8 : 16;   // epilogue warps
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled stages.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stages = a.stages;
  const uint32_t a_bytes = BM * BK * 2;
  const uint32_t b_bytes = (uint32_t)(a.block_n / CG) * BK * 2;  // this CTA's share of B
  const uint32_t raw_bytes = W4 ? (uint32_t)a.block_n * (BK / 2) : 0u;                 // packed FP4
  const uint32_t scl_bytes = W4 ? (uint32_t)a.block_n * (BK / W4_GROUP) * 4u : 0u;     // fp32 scales
  // Resident B (bres, single CTAs, bf16/fp16): the CTA's whole B column block
  // (k_blocks x b_bytes) is loaded once; only A streams through the stages.
  const bool bres = MODE == 0 && CG == 1 && a.bres != 0;
  uint8_t* sa = smem;
  uint8_t* sb = smem + (size_t)stages * a_bytes;
  uint8_t* sraw = sb + (size_t)(bres ? a.k_blocks : stages) * b_bytes;
  uint8_t* sscl = sraw + (size_t)stages * raw_bytes;
  // fused shortcut weights: cblocks x [aux_n rows x 128 bytes], 128-byte swizzle
  constexpr bool aux = AUX;  // fused 1x1 shortcut (conv launches with has_shortcut)
  static_assert(!AUX || (MODE == 0 && CG == 1), "fused shortcut: single bf16/fp16 tiles");
  uint8_t* saux = sscl + (size_t)stages * scl_bytes;  // 1024-byte aligned: every region above is
  const uint32_t aux_kb_bytes = (uint32_t)a.aux_n * 128u;
  // per-warp output tiles (2 per epilogue warp: 1 KB for 16-bit output, 2 KB
  // for f32 output; 1024-byte aligned)
  const uint32_t tile_bytes = a.tma_out == 2 ? 2048u : 1024u;
  uint8_t* stg = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(saux + (aux ? (size_t)a.cblocks * aux_kb_bytes : 0)) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(stg + (a.tma_out ? (size_t)EPIW * 2 * tile_bytes : 0));
  uint64_t* full = bars;
  uint64_t* empty = bars + stages;
  uint64_t* bready = bars + 2 * stages;  // MODE 2: B stage expanded
  uint64_t* tfull = bars + 3 * stages;
  uint64_t* tempty = tfull + 2;
  uint64_t* rbar = tempty + 2;  // f32 TMA epilogue: residual tile landed (2 per epilogue warp)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 2 * EPIW);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // one accumulator buffer: block_n columns (+ aux_n); recomputed where used
  // from the kernel parameters, which costs no register
#define ACC_COLS ((uint32_t)(a.block_n + (aux ? a.aux_n : 0)))
  const uint32_t tmem_cols = ACC_COLS * 2;

  if (aux) {
    // constant weights: read before the dependency wait, made visible to the
    // MMA (async proxy) by the fence before the barrier below
    const int chunks = a.aux_n * a.cblocks * 8;  // 16-byte chunks
    for (int i = threadIdx.x; i < chunks; i += blockDim.x) {
      const int c = i & 7, n = (i >> 3) % a.aux_n, cb = (i >> 3) / a.aux_n;
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(a.aux_w + (size_t)n * a.cin + cb * BK + c * 8));
      *reinterpret_cast<uint4*>(saux + (size_t)cb * aux_kb_bytes + n * 128 + ((c ^ (n & 7)) << 4)) = v;
    }
    fence_proxy_async();
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
      mbar_init(&bready[i], bres ? 1 : 8);  // bres: bready[0] = B resident
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], EPIW * CG);  // CTA pairs: both CTAs' epilogues release CTA 0's accumulator
    }
    for (int i = 0; i < 2 * EPIW; ++i) mbar_init(&rbar[i], 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < 4; ++i) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.a[i])));
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.b)));
  }
  if (warp == 1) {
    if (CG == 2) {
      // one warp of each CTA of the pair allocates collectively
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(tmem_cols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(tmem_cols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  tc_fence_before();
  __syncthreads();
  if (CG == 2) cluster_sync();  // the peer's barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (bres && warp == 0 && lane == 0 && cid < a.n_tiles) {
    // resident B (constant weights, so before the dependency wait): every tile
    // of this CTA has column block cid % n_tiles_n (the grid is a multiple of
    // n_tiles_n)
    const int n0 = (cid % a.n_tiles_n) * a.block_n;
    mbar_arrive_tx(&bready[0], (uint32_t)a.k_blocks * b_bytes);
    for (int kb = 0; kb < a.k_blocks; ++kb)
      tma_load_2d(sb + (size_t)kb * b_bytes, &maps.b, &bready[0], kb * BK, n0);
  }
  // Programmatic dependent launch: the prologue above (barriers, TMEM, tensor
  // maps, constant weights) may overlap the previous kernel's tail; every
  // activation read and every global write comes after it has completed.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // every CTA of this persistent grid is resident: the next kernel may launch
  // onto SMs as they free up (it waits on griddepcontrol before its activations)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = cid; t < a.n_tiles; t += ncl) {
        const int mb = t / a.n_tiles_n, nb = t % a.n_tiles_n;
        const int m0 = (mb * CG + (int)rank) * BM, n0 = nb * a.block_n + (int)rank * (a.block_n / CG);
        int img0 = 0, oh0 = 0;
        if (a.conv) {
          img0 = m0 / a.pix;
          oh0 = (m0 % a.pix) / a.wo;
        }
        for (int kb = 0; kb < a.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, 11)) goto producer_done;
          uint8_t* dA = sa + (size_t)stage * a_bytes;
          uint8_t* dB = sb + (size_t)stage * b_bytes;
          if (W4) {
            mbar_arrive_tx(&full[stage], a_bytes + raw_bytes + scl_bytes);
            tma_load_2d(dA, &maps.a[0], &full[stage], kb * BK, m0);
            tma_load_2d(sraw + (size_t)stage * raw_bytes, &maps.a[1], &full[stage], kb * (BK / 2), n0);
            tma_load_3d(sscl + (size_t)stage * scl_bytes, &maps.a[2], &full[stage], 0, n0, kb);
          } else if (CG == 2) {
            // both CTAs' bytes are counted on CTA 0's barrier; only CTA 0 arrives
            const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
            if (rank == 0) mbar_arrive_tx(&full[stage], 2 * (a_bytes + b_bytes));
            if (!a.conv) {
              tma_load_2d_pair(dA, &maps.a[0], fb, kb * KEL, m0);
            } else {
              const int tap = kb / a.cblocks, cb = kb % a.cblocks;
              const int r = tap / a.ksz, s = tap % a.ksz;
              int map = 0, ro, so;
              if (a.stride == 1) {
                ro = r - a.pad;
                so = s - a.pad;
              } else {
                const int dr = r - a.pad, ds = s - a.pad;
                const int pr = dr & 1, ps = ds & 1;
                ro = (dr - pr) / 2;
                so = (ds - ps) / 2;
                map = pr * 2 + ps;
              }
              tma_load_4d_pair(dA, &maps.a[map], fb, cb * BK, so, oh0 + ro, img0);
            }
            tma_load_2d_pair(dB, &maps.b, fb, kb * KEL, n0);
          } else if (!a.conv) {
            mbar_arrive_tx(&full[stage], bres ? a_bytes : a_bytes + b_bytes);
            tma_load_2d(dA, &maps.a[0], &full[stage], kb * KEL, m0);
            if (!bres) tma_load_2d(dB, &maps.b, &full[stage], kb * KEL, n0);
          } else {
            mbar_arrive_tx(&full[stage], bres ? a_bytes : a_bytes + b_bytes);
            const int tap = kb / a.cblocks, cb = kb % a.cblocks;
            const int r = tap / a.ksz, s = tap % a.ksz;
            int map = 0, ro, so;
            if (a.stride == 1) {
              ro = r - a.pad;
              so = s - a.pad;
            } else {
              const int dr = r - a.pad, ds = s - a.pad;
              const int pr = dr & 1, ps = ds & 1;
              ro = (dr - pr) / 2;
              so = (ds - ps) / 2;
              map = pr * 2 + ps;
            }
            tma_load_4d(dA, &maps.a[map], &full[stage], cb * BK, so, oh0 + ro, img0);
            if (!bres) tma_load_2d(dB, &maps.b, &full[stage], kb * BK, n0);
          }
          if (++stage == stages) { stage = 0; phase ^= 1; }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (CTA pairs: CTA 0 only)
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = F8   ? instr_desc_e4m3(BM, a.block_n)
                             : TF ? instr_desc_tf32(BM, a.block_n)
                                  : instr_desc_h(BM * CG, a.block_n, a.h16);
      const uint32_t idesc_aux = aux ? instr_desc_h(BM, a.aux_n, a.h16) : 0u;
      const uint64_t xd0 = smem_desc(smem_u32(saux));
      // stage descriptors = base descriptor + offset in 16-byte units
      const uint64_t ad0 = smem_desc(smem_u32(sa)), bd0 = smem_desc(smem_u32(sb));
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool b_ok = !bres || cid >= a.n_tiles || mbar_wait(&bready[0], 0, abort_flag, 17);
      for (int t = cid; t < a.n_tiles && b_ok; t += ncl) {
        if (!(CG == 2 ? mbar_wait_cluster(&tempty[acc], acc_phase ^ 1, abort_flag, 12)
                      : mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, 12)))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)acc * ACC_COLS;
        bool ok = true;
        for (int kb = 0; kb < a.k_blocks; ++kb) {
          if (!mbar_wait(W4 ? &bready[stage] : &full[stage], phase, abort_flag, 13)) { ok = false; break; }
          tc_fence_after();
          const uint64_t ad = ad0 + (uint64_t)stage * (a_bytes >> 4);
          const uint64_t bd = bd0 + (uint64_t)(bres ? kb : stage) * (b_bytes >> 4);
#pragma unroll
          for (int k = 0; k < 4; ++k) {  // four 32-byte K steps per 128-byte row
            if (CG == 2)
              mma_bf16_pair(d_tmem, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc, (kb > 0 || k > 0) ? 1u : 0u);
            else if (F8)
              mma_e4m3(d_tmem, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc, (kb > 0 || k > 0) ? 1u : 0u);
            else if (TF)
              mma_tf32(d_tmem, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc, (kb > 0 || k > 0) ? 1u : 0u);
            else
              mma_bf16(d_tmem, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          if (aux && kb >= a.aux_kb0 && kb < a.aux_kb0 + a.cblocks) {
            // the centre tap's A block is the shortcut's A: its N columns go
            // to the accumulator block after the tile's own
            const uint64_t xd = xd0 + (uint64_t)(((uint32_t)(kb - a.aux_kb0) * aux_kb_bytes) >> 4);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_bf16(d_tmem + (uint32_t)a.block_n, ad + (uint64_t)(2 * k), xd + (uint64_t)(2 * k), idesc_aux,
                       (kb > a.aux_kb0 || k > 0) ? 1u : 0u);
          }
          if (CG == 2)
            mma_commit_pair(&empty[stage]);
          else
            mma_commit(&empty[stage]);
          if (++stage == stages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        if (CG == 2)
          mma_commit_pair(&tfull[acc]);
        else
          mma_commit(&tfull[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
    }
  } else if (W4 && warp >= 2 + EPIW) {
    // ---------------- FP4 converters (warps 10..17): each K block of B is
    // block_n rows x 64 elements; a unit is one row's 8-element chunk (4 packed
    // bytes, one scale) written as 16 bf16 bytes at its 128-byte-swizzle slot.
    const int ct = threadIdx.x - (2 + EPIW) * 32;  // 0..255
    const int units = a.block_n * 8;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < a.n_tiles && ok; t += gridDim.x) {
      for (int kb = 0; kb < a.k_blocks; ++kb) {
        ok = mbar_wait(&full[stage], phase, abort_flag, 15);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        const uint8_t* raw = sraw + (size_t)stage * raw_bytes;
        const float* scl = reinterpret_cast<const float*>(sscl + (size_t)stage * scl_bytes);
        uint8_t* dst = sb + (size_t)stage * b_bytes;
        // all loads of this thread's units first (up to 8: block_n / 32), then
        // the conversions and stores, so the shared-memory latencies overlap
        uint32_t pk[8];
        float sc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int u = ct + 256 * i;
          if (u < units) {
            const int r = u >> 3, c = u & 7;
            pk[i] = *reinterpret_cast<const uint32_t*>(raw + r * 32 + c * 4);
            sc[i] = scl[r * (BK / W4_GROUP) + (c >> 1)];
          }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int u = ct + 256 * i;
          if (u < units) {
            const int r = u >> 3, c = u & 7;
            const float2 s2 = make_float2(sc[i], sc[i]);
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const __half2_raw h =
                  __nv_cvt_fp4x2_to_halfraw2((__nv_fp4x2_storage_t)((pk[i] >> (8 * j)) & 0xFF), __NV_E2M1);
              const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
              o[j] = pack2h(__fmul2_rn(f, s2), a.h16);
            }
            *reinterpret_cast<uint4*>(dst + r * 128 + ((c ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
          }
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bready[stage]);
        if (++stage == stages) { stage = 0; phase ^= 1; }
      }
    }
  } else {
    // ---------------- epilogue warps 2..17: warp w drains TMEM lane quarter
    // (w % 4) and one quarter of the tile's columns in 16-column chunks.  Four
    // warps per quarter keep the issue slots busy (the epilogue runs ~30
    // instructions per element with GELU and fp8 scales); 16-column chunks keep
    // the live set within the 96 registers of a 576-thread CTA.  The residual
    // is prefetched one chunk ahead.
    const int q = warp & 3;
    const int part = (warp - 2) >> 2;
    const int cols = a.block_n / (EPIW / 4);  // columns per warp
    int acc = 0;
    uint32_t acc_phase = 0;
    uint8_t* my_stg = stg + (size_t)(warp - 2) * 2 * tile_bytes;
    uint32_t n_st = 0;  // TMA stores this warp has issued
    // f32 output through TMA (tma_out == 2): chunk g of this warp (16 columns
    // x 32 rows, 2 KB, 64-byte swizzle) lives in tile g & 1.  Its residual
    // arrives there by TMA, issued while chunk g-1 is finished (the first one
    // before the accumulator wait), the result overwrites it in place and
    // leaves by TMA store.
    uint64_t* my_rbar = rbar + 2 * (warp - 2);
    const bool f32_tma = a.tma_out == 2;
    const bool res_tma = f32_tma && a.res != nullptr;
    uint32_t g = 0;
    if (res_tma && lane == 0 && cid < a.n_tiles) {
      const int mb = cid / a.n_tiles_n, nb = cid % a.n_tiles_n;
      mbar_arrive_tx(&my_rbar[0], 2048);
      tma_load_2d(my_stg, &maps.res, &my_rbar[0], nb * a.block_n + part * cols, (mb * CG + (int)rank) * BM + q * 32);
    }
    for (int t = cid; t < a.n_tiles; t += ncl) {
      const int mb = t / a.n_tiles_n, nb = t % a.n_tiles_n;
      const int64_t row0 = ((int64_t)mb * CG + rank) * BM + q * 32;  // first row of this warp's lanes
      const int64_t row = row0 + lane;
      const int64_t col_base = (int64_t)nb * a.block_n + part * cols;
      const bool row_ok = row < a.M && col_base < a.N;
      const float rs = (F8 && row_ok) ? __ldg(a.a_scale + row) : 1.0f;
      uint4 rc[4], rn[4];
      if (a.res && row_ok && !f32_tma) load_res16(a, row * a.N + col_base, rc);
      const bool ok = mbar_wait(&tfull[acc], acc_phase, abort_flag, 14);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)acc * ACC_COLS + (uint32_t)(part * cols);
#pragma unroll 1
      for (int c0 = 0; f32_tma && c0 < cols; c0 += 16) {
        float v[16];
        tmem_ld16(tbase + c0, v);
          const uint32_t slot = g & 1;
          uint8_t* tile = my_stg + slot * 2048;
          if (lane == 0) {
            // the next chunk's residual into the other tile, once the store
            // that last used it has read it
            int nrow0 = (int)row0, ncol = (int)col_base + c0 + 16;
            bool next = true;
            if (c0 + 16 >= cols) {
              const int t2 = t + ncl;
              next = t2 < a.n_tiles;
              if (next) {
                const int mb2 = t2 / a.n_tiles_n, nb2 = t2 - mb2 * a.n_tiles_n;
                nrow0 = (mb2 * CG + (int)rank) * BM + q * 32;
                ncol = nb2 * a.block_n + part * cols;
              }
            }
            bulk_wait_read0();
            if (res_tma && next) {
              mbar_arrive_tx(&my_rbar[slot ^ 1], 2048);
              tma_load_2d(my_stg + (slot ^ 1) * 2048, &maps.res, &my_rbar[slot ^ 1], ncol, nrow0);
            }
          }
          if (res_tma) {
            const bool rok = mbar_wait(&my_rbar[slot], (g >> 1) & 1, abort_flag, 16);
            if (!__all_sync(0xffffffffu, rok)) break;
          }
          __syncwarp();
          // (chunks past N hold padding: no bias or scale reads there; each
          // lane reads and then overwrites only its own row of the tile)
          if (col_base + c0 < a.N) epi16(a, col_base + c0, v, nullptr, rs, res_tma ? tile : nullptr, lane);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            *reinterpret_cast<float4*>(tile + swz64(lane, i)) =
                make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          fence_proxy_async();
          __syncwarp();
          if (lane == 0 && row0 < a.M && col_base + c0 < a.N) {
            tma_store_2d(&maps.out, tile, (int)(col_base + c0), (int)row0);
            bulk_commit();
          }
          ++g;
      }
#pragma unroll 1
      for (int c0 = 0; !f32_tma && c0 < cols; c0 += 16) {
        const bool more = a.res && !f32_tma && row_ok && c0 + 16 < cols && col_base + c0 + 16 < a.N;
        if (more) load_res16(a, row * a.N + col_base + c0 + 16, rn);
        float v[16];
        tmem_ld16(tbase + c0, v);
        if (a.tma_out) {
          // bf16 rows through the warp's tile: 32 rows x 32 bytes with the
          // 32-byte swizzle (16-byte chunk bit 4 ^= address bit 7, conflict
          // free), then one TMA store of 16 columns x 32 rows; rows past M
          // are clipped by the tensor map
          if (row0 < a.M && col_base + c0 < a.N) {
            epi16(a, col_base + c0, v, a.res ? rc : nullptr, rs);
            uint8_t* tile = my_stg + (n_st & 1) * 1024;
            if (lane == 0) bulk_wait_read1();  // the store that last used this tile has read it
            __syncwarp();
#pragma unroll
            for (int h = 0; h < 2; ++h)
              *reinterpret_cast<uint4*>(tile + lane * 32 + ((h ^ ((lane >> 2) & 1)) << 4)) = pack8h(v + 8 * h, a.h16);
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&maps.out, tile, (int)(col_base + c0), (int)row0);
              bulk_commit();
            }
            ++n_st;
          }
        } else if (row_ok && col_base + c0 < a.N) {
          finish16(a, row * a.N + col_base + c0, col_base + c0, v, a.res ? rc : nullptr, rs);
        }
        if (more) {
#pragma unroll
          for (int i = 0; i < 4; ++i) rc[i] = rn[i];
        }
      }
      if (aux) {
        // fused shortcut: this warp's quarter of the aux_n columns, + bias,
        // no activation, 16-bit rows straight from registers
        const int acols = a.aux_n / (EPIW / 4);
#pragma unroll 1
        for (int c0 = 0; c0 < acols; c0 += 16) {
          float v[16];
          tmem_ld16(tbase - (uint32_t)(part * cols) + (uint32_t)(a.block_n + part * acols + c0), v);
          if (row < a.M) {
            const float4* bp = reinterpret_cast<const float4*>(a.aux_bias + part * acols + c0);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float4 b = __ldg(bp + i);
              v[4 * i] += b.x; v[4 * i + 1] += b.y; v[4 * i + 2] += b.z; v[4 * i + 3] += b.w;
            }
            uint4* op = reinterpret_cast<uint4*>(a.aux_out + row * a.aux_n + part * acols + c0);
            op[0] = pack8h(v, a.h16);
            op[1] = pack8h(v + 8, a.h16);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (CG == 2)
          mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
        else
          mbar_arrive(&tempty[acc]);
      }
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
    if (a.tma_out && lane == 0) bulk_wait0();
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {
    // Give copies still in flight time to land before shared memory is released.
    for (int i = 0; i < 1000; ++i) __nanosleep(1000);
  }
  // CTA pairs: neither CTA leaves (releasing its shared memory and TMEM) while
  // the pair's MMAs or the peer's remote arrivals may still reach it
  if (CG == 2) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if (CG == 2)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols));
  }
#undef ACC_COLS
}

// Epilogue for one 16-column chunk of one output row: +bias [+residual] -> act -> store.
__device__ __forceinline__ void store_chunk(const TcArgs& a, int64_t off, int64_t col0, float* v) {
  if (a.bias) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] += a.bias[col0 + i];
  }
  if (a.res) {
    if (a.dt_res != C3B_F32) {
      const uint4* rp = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.res) + off);
      float rr[16];
      unpack8h(rp[0], rr, a.h16);
      unpack8h(rp[1], rr + 8, a.h16);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] += rr[i];
    } else {
      const float4* rp = reinterpret_cast<const float4*>(static_cast<const float*>(a.res) + off);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float4 r = rp[i];
        v[4 * i] += r.x; v[4 * i + 1] += r.y; v[4 * i + 2] += r.z; v[4 * i + 3] += r.w;
      }
    }
  }
  act_inplace<16>(v, a.act, a.dt_out != C3B_F32);
  if (a.dt_out != C3B_F32) {
    uint4* op = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + off);
    op[0] = pack8h(v, a.h16);
    op[1] = pack8h(v + 8, a.h16);
  } else {
    float4* op = reinterpret_cast<float4*>(static_cast<float*>(a.out) + off);
#pragma unroll
    for (int i = 0; i < 4; ++i) op[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  }
}

// 3x3 stride-1 pad-1 convolution with halo tiles.
//
// A super-tile is `rows` output rows x `wt` output columns x `img` images
// (each row block = 128 pixels = one M=128 MMA).  The producer loads the input
// halo for a 64-channel block ONCE — (rows+2) input rows x (wt+2) columns x
// img images, 4-D box over dims (C, N, W, H) so that shared-memory row index
// = img + IMG*(w + (wt+2)*h) — and every one of the 9 taps is then a shifted
// window of that halo: tap (r,s) for output row j starts at shared row
// ((j+r)*(wt+2) + s)*IMG, always a multiple of 8 rows (IMG >= 8), so each
// window is a standard 1024-byte-aligned SW128 K-major operand.  Each weight
// tap (BN x 64) is loaded once and used by all `rows` MMAs.  Versus one TMA
// window per tap, this cuts L2->SM traffic about 3x for Cout <= 128.
__global__ void __launch_bounds__(HALO16_THREADS, 1) tc_conv_halo_kernel(const __grid_constant__ TmaMaps maps,
                                                                      const TcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int bst = a.stages;       // weight-tap ring depth
  const int hst = a.hstages;      // halo ring depth
  const uint32_t hbytes_al = (uint32_t)((a.halo_bytes + 1023) & ~1023);
  const uint32_t b_bytes = (uint32_t)a.block_n * BK * 2;
  uint8_t* sh = smem;
  uint8_t* sb = smem + (size_t)hst * hbytes_al;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sb + (size_t)bst * b_bytes);
  uint64_t* hfull = bars;
  uint64_t* hempty = hfull + hst;
  uint64_t* bfull = hempty + hst;
  uint64_t* bempty = bfull + bst;
  uint64_t* tfull = bempty + bst;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // output tiles (a.tma_out): 1 KB per epilogue warp, 1024-byte aligned after the barriers
  uint8_t* stg = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(abort_flag + 1) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr int R = 2;  // output rows per tile (the host sets a.rows = 2)
  const uint32_t tmem_cols = (uint32_t)(a.block_n * R * 2);
  const int WT2 = a.wt + 2;

  if (threadIdx.x == 0) {
    for (int i = 0; i < hst; ++i) {
      mbar_init(&hfull[i], 1);
      mbar_init(&hempty[i], 1);
    }
    for (int i = 0; i < bst; ++i) {
      mbar_init(&bfull[i], 1);
      mbar_init(&bempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 16);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.a[0])));
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.b)));
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Programmatic dependent launch: the prologue above (barriers, TMEM, tensor
  // maps, constant weights) may overlap the previous kernel's tail; every
  // activation read and every global write comes after it has completed.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // every CTA of this persistent grid is resident: the next kernel may launch
  // onto SMs as they free up (it waits on griddepcontrol before its activations)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    if (lane == 0) {
      int hs = 0, bs = 0;
      uint32_t hph = 0, bph = 0;
      if (a.bres) {
        // every (cin block, tap) weight tile once, into its own slot
        const int nk = 9 * a.cblocks;
        mbar_arrive_tx(&bfull[0], (uint32_t)nk * b_bytes);
        for (int kb = 0; kb < nk; ++kb)
          tma_load_2d(sb + (size_t)kb * b_bytes, &maps.b, &bfull[0], (kb % 9) * a.cin + (kb / 9) * BK, 0);
      }
      for (int t = blockIdx.x; t < a.n_tiles; t += gridDim.x) {
        const int nb = t % a.n_tiles_n;
        int pt = t / a.n_tiles_n;
        const int wb = pt % a.wblocks;
        pt /= a.wblocks;
        const int hb = pt % (a.ho / R);
        const int ib = pt / (a.ho / R);
        const int n0 = ib * a.img, w0 = wb * a.wt, h0 = hb * R;
        for (int cb = 0; cb < a.cblocks; ++cb) {
          if (!mbar_wait(&hempty[hs], hph ^ 1, abort_flag, 21)) goto producer_done;
          mbar_arrive_tx(&hfull[hs], (uint32_t)a.halo_bytes);
          tma_load_4d(sh + (size_t)hs * hbytes_al, &maps.a[0], &hfull[hs], cb * BK, n0, w0 - 1, h0 - 1);
          if (++hs == hst) { hs = 0; hph ^= 1; }
          for (int tap = 0; tap < 9 && !a.bres; ++tap) {
            if (!mbar_wait(&bempty[bs], bph ^ 1, abort_flag, 22)) goto producer_done;
            mbar_arrive_tx(&bfull[bs], b_bytes);
            tma_load_2d(sb + (size_t)bs * b_bytes, &maps.b, &bfull[bs], tap * a.cin + cb * BK, nb * a.block_n);
            if (++bs == bst) { bs = 0; bph ^= 1; }
          }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = instr_desc_h(BM, a.block_n, a.h16);
      const uint64_t bd0 = smem_desc(smem_u32(sb));
      int hs = 0, bs = 0, acc = 0;
      uint32_t hph = 0, bph = 0, acc_phase = 0;
      bool bres_ok = true;
      if (a.bres) {
        bres_ok = mbar_wait(&bfull[0], 0, abort_flag, 27);
        tc_fence_after();
      }
      for (int t = blockIdx.x; t < a.n_tiles && bres_ok; t += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, 23)) break;
        tc_fence_after();
        const uint32_t d0 = tmem_base + (uint32_t)(acc * R * a.block_n);
        bool ok = true;
        for (int cb = 0; cb < a.cblocks && ok; ++cb) {
          if (!mbar_wait(&hfull[hs], hph, abort_flag, 24)) { ok = false; break; }
          tc_fence_after();
          // descriptors: halo base + compile-time tap/row offsets (16-byte units)
          const uint64_t hd = smem_desc(smem_u32(sh + (size_t)hs * hbytes_al));
          const uint64_t sstep = (uint64_t)(a.img * 128) >> 4;
          const uint64_t rstep = (uint64_t)WT2 * sstep;
#pragma unroll
          for (int tap = 0; tap < 9; ++tap) {
            if (!a.bres) {
              if (!mbar_wait(&bfull[bs], bph, abort_flag, 25)) { ok = false; break; }
              tc_fence_after();
            }
            const int r = tap / 3, s = tap % 3;
            const uint64_t bd = bd0 + (uint64_t)(a.bres ? cb * 9 + tap : bs) * (b_bytes >> 4);
#pragma unroll
            for (int j = 0; j < R; ++j) {
              const uint64_t ad = hd + (uint64_t)(j + r) * rstep + (uint64_t)s * sstep;
#pragma unroll
              for (int k = 0; k < BK / 16; ++k)
                mma_bf16(d0 + (uint32_t)(j * a.block_n), ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc,
                         (cb > 0 || tap > 0 || k > 0) ? 1u : 0u);
            }
            if (!a.bres) {
              mma_commit(&bempty[bs]);
              if (++bs == bst) { bs = 0; bph ^= 1; }
            }
          }
          if (!ok) break;
          mma_commit(&hempty[hs]);
          if (++hs == hst) { hs = 0; hph ^= 1; }
        }
        if (!ok) break;
        mma_commit(&tfull[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
    }
  } else {
    // 8 epilogue warps: warp w reads TMEM lane quarter (w % 4) and one half of
    // the tile's columns.  Residual rows are prefetched into registers before
    // waiting for the accumulator, so their latency overlaps the MMAs.
    // 16 epilogue warps, four per TMEM lane quarter (warp % 4).  The tile's
    // (row, 32-column chunk) pairs of a quarter are dealt round-robin, so a
    // warp owns at most two chunks (Cout = 128) and prefetches both residual
    // chunks before the accumulator wait: no load latency after it.
    const int q = warp & 3;
    const int sub = (warp - 2) >> 2;  // 0..3
    const int nch = a.block_n >> 5;   // chunks per row: 2 or 4
    int jj[2], cc[2];
    bool own[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int idx = sub + 4 * u;
      own[u] = idx < R * nch;
      jj[u] = own[u] ? idx / nch : 0;
      cc[u] = own[u] ? idx % nch : 0;
    }
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < a.n_tiles; t += gridDim.x) {
      const int nb = t % a.n_tiles_n;
      int pt = t / a.n_tiles_n;
      const int wb = pt % a.wblocks;
      pt /= a.wblocks;
      const int hb = pt % (a.ho / R);
      const int ib = pt / (a.ho / R);
      const int m = q * 32 + lane;
      const int img = ib * a.img + (m % a.img);
      const int w = wb * a.wt + m / a.img;
      const bool img_ok = img < a.n_img;
      int64_t off[2];
#pragma unroll
      for (int u = 0; u < 2; ++u)
        off[u] = (((int64_t)img * a.ho + hb * R + jj[u]) * a.wo + w) * a.N + (int64_t)nb * a.block_n + cc[u] * 32;
      uint4 rv[2][4];
      if (a.res && img_ok) {
#pragma unroll
        for (int u = 0; u < 2; ++u)
          if (own[u]) {
            const uint4* rp = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.res) + off[u]);
#pragma unroll
            for (int i = 0; i < 4; ++i) rv[u][i] = rp[i];
          }
      }
      const bool ok = mbar_wait(&tfull[acc], acc_phase, abort_flag, 26);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (!own[u]) continue;
        const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) +
                            (uint32_t)((acc * R + jj[u]) * a.block_n + cc[u] * 32);
        // two 16-column halves keep the live set within the 96 registers a
        // thread gets at 576 threads per CTA
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float v[16];
          tmem_ld16(tb + h * 16, v);
          if (!img_ok && !a.tma_out) continue;
          const float4* bp = reinterpret_cast<const float4*>(a.bias + nb * a.block_n + cc[u] * 32 + h * 16);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 b = __ldg(bp + i);
            v[4 * i] += b.x; v[4 * i + 1] += b.y; v[4 * i + 2] += b.z; v[4 * i + 3] += b.w;
          }
          if (a.res) {
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              float rr[8];
              unpack8h(rv[u][2 * h + i], rr, a.h16);
#pragma unroll
              for (int e = 0; e < 8; ++e) v[8 * i + e] += rr[e];
            }
          }
          act_inplace<16>(v, a.act, true);
          if (a.tma_out) {
            // the warp's 32 pixels x 16 channels through its tile (32-byte
            // swizzle) and one TMA store; images past the batch are clipped
            uint8_t* tile = stg + (size_t)(warp - 2) * 1024;
            if (lane == 0) bulk_wait_read0();  // the previous store has read the tile
            __syncwarp();
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
              *reinterpret_cast<uint4*>(tile + lane * 32 + ((hh ^ ((lane >> 2) & 1)) << 4)) =
                  pack8h(v + 8 * hh, a.h16);
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
              tma_store_4d(&maps.out, tile, nb * a.block_n + cc[u] * 32 + h * 16, ib * a.img,
                           wb * a.wt + q * (32 / a.img), hb * R + jj[u]);
              bulk_commit();
            }
            continue;
          }
          uint4* op = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + off[u] + h * 16);
#pragma unroll
          for (int i = 0; i < 2; ++i) op[i] = pack8h(v + 8 * i, a.h16);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
    if (a.tma_out && lane == 0) bulk_wait0();
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {
    for (int i = 0; i < 1000; ++i) __nanosleep(1000);
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols));
  }
}

// 3x3 stride-1 convolution, Cin = 64 (one channel block), weights resident:
// row-ring variant of the halo kernel.  Work items are column strips of one
// image group (IMG images x WT output columns) split into segments of
// `seg_rows` output rows; a CTA walks a segment top to bottom two output rows
// at a time.  Input rows (IMG x (WT+2) pixels x 64 channels = one 128-byte
// swizzled row per pixel) live in a ring of `ring` shared-memory slots, so each
// input row is loaded once per segment instead of once per output row pair;
// every tap window of an MMA lies inside one slot (start (s*IMG) rows, a
// multiple of 8).
__global__ void __launch_bounds__(HALO_THREADS, 1) tc_conv_rowring_kernel(const __grid_constant__ TmaMaps maps,
                                                                         const TcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int NS = a.ring;
  const uint32_t rb_al = (uint32_t)((a.row_bytes + 1023) & ~1023);
  const uint32_t b_bytes = (uint32_t)a.block_n * BK * 2;
  uint8_t* sr = smem;
  uint8_t* sb = smem + (size_t)NS * rb_al;
  uint8_t* stg = sb + (size_t)9 * b_bytes;  // 8 epilogue warps x 2 rows x 2 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(stg + 8 * 4096);
  uint64_t* rfull = bars;
  uint64_t* rempty = rfull + NS;
  uint64_t* wfull = rempty + NS;
  uint64_t* tfull = wfull + 1;
  uint64_t* tempty = tfull + 2;
  uint64_t* resbar = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(resbar + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t tmem_cols = (uint32_t)(a.block_n * 4);  // 2 rows x 2 buffers
  const int SR = a.seg_rows;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&rfull[i], 1);
      mbar_init(&rempty[i], 1);
    }
    mbar_init(&wfull[0], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 8);
    }
    for (int i = 0; i < 8; ++i) mbar_init(&resbar[i], 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.a[0])));
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.b)));
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Programmatic dependent launch: the prologue above (barriers, TMEM, tensor
  // maps, constant weights) may overlap the previous kernel's tail; every
  // activation read and every global write comes after it has completed.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // every CTA of this persistent grid is resident: the next kernel may launch
  // onto SMs as they free up (it waits on griddepcontrol before its activations)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_tx(&wfull[0], 9u * b_bytes);
      // weight block order [W(2,s), W(1,s), W(0,s)] per column shift s, so that
      // W(r,s) followed by W(r-1,s) is one 128-row B operand
      for (int tap = 0; tap < 9; ++tap)
        tma_load_2d(sb + (size_t)((tap % 3) * 3 + 2 - tap / 3) * b_bytes, &maps.b, &wfull[0], tap * a.cin, 0);
      uint32_t c = 0;  // rows loaded so far
      const long long pt0 = a.prof ? clock64() : 0;
      long long pw = 0;
      for (int u = blockIdx.x; u < a.n_items; u += gridDim.x) {
        const int seg = u % a.segs;
        const int strip = u / a.segs;
        const int wb = strip % a.wblocks, ib = strip / a.wblocks;
        const int h0 = seg * SR;
        for (int ir = 0; ir < SR + 2; ++ir, ++c) {
          const int slot = (int)(c % NS);
          const long long w0 = a.prof ? clock64() : 0;
          if (!mbar_wait(&rempty[slot], ((c / NS) & 1) ^ 1, abort_flag, 31)) goto producer_done;
          if (a.prof) pw += clock64() - w0;
          mbar_arrive_tx(&rfull[slot], (uint32_t)a.row_bytes);
          tma_load_4d(sr + (size_t)slot * rb_al, &maps.a[0], &rfull[slot], 0, ib * a.img, wb * a.wt - 1,
                      h0 - 1 + ir);
        }
      }
    producer_done:
      if (a.prof) {
        atomicAdd(&a.prof[RP_PROD_TOTAL], (unsigned long long)(clock64() - pt0));
        atomicAdd(&a.prof[RP_PROD_EMPTY], (unsigned long long)pw);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc64 = instr_desc_h(BM, 64, a.h16), idesc128 = instr_desc_h(BM, 128, a.h16);
      const long long mt0 = a.prof ? clock64() : 0;
      long long m_rf = 0, m_te = 0, pairs = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      uint32_t cbase = 0;
      bool ok = mbar_wait(&wfull[0], 0, abort_flag, 32);
      tc_fence_after();
      for (int u = blockIdx.x; u < a.n_items && ok; u += gridDim.x) {
        for (int pr = 0; pr < SR / 2 && ok; ++pr) {
          // input rows 2pr .. 2pr+3 of this segment; the first pair waits for
          // all four, later pairs for the two new ones
          long long w0 = a.prof ? clock64() : 0;
          for (int ir = (pr == 0 ? 0 : 2 * pr + 2); ir <= 2 * pr + 3; ++ir) {
            const uint32_t c = cbase + ir;
            if (!mbar_wait(&rfull[c % NS], (c / NS) & 1, abort_flag, 33)) { ok = false; break; }
          }
          if (!ok) break;
          tc_fence_after();
          if (a.prof) { const long long t = clock64(); m_rf += t - w0; w0 = t; ++pairs; }
          if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, 34)) { ok = false; break; }
          tc_fence_after();
          if (a.prof) m_te += clock64() - w0;
          const uint32_t d0 = tmem_base + (uint32_t)(acc * 2 * a.block_n);
          // One thread issues all MMAs of the pair, so their operands are
          // precomputed descriptors plus compile-time offsets (the descriptor
          // address field is in 16-byte units).  Input row i of the pair feeds
          // output row 0 through tap r = i and output row 1 through r = i - 1:
          // rows 1 and 2 use one N=128 MMA with B = [W(i,s); W(i-1,s)] into both
          // accumulator halves; rows 0 and 3 use N=64 MMAs into one half and go
          // first, so that they initialise the accumulators.
          uint64_t arow[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) arow[i] = smem_desc(smem_u32(sr + (size_t)((cbase + 2 * pr + i) % NS) * rb_al));
          const uint64_t bd0 = smem_desc(smem_u32(sb));
          const uint64_t sstep = (uint64_t)(a.img * 128) >> 4;
          constexpr uint64_t WB = (64 * BK * 2) >> 4;  // one weight block
#pragma unroll
          for (int step = 0; step < 4; ++step) {
            const int i = step == 0 ? 0 : step == 1 ? 3 : step - 1;  // 0, 3, 1, 2
#pragma unroll
            for (int s = 0; s < 3; ++s) {
              const uint64_t ad = arow[i] + (uint64_t)s * sstep;
              // block of W(r,s) is s*3 + 2 - r
              const int r_top = i == 3 ? 2 : i;
              const uint64_t bd = bd0 + (uint64_t)(s * 3 + 2 - r_top) * WB;
              const uint32_t d = d0 + (i == 3 ? 64u : 0u);
              const uint32_t id = (i == 0 || i == 3) ? idesc64 : idesc128;
#pragma unroll
              for (int k = 0; k < BK / 16; ++k)
                mma_bf16(d, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), id, (step > 1 || s > 0 || k > 0) ? 1u : 0u);
            }
          }
          mma_commit(&tfull[acc]);
          if (++acc == 2) { acc = 0; acc_phase ^= 1; }
          // rows 2pr and 2pr+1 are no longer needed (all rows at segment end)
          const int rel_end = (pr == SR / 2 - 1) ? SR + 2 : 2 * pr + 2;
          for (int ir = 2 * pr; ir < rel_end; ++ir) mma_commit(&rempty[(cbase + ir) % NS]);
        }
        cbase += SR + 2;
      }
      if (a.prof) {
        atomicAdd(&a.prof[RP_MMA_TOTAL], (unsigned long long)(clock64() - mt0));
        atomicAdd(&a.prof[RP_MMA_RFULL], (unsigned long long)m_rf);
        atomicAdd(&a.prof[RP_MMA_TEMPTY], (unsigned long long)m_te);
        atomicAdd(&a.prof[RP_PAIRS], (unsigned long long)pairs);
      }
    }
  } else if (!a.res) {
    // Epilogue without a residual: direct 16-byte stores from registers.
    // (Measured ~4% faster than the staged tiles below, which leave shared
    // memory bandwidth to the MMAs; with a residual the staged path is 23%
    // faster because the residual arrives in whole rows.)
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int cols = a.block_n >> 1;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool run = true;
    const long long et0 = a.prof ? clock64() : 0;
    long long e_tf = 0;
    for (int u = blockIdx.x; u < a.n_items && run; u += gridDim.x) {
      const int seg = u % a.segs;
      const int strip = u / a.segs;
      const int wb = strip % a.wblocks, ib = strip / a.wblocks;
      const int m = q * 32 + lane;
      const int img = ib * a.img + (m % a.img);
      const int w = wb * a.wt + m / a.img;
      const bool img_ok = img < a.n_img;
      const int64_t col_base = half * cols;
      for (int pr = 0; pr < SR / 2; ++pr) {
        const int hrow = seg * SR + 2 * pr;
        const long long w0 = a.prof ? clock64() : 0;
        const bool ok = mbar_wait(&tfull[acc], acc_phase, abort_flag, 35);
        if (!__all_sync(0xffffffffu, ok)) { run = false; break; }
        tc_fence_after();
        if (a.prof) e_tf += clock64() - w0;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int64_t pix = ((int64_t)img * a.ho + hrow + j) * a.wo + w;
          const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) +
                              (uint32_t)((acc * 2 + j) * a.block_n + half * cols);
          float v[32];
          tmem_ld32(tb, v);
          if (img_ok) store32_bf16(a, pix * a.N + col_base, col_base, v, nullptr);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
    }
    if (a.prof && lane == 0) {
      atomicAdd(&a.prof[RP_EPI_TOTAL], (unsigned long long)(clock64() - et0));
      atomicAdd(&a.prof[RP_EPI_TFULL], (unsigned long long)e_tf);
    }

  } else {
    // Epilogue: warp (q, half) owns TMEM lanes 32q..32q+31 (pixels) and
    // channels 32*half..+31 of both output rows.  Its residual rows arrive by
    // TMA into a private 2 x 2 KB tile; results overwrite the tile in place and
    // leave by TMA store, so global traffic is whole 64-byte rows instead of
    // one 16-byte piece per lane per instruction.
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int ew = warp - 2;
    uint8_t* tile = stg + (size_t)ew * 4096;
    uint64_t* rbar = &resbar[ew];
    uint32_t rphase = 0;
    const int pw = 32 / a.img;  // output columns per warp
    int acc = 0;
    uint32_t acc_phase = 0;
    bool run = true;
    float bias[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) bias[i] = a.bias ? __ldg(a.bias + half * 32 + i) : 0.f;
    const long long et0 = a.prof ? clock64() : 0;
    long long e_tf = 0, e_rs = 0;
    for (int u = blockIdx.x; u < a.n_items && run; u += gridDim.x) {
      const int seg = u % a.segs;
      const int strip = u / a.segs;
      const int wb = strip % a.wblocks, ib = strip / a.wblocks;
      const int img0 = ib * a.img;
      const int w0 = wb * a.wt + q * pw;
      for (int pr = 0; pr < SR / 2; ++pr) {
        const int hrow = seg * SR + 2 * pr;
        if (lane == 0) {
          bulk_wait_read0();  // the previous stores have left the tile
          if (a.res) {
            mbar_arrive_tx(rbar, 4096);
            tma_load_4d(tile, &maps.res, rbar, half * 32, img0, w0, hrow);
            tma_load_4d(tile + 2048, &maps.res, rbar, half * 32, img0, w0, hrow + 1);
          }
        }
        long long tw = a.prof ? clock64() : 0;
        const bool ok = mbar_wait(&tfull[acc], acc_phase, abort_flag, 35);
        if (!__all_sync(0xffffffffu, ok)) { run = false; break; }
        tc_fence_after();
        if (a.prof) { const long long t = clock64(); e_tf += t - tw; tw = t; }
        float v[2][32];
#pragma unroll
        for (int j = 0; j < 2; ++j)
          tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)((acc * 2 + j) * a.block_n + half * 32), v[j]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        if (a.res) {
          const bool rok = mbar_wait(rbar, rphase, abort_flag, 36);
          rphase ^= 1;
          if (!__all_sync(0xffffffffu, rok)) { run = false; break; }
          if (a.prof) e_rs += clock64() - tw;
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          uint8_t* trow = tile + j * 2048;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint4* cp = reinterpret_cast<uint4*>(trow + swz64(lane, c));
            float x[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) x[e] = v[j][c * 8 + e] + bias[c * 8 + e];
            if (a.res) {
              float rr[8];
              unpack8h(*cp, rr, a.h16);
#pragma unroll
              for (int e = 0; e < 8; ++e) x[e] += rr[e];
            }
            act_inplace<8>(x, a.act, true);
            *cp = pack8h(x, a.h16);
          }
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          tma_store_4d(&maps.out, tile, half * 32, img0, w0, hrow);
          tma_store_4d(&maps.out, tile + 2048, half * 32, img0, w0, hrow + 1);
          bulk_commit();
        }
      }
    }
    if (lane == 0) bulk_wait0();
    if (a.prof && lane == 0) {
      atomicAdd(&a.prof[RP_EPI_TOTAL], (unsigned long long)(clock64() - et0));
      atomicAdd(&a.prof[RP_EPI_TFULL], (unsigned long long)e_tf);
      atomicAdd(&a.prof[RP_EPI_RES], (unsigned long long)e_rs);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {
    for (int i = 0; i < 1000; ++i) __nanosleep(1000);
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols));
  }
}

// 3x3 stride-1 convolution, Cin = Cout = 64, weights resident: sliding-window
// variant of the row-ring kernel.  The input-row ring and work items are the
// row ring's, but the accumulators are a ring of NB output rows in TMEM
// (64 columns each).  Input row i of a segment feeds output rows i-2, i-1, i
// through taps r = 2, 1, 0; with the weights stored [W(2,s), W(1,s), W(0,s)]
// per column shift s, those three are one N=192 MMA per (s, K step) whose
// accumulator columns are three consecutive ring blocks: 12 MMAs per output
// row (two where the three blocks wrap around the ring, and fewer at segment
// ends).  Every MMA accumulates; the epilogue zeroes a block after draining it
// (and all blocks at start), which is what lets one instruction start one
// output row while it continues two others.
// Accumulator ring: SLIDE_NL output-row blocks of 64 TMEM columns.  A window
// of three rows that wraps around the ring is issued as two MMAs (N=128 +
// N=64), so every output row accumulates in one block and its result does not
// depend on where the ring stands.  (Aliasing blocks 0 and 1 into two spare
// blocks, which kept every window one MMA, split those rows' sums in two and
// made their bits depend on the schedule, i.e. on the batch size.)
constexpr int SLIDE_NL = 8;
constexpr int SLIDE_NPHYS = 8;
constexpr int SLIDE_THREADS = 320;  // producer, MMA, 8 epilogue warps

__global__ void __launch_bounds__(SLIDE_THREADS, 1) tc_conv_rowslide_kernel(const __grid_constant__ TmaMaps maps,
                                                                          const TcArgs a) {
  constexpr int NB = SLIDE_NL;        // accumulator blocks (one output row each)
  constexpr int NPHYS = SLIDE_NPHYS;  // TMEM blocks allocated
  static_assert(NPHYS == NB, "every row accumulates in its own block");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int NS = a.ring;
  const uint32_t rb_al = (uint32_t)((a.row_bytes + 1023) & ~1023);
  constexpr uint32_t b_bytes = 64u * BK * 2;
  uint8_t* sr = smem;
  uint8_t* sb = smem + (size_t)NS * rb_al;
  // residual layers: every epilogue warp stages its own residual box (32
  // channels x its 32 pixels, 2 KB) by TMA in two tiles, adds it in place,
  // writes the output over it and TMA-stores the tile
  const bool has_res = a.rring == 1;
  const bool tiles_out = a.rring != 0;     // output through the per-warp tiles and TMA stores
  uint8_t* rs = sb + (size_t)9 * b_bytes;  // 8 epilogue warps x 2 x 2 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(rs + (tiles_out ? 8 * 4096 : 0));
  uint64_t* rfull = bars;
  uint64_t* rempty = rfull + NS;
  uint64_t* wfull = rempty + NS;
  uint64_t* tfull = wfull + 1;
  uint64_t* tempty = tfull + NB;
  uint64_t* rbar = tempty + NB;  // residual tile landed: 2 per epilogue warp
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr uint32_t tmem_cols = 64u * NPHYS;
  const int SR = a.seg_rows;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&rfull[i], 1);
      mbar_init(&rempty[i], 1);
    }
    mbar_init(&wfull[0], 1);
    for (int i = 0; i < NB; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 8);
    }
    for (int i = 0; i < 16; ++i) mbar_init(&rbar[i], 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.a[0])));
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.b)));
    if (has_res) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.res)));
    if (tiles_out) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.out)));
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (warp == 0 && lane == 0) {
    // the 9 weight taps are constants: loaded before the dependency wait
    mbar_arrive_tx(&wfull[0], 9u * b_bytes);
    for (int tap = 0; tap < 9; ++tap)
      tma_load_2d(sb + (size_t)((tap % 3) * 3 + 2 - tap / 3) * b_bytes, &maps.b, &wfull[0], tap * a.cin, 0);
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // every CTA of this persistent grid is resident: the next kernel may launch
  // onto SMs as they free up (it waits on griddepcontrol before its activations)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    if (lane == 0) {
      uint32_t c = 0;
      const long long pt0 = a.prof ? clock64() : 0;
      long long pw = 0;
      for (int u = blockIdx.x; u < a.n_items; u += gridDim.x) {
        const int seg = u % a.segs;
        const int strip = u / a.segs;
        const int wb = strip % a.wblocks, ib = strip / a.wblocks;
        const int h0 = seg * SR;
        for (int ir = 0; ir < SR + 2; ++ir, ++c) {
          const int slot = (int)(c % NS);
          const long long t0 = a.prof ? clock64() : 0;
          if (!mbar_wait(&rempty[slot], ((c / NS) & 1) ^ 1, abort_flag, 41)) goto producer_done;
          if (a.prof) pw += clock64() - t0;
          mbar_arrive_tx(&rfull[slot], (uint32_t)a.row_bytes);
          tma_load_4d(sr + (size_t)slot * rb_al, &maps.a[0], &rfull[slot], 0, ib * a.img, wb * a.wt - 1,
                      h0 - 1 + ir);
        }
      }
    producer_done:
      if (a.prof) {
        atomicAdd(&a.prof[RP_PROD_TOTAL], (unsigned long long)(clock64() - pt0));
        atomicAdd(&a.prof[RP_PROD_EMPTY], (unsigned long long)pw);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc64 = instr_desc_h(BM, 64, a.h16), idesc128 = instr_desc_h(BM, 128, a.h16),
                     idesc192 = instr_desc_h(BM, 192, a.h16);
      const long long mt0 = a.prof ? clock64() : 0;
      long long m_rf = 0, m_te = 0, rows = 0;
      bool ok = mbar_wait(&wfull[0], 0, abort_flag, 42);
      tc_fence_after();
      const uint64_t bd0 = smem_desc(smem_u32(sb));
      const uint64_t sstep = (uint64_t)(a.img * 128) >> 4;
      constexpr uint64_t WB = (64 * BK * 2) >> 4;  // one weight block, 16-byte units
      uint32_t G = 0;  // output rows started so far (ring position)
      uint32_t c = 0;  // input rows consumed so far
      for (int u = blockIdx.x; u < a.n_items && ok; u += gridDim.x) {
        for (int i = 0; i < SR + 2; ++i, ++c) {
          const int slot = (int)(c % NS);
          long long t0 = a.prof ? clock64() : 0;
          if (!mbar_wait(&rfull[slot], (c / NS) & 1, abort_flag, 43)) { ok = false; break; }
          if (a.prof) { const long long t = clock64(); m_rf += t - t0; t0 = t; }
          if (i < SR) {
            // output row i starts here: its block must have been drained and zeroed
            const uint32_t gi = G + (uint32_t)i;
            if (!mbar_wait(&tempty[gi % NB], (gi / NB) & 1, abort_flag, 44)) { ok = false; break; }
            if (a.prof) { m_te += clock64() - t0; ++rows; }
          }
          tc_fence_after();
          const int j0 = i >= 2 ? i - 2 : 0;
          const int j1 = i < SR ? i : SR - 1;
          const int cnt = j1 - j0 + 1;
          const int b0 = (int)((G + (uint32_t)j0) % NB);
          const int n1 = cnt < NB - b0 ? cnt : NB - b0;  // blocks before the ring wraps
          const int n2 = cnt - n1;
          const int r0 = i - j0;  // tap row of block j0; the next blocks take r0-1, r0-2
          const uint64_t ad = smem_desc(smem_u32(sr + (size_t)slot * rb_al));
          const uint64_t bd = bd0 + (uint64_t)(2 - r0) * WB;
          const uint32_t d1 = tmem_base + (uint32_t)(b0 * 64);
          const uint32_t id1 = n1 == 3 ? idesc192 : n1 == 2 ? idesc128 : idesc64;
          if (n2 == 0) {
#pragma unroll
            for (int s = 0; s < 3; ++s)
#pragma unroll
              for (int k = 0; k < BK / 16; ++k)
                mma_bf16(d1, ad + (uint64_t)s * sstep + (uint64_t)(2 * k), bd + (uint64_t)(s * 3) * WB + (uint64_t)(2 * k),
                         id1, 1u);
          } else {
            const uint32_t id2 = n2 == 2 ? idesc128 : idesc64;
            const uint64_t bd2 = bd + (uint64_t)n1 * WB;
#pragma unroll
            for (int s = 0; s < 3; ++s)
#pragma unroll
              for (int k = 0; k < BK / 16; ++k) {
                const uint64_t aa = ad + (uint64_t)s * sstep + (uint64_t)(2 * k);
                mma_bf16(d1, aa, bd + (uint64_t)(s * 3) * WB + (uint64_t)(2 * k), id1, 1u);
                mma_bf16(tmem_base, aa, bd2 + (uint64_t)(s * 3) * WB + (uint64_t)(2 * k), id2, 1u);
              }
          }
          mma_commit(&rempty[slot]);
          if (i >= 2) mma_commit(&tfull[(G + (uint32_t)(i - 2)) % NB]);
        }
        G += (uint32_t)SR;
      }
      if (a.prof) {
        atomicAdd(&a.prof[RP_MMA_TOTAL], (unsigned long long)(clock64() - mt0));
        atomicAdd(&a.prof[RP_MMA_RFULL], (unsigned long long)m_rf);
        atomicAdd(&a.prof[RP_MMA_TEMPTY], (unsigned long long)m_te);
        atomicAdd(&a.prof[RP_PAIRS], (unsigned long long)rows);
      }
    }
  } else {
    // Epilogue: warp (q, half) owns TMEM lanes 32q..32q+31 (pixels) and
    // channels 32*half..+31 of every output row.  It drains a block, zeroes
    // it, finishes the row from registers (+bias, +residual from the staged
    // ring, activation, 64-byte stores) and then hands the block back.
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int col0 = half * 32;
    const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)col0;
#pragma unroll 1
    for (int b = 0; b < NPHYS; ++b) tmem_st32_zero(lane_base + (uint32_t)(b * 64));
    tmem_st_wait();
    tc_fence_before();
    __syncwarp();
    if (lane == 0)
      for (int b = 0; b < NB; ++b) mbar_arrive(&tempty[b]);
    float bias[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) bias[i] = a.bias ? __ldg(a.bias + col0 + i) : 0.f;
    uint16_t* out = static_cast<uint16_t*>(a.out);
    const long long et0 = a.prof ? clock64() : 0;
    long long e_tf = 0;
    uint32_t G = 0;
    bool run = true;
    const int ew = warp - 2;
    uint8_t* tiles = rs + (size_t)ew * 4096;
    uint64_t* mybar = rbar + 2 * ew;
    const int pw = 32 / a.img;  // output columns per warp
    // TMA coordinates (channel, image, column, row) of this warp's box of
    // output row j of item u
    auto box = [&](int u, int j, int* c) {
      const int seg = u % a.segs;
      const int strip = u / a.segs;
      const int wb = strip % a.wblocks, ib = strip / a.wblocks;
      c[0] = half * 32;
      c[1] = ib * a.img;
      c[2] = wb * a.wt + q * pw;
      c[3] = seg * SR + j;
    };
    if (has_res && lane == 0 && (int)blockIdx.x < a.n_items) {
      int c[4];
      box(blockIdx.x, 0, c);
      mbar_arrive_tx(&mybar[0], 2048);
      tma_load_4d(tiles, &maps.res, &mybar[0], c[0], c[1], c[2], c[3]);
    }
    uint32_t g = 0;  // rows this warp has finished (residual tiles alternate)
    for (int u = blockIdx.x; u < a.n_items && run; u += gridDim.x) {
      const int seg = u % a.segs;
      const int strip = u / a.segs;
      const int wb = strip % a.wblocks, ib = strip / a.wblocks;
      const int m = q * 32 + lane;
      const int img = ib * a.img + (m % a.img);
      const int w = wb * a.wt + m / a.img;
      const bool img_ok = img < a.n_img;
      const int64_t pix0 = ((int64_t)img * a.ho + seg * SR) * a.wo + w;  // output row 0 of the segment
      for (int j = 0; j < SR; ++j, ++g) {
        const uint32_t gj = G + (uint32_t)j;
        const uint32_t blk = gj % NB;
        const uint32_t tl = g & 1;
        if (has_res && lane == 0) {
          // the next row's residual into the other tile, once the store that
          // last used that tile has read it
          const int nu = j + 1 < SR ? u : u + (int)gridDim.x;
          if (nu < a.n_items) {
            // (every residual row is loaded; this also runs only for residual layers)
            int c[4];
            box(nu, j + 1 < SR ? j + 1 : 0, c);
            bulk_wait_read0();
            mbar_arrive_tx(&mybar[tl ^ 1], 2048);
            tma_load_4d(tiles + (tl ^ 1) * 2048, &maps.res, &mybar[tl ^ 1], c[0], c[1], c[2], c[3]);
          }
        }
        const long long t0 = a.prof ? clock64() : 0;
        const bool ok = mbar_wait(&tfull[blk], (gj / NB) & 1, abort_flag, 45);
        if (!__all_sync(0xffffffffu, ok)) { run = false; break; }
        tc_fence_after();
        if (a.prof) e_tf += clock64() - t0;
        float v[32];
        tmem_ld32(lane_base + blk * 64, v);
        tmem_st32_zero(lane_base + blk * 64);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[blk]);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += bias[i];
        if (tiles_out) {
          uint8_t* tile = tiles + tl * 2048;
          if (has_res) {
            const bool rok = mbar_wait(&mybar[tl], (g >> 1) & 1, abort_flag, 47);
            if (!__all_sync(0xffffffffu, rok)) { run = false; break; }
          } else {
            if (lane == 0) bulk_wait_read1();  // the store two rows back has read this tile
            __syncwarp();
          }
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint4* cp = reinterpret_cast<uint4*>(tile + swz64(lane, c));
            if (has_res) {
              float rr[8];
              unpack8h(*cp, rr, a.h16);
#pragma unroll
              for (int e = 0; e < 8; ++e) v[8 * c + e] += rr[e];
            }
            act_inplace<8>(v + 8 * c, a.act, true);
            *cp = pack8h(v + 8 * c, a.h16);
          }
          // one proxy fence orders both the residual reads (before the tile's
          // next TMA load) and the result writes (before this TMA store)
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            int c[4];
            box(u, j, c);
            tma_store_4d(&maps.out, tile, c[0], c[1], c[2], c[3]);
            bulk_commit();
          }
        } else if (img_ok) {
          act_inplace<32>(v, a.act, true);
          const int64_t off = (pix0 + (int64_t)j * a.wo) * 64 + col0;
          uint4* op = reinterpret_cast<uint4*>(out + off);
#pragma unroll
          for (int i = 0; i < 4; ++i) op[i] = pack8h(v + 8 * i, a.h16);
        }
      }
      G += (uint32_t)SR;
    }
    if (tiles_out && lane == 0) bulk_wait0();
    tmem_st_wait();  // (an aborted row may leave its zeroing store unwaited)
    if (a.prof && lane == 0) {
      atomicAdd(&a.prof[RP_EPI_TOTAL], (unsigned long long)(clock64() - et0));
      atomicAdd(&a.prof[RP_EPI_TFULL], (unsigned long long)e_tf);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {
    for (int i = 0; i < 1000; ++i) __nanosleep(1000);
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols));
  }
}

// Stem convolution on tcgen05: NCHW f32 input with Cin*kh*kw <= 32, 64 output
// channels, NHWC bf16 output = act(conv + bias).  Persistent CTAs walk tiles of
// 128 consecutive output pixels.  Warps 0-7, in two groups taking alternate
// tiles, gather a tile's patch rows (one pixel per lane, lanes on consecutive
// pixels so the NCHW loads coalesce) as bf16 K values 0..31 of a 128-byte
// swizzled row; warp 12 issues two M=128,
// N=64, K=16 MMAs per tile against the weights, resident in shared memory as
// a [64][K] K-major operand; warps 8-11 drain their TMEM lane quarter, add
// bias, apply the activation and TMA-store 32 pixels x 128 bytes.  Patch
// tiles (4 stages) and accumulators (2 x 64 columns) are double-buffered.
constexpr int STEM_THREADS = 416;  // 8 gather warps, 4 epilogue warps, 1 MMA warp
constexpr int STEM_STAGES = 4;

// IMG = true (3x3, stride 1, pad 1, W = 32, C <= 3, C*H*W*4 <= 12 KB): work is
// whole images.  Warp 17 TMA-loads each image (NCHW f32, 12 KB) into a ring of
// STEM_IMGS shared-memory slots, and the gather warps build the patch tiles of
// its H*W/128 tiles from shared memory (no global loads on the gather path);
// HBM then sees one read of the input and one write of the output.
constexpr int STEM_IMGS = 3;
constexpr int STEM_IMG_BYTES = 12288;

// IMG: warps 0-7 gather, 8-15 epilogue (two per TMEM lane quarter, 32
// channels each), 16 MMA, 17 image loads; otherwise warps 0-7 gather, 8-11
// epilogue (64 channels each), 12 MMA.
constexpr int STEM_IMG_THREADS = 576;

template <bool IMG>
__global__ void __launch_bounds__(IMG ? STEM_IMG_THREADS : STEM_THREADS, 1)
    tc_stem_kernel(const __grid_constant__ TmaMaps maps, const float* __restrict__ x, const float* __restrict__ wt,
                   const float* __restrict__ bias, c3b_stem_params g, int act, int64_t M, int n_tiles, int h16,
                   unsigned long long* prof) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;                                   // STEM_STAGES x 16 KB patch tiles
  uint8_t* sbw = sa + STEM_STAGES * 16384;              // weights [64][64] bf16, 8 KB
  constexpr int EPI = IMG ? 8 : 4;                      // epilogue warps
  constexpr int NACC = IMG ? 4 : 2;                     // TMEM accumulators (64 columns each)
  constexpr int NG = IMG ? 2 : 1;                       // epilogue groups taking alternate tiles
  constexpr int MMA_WARP = IMG ? 16 : 12;
  uint8_t* so = sbw + 8192;                             // EPI epilogue warps x 4 KB output tiles
  float* simg = reinterpret_cast<float*>(so + EPI * 4096);  // IMG: STEM_IMGS image slots (1024-byte aligned)
  int4* ktab = reinterpret_cast<int4*>(reinterpret_cast<uint8_t*>(simg) + (IMG ? STEM_IMGS * STEM_IMG_BYTES : 0));
  uint64_t* bars = reinterpret_cast<uint64_t*>(ktab + 32);  // ktab: per K index input offset, row / col step, valid
  uint64_t* afull = bars;
  uint64_t* aempty = afull + STEM_STAGES;
  uint64_t* tfull = aempty + STEM_STAGES;
  uint64_t* tempty = tfull + NACC;
  uint64_t* ifull = tempty + NACC;     // IMG: image slot loaded
  uint64_t* iempty = ifull + STEM_IMGS;  // IMG: image slot gathered (4 arrivals per tile)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(iempty + STEM_IMGS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = g.c * g.g.kh * g.g.kw;

  // weights -> B operand: row n (output channel), K-major, zero beyond K
  for (int i = threadIdx.x; i < 64 * 8; i += STEM_THREADS) {
    const int n = i >> 3, c = i & 7;  // 16-byte chunk c = K elements 8c..8c+7
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k0 = c * 8 + 2 * j;
      o[j] = pack2h(make_float2(k0 < K ? wt[k0 * 64 + n] : 0.f, k0 + 1 < K ? wt[(k0 + 1) * 64 + n] : 0.f), h16);
    }
    *reinterpret_cast<uint4*>(sbw + n * 128 + ((c ^ (n & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  if (threadIdx.x < 32) {
    const int k = threadIdx.x;
    const int KHW0 = g.g.kh * g.g.kw;
    const int c = k / KHW0, rr = (k / g.g.kw) % g.g.kh, ss = k % g.g.kw;
    ktab[k] = k < K ? make_int4((c * g.h + rr * g.g.dh) * g.w + ss * g.g.dw, rr * g.g.dh, ss * g.g.dw, 1)
                    : make_int4(0, 0, 0, 0);
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < STEM_STAGES; ++i) {
      mbar_init(&afull[i], 4);
      mbar_init(&aempty[i], 1);
    }
    for (int i = 0; i < NACC; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], EPI / NG);
    }
    if (IMG) {
      const int tpi = g.ho * g.wo / 128;
      for (int i = 0; i < STEM_IMGS; ++i) {
        mbar_init(&ifull[i], 1);
        mbar_init(&iempty[i], 4 * tpi);
      }
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  fence_proxy_async();  // the weight rows are read by the MMA (async proxy)
  if (warp == MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(NACC * 64));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Programmatic dependent launch: the prologue above (barriers, TMEM, tensor
  // maps, constant weights) may overlap the previous kernel's tail; every
  // activation read and every global write comes after it has completed.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // every CTA of this persistent grid is resident: the next kernel may launch
  // onto SMs as they free up (it waits on griddepcontrol before its activations)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int HW = g.ho * g.wo;
  long long pc[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // wait profiler (prof != null), per thread
  // IMG: the CTA's i-th tile is tile i % tpi of its (i / tpi)-th image
  const int tpi = HW / 128;
  auto tile_of = [&](int i) -> int {
    if (!IMG) return blockIdx.x + i * gridDim.x;
    const int u = blockIdx.x + (i / tpi) * gridDim.x;
    return u < g.n ? u * tpi + i % tpi : n_tiles;
  };

  if (warp < 8) {
    // ---------------- patch gather: two groups of 4 warps take alternate
    // tiles (two tiles' loads in flight); row r of a tile = one output pixel
    const int grp = warp >> 2;
    const int r = (warp & 3) * 32 + lane;
    for (int i = grp;; i += 2) {
      const int t = tile_of(i);
      if (t >= n_tiles) break;
      const int stage = i % STEM_STAGES;
      const uint32_t phase = (uint32_t)(i / STEM_STAGES) & 1u;
      long long pt0 = prof ? clock64() : 0;
      if (!mbar_wait(&aempty[stage], phase ^ 1, abort_flag, 51)) break;
      if (prof) { const long long t1 = clock64(); pc[0] += t1 - pt0; pt0 = t1; }
      const int64_t m = (int64_t)t * 128 + r;
      float v[32];
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = 0.f;
      if (IMG) {
        const int j = i / tpi, slot = j % STEM_IMGS;
        if (!mbar_wait(&ifull[slot], (uint32_t)(j / STEM_IMGS) & 1u, abort_flag, 55)) break;
        if (prof) { const long long t1 = clock64(); pc[1] += t1 - pt0; pt0 = t1; }
        const int oh = (i % tpi) * 4 + (r >> 5), ow = r & 31;
        const float* sp = simg + slot * (STEM_IMG_BYTES / 4) + (oh - 1) * 32 + ow - 1;
        bool rok[3], cok[3];
#pragma unroll
        for (int q = 0; q < 3; ++q) {
          rok[q] = oh - 1 + q >= 0 && oh - 1 + q < g.h;
          cok[q] = ow - 1 + q >= 0 && ow - 1 + q < 32;
        }
        const int hw = g.h * 32;
#pragma unroll
        for (int c = 0; c < 3; ++c)
          if (c < g.c) {
#pragma unroll
            for (int rr = 0; rr < 3; ++rr)
#pragma unroll
              for (int q = 0; q < 3; ++q)
                if (rok[rr] && cok[q]) v[c * 9 + rr * 3 + q] = sp[c * hw + rr * 32 + q];
          }
        fence_proxy_async();  // generic reads of the slot before its next TMA refill
        __syncwarp();
        if (lane == 0) mbar_arrive(&iempty[slot]);
      } else if (m < M) {
        const int img = (int)(m / HW), rem = (int)(m % HW);
        const int oh = rem / g.wo, ow = rem % g.wo;
        const int ih0 = oh * g.g.sh - g.g.ph0, iw0 = ow * g.g.sw - g.g.pw0;
        const float* xb = x + (int64_t)img * g.c * g.h * g.w + (int64_t)ih0 * g.w + iw0;
        if (g.g.kh == 3 && g.g.kw == 3 && g.g.dh == 1 && g.g.dw == 1) {
          // 3x3, dilation 1 (C <= 3): three row and three column flags per
          // pixel, then one predicated load per element at a fixed offset
          bool rok[3], cok[3];
#pragma unroll
          for (int i = 0; i < 3; ++i) {
            rok[i] = ih0 + i >= 0 && ih0 + i < g.h;
            cok[i] = iw0 + i >= 0 && iw0 + i < g.w;
          }
          const int64_t hw = (int64_t)g.h * g.w;
#pragma unroll
          for (int c = 0; c < 3; ++c) {
            if (c < g.c) {
#pragma unroll
              for (int r = 0; r < 3; ++r)
#pragma unroll
                for (int q = 0; q < 3; ++q)
                  if (rok[r] && cok[q]) v[c * 9 + r * 3 + q] = __ldg(xb + c * hw + r * g.w + q);
            }
          }
        } else {
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            const int4 e = ktab[k];  // broadcast read
            const int ih = ih0 + e.y, iw = iw0 + e.z;
            if (e.w && ih >= 0 && ih < g.h && iw >= 0 && iw < g.w) v[k] = __ldg(xb + e.x);
          }
        }
      }
      uint8_t* row = sa + (size_t)stage * 16384 + r * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) << 4)) = pack8h(v + c * 8, h16);
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[stage]);
      if (prof) pc[2] += clock64() - pt0;
    }
  } else if (warp < 8 + EPI) {
    // ---------------- epilogue: TMEM lane quarter q = warp % 4, all 64
    // channels of its 32 pixels.  IMG: two groups of 4 warps take alternate
    // tiles (two tiles drain at once, four accumulators), each in two
    // 32-channel passes with 64-byte-swizzled halves of its 4 KB tile.
    const int q = warp & 3;
    const int grp = (warp - 8) >> 2;
    constexpr int NC = IMG ? 32 : 64;
    uint8_t* tile = so + (size_t)(warp - 8) * 4096;
    for (int i = grp;; i += NG) {
      const int acc = i % NACC;
      const uint32_t acc_phase = (uint32_t)(i / NACC) & 1u;
      const int t = tile_of(i);
      if (t >= n_tiles) break;
      long long pt0 = prof ? clock64() : 0;
      const bool ok = mbar_wait(&tfull[acc], acc_phase, abort_flag, 52);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      if (prof) { const long long t1 = clock64(); pc[3] += t1 - pt0; pt0 = t1; }
      if (IMG) {
        if (lane == 0) bulk_wait_read0();  // the previous stores have read the tile
        __syncwarp();
        // four 16-channel chunks; chunk c+1's TMEM load is in flight while
        // chunk c is finished (the wait names the registers it fills)
        const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * 64);
        uint32_t ra[16], rb[16];
        tmem_ld16_nowait(tb, ra);
        tmem_wait_ld16(ra);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t* cur = (c & 1) ? rb : ra;
          uint32_t* nxt = (c & 1) ? ra : rb;
          if (c < 3) tmem_ld16_nowait(tb + (uint32_t)(16 * (c + 1)), nxt);
          float v[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(cur[j]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float4 b = __ldg(reinterpret_cast<const float4*>(bias) + c * 4 + j);
            v[4 * j] += b.x; v[4 * j + 1] += b.y; v[4 * j + 2] += b.z; v[4 * j + 3] += b.w;
          }
          act_inplace<16>(v, act, true);
          // chunk c = 16-byte pieces 2(c&1), 2(c&1)+1 of half-tile c>>1
#pragma unroll
          for (int e = 0; e < 2; ++e)
            *reinterpret_cast<uint4*>(tile + (c >> 1) * 2048 + swz64(lane, 2 * (c & 1) + e)) = pack8h(v + e * 8, h16);
          if (c < 3) {
            tmem_wait_ld16(nxt);
          } else {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
          }
        }
        if (prof) { const long long t1 = clock64(); pc[4] += t1 - pt0; pt0 = t1; }
        fence_proxy_async();
        __syncwarp();
        const int64_t row0 = (int64_t)t * 128 + q * 32;
        if (lane == 0 && row0 < M) {
          // maps.b: the output with 32-channel, 64-byte-swizzled boxes
          tma_store_2d(&maps.b, tile, 0, (int)row0);
          tma_store_2d(&maps.b, tile + 2048, 32, (int)row0);
          bulk_commit();
        }
        if (prof) { pc[6] += clock64() - pt0; pc[7] += 1; }
        continue;
      }
      float v[NC];
      tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * 64), v);
      tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * 64 + 32), v + 32);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
#pragma unroll
      for (int i = 0; i < NC / 4; ++i) {
        const float4 b = __ldg(reinterpret_cast<const float4*>(bias) + i);
        v[4 * i] += b.x; v[4 * i + 1] += b.y; v[4 * i + 2] += b.z; v[4 * i + 3] += b.w;
      }
      act_inplace<NC>(v, act, true);
      if (prof) { const long long t1 = clock64(); pc[4] += t1 - pt0; pt0 = t1; }
      if (lane == 0) bulk_wait_read0();  // the previous store has read the tile
      __syncwarp();
      if (prof) { const long long t1 = clock64(); pc[5] += t1 - pt0; pt0 = t1; }
      {
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(tile + lane * 128 + ((c ^ (lane & 7)) << 4)) = pack8h(v + c * 8, h16);
      }
      fence_proxy_async();
      __syncwarp();
      const int64_t row0 = (int64_t)t * 128 + q * 32;
      if (lane == 0 && row0 < M) {
        tma_store_2d(&maps.out, tile, 0, (int)row0);
        bulk_commit();
      }
      if (prof) { pc[6] += clock64() - pt0; pc[7] += 1; }
    }
    if (lane == 0) bulk_wait0();
  } else if (IMG && warp == 17) {
    // ---------------- image loads (IMG)
    if (lane == 0) {
      for (int j = 0;; ++j) {
        const int u = blockIdx.x + j * gridDim.x;
        if (u >= g.n) break;
        const int slot = j % STEM_IMGS;
        if (!mbar_wait(&iempty[slot], ((uint32_t)(j / STEM_IMGS) & 1u) ^ 1u, abort_flag, 56)) break;
        mbar_arrive_tx(&ifull[slot], (uint32_t)(g.c * g.h * 32 * 4));
        tma_load_4d(simg + slot * (STEM_IMG_BYTES / 4), &maps.a[0], &ifull[slot], 0, 0, 0, u);
      }
    }
  } else if (warp == MMA_WARP && lane == 0) {
    // ---------------- MMA issue
    const uint32_t idesc = instr_desc_h(BM, 64, h16);
    const uint64_t ad0 = smem_desc(smem_u32(sa)), bd = smem_desc(smem_u32(sbw));
    int stage = 0;
    uint32_t phase = 0;
    for (int i = 0; tile_of(i) < n_tiles; ++i) {
      const int acc = i % NACC;
      const uint32_t acc_phase = (uint32_t)(i / NACC) & 1u;
      if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, 53)) break;
      if (!mbar_wait(&afull[stage], phase, abort_flag, 54)) break;
      tc_fence_after();
      const uint64_t ad = ad0 + (uint64_t)stage * (16384 >> 4);
      const uint32_t d = tmem_base + (uint32_t)(acc * 64);
      mma_bf16(d, ad, bd, idesc, 0u);
      mma_bf16(d, ad + 2, bd + 2, idesc, 1u);  // K 16..31 (32 bytes further)
      mma_commit(&aempty[stage]);
      mma_commit(&tfull[acc]);
      if (++stage == STEM_STAGES) { stage = 0; phase ^= 1; }
    }
  }

  if (prof && lane == 0)
    for (int i = 0; i < 8; ++i)
      if (pc[i]) atomicAdd(&prof[i], (unsigned long long)pc[i]);
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {
    for (int i = 0; i < 1000; ++i) __nanosleep(1000);
  }
  if (warp == MMA_WARP) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(NACC * 64));
  }
}

}  // namespace tc

// ------------------------------------------------------------------ host side

static int pick_block_n(int64_t N, int requested) {
  if (requested == 64 || requested == 128 || requested == 256) return requested;
  if (N <= 64) return 64;
  if (N <= 128) return 128;
  if (N % 256 == 0) return 256;
  return 128;
}

// bf16 GEMM outputs leave through TMA stores (tc_gemm_kernel's per-warp
// tiles): Tx-large fp8 QKV 0.62 -> 0.39 ms, ResNet 1x1 shortcuts up to 1.5x, and
// long-K convolutions a little faster once the stage budget grows to the opt-in
// shared-memory maximum.  C3B200_GEMM_TMA_OUT=0 keeps the per-lane stores
// everywhere (A/B timing).
static int enable_tma_out(tc::TmaMaps& maps, tc::TcArgs& a) {
  static const bool on = [] {
    const char* e = getenv("C3B200_GEMM_TMA_OUT");
    return !(e && e[0] == '0');
  }();
  a.tma_out = 0;
  if (!on || a.N % 16) return C3B_OK;
  if (a.dt_out == C3B_F32) {
    // f32 output (and f32 residual) through 2 KB tiles: 16 columns x 32 rows, 64-byte swizzle
    static const bool f32_on = [] {
      const char* e = getenv("C3B200_GEMM_TMA_OUT32");
      return !(e && e[0] == '0');
    }();
    if (!f32_on || (a.res && a.dt_res != C3B_F32)) return C3B_OK;
    uint64_t dims[2] = {(uint64_t)a.N, (uint64_t)a.M};
    uint64_t str[1] = {(uint64_t)a.N * 4};
    uint32_t box[2] = {16, 32};
    int rc = encode(&maps.out, a.out, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_DATA_TYPE_FLOAT32);
    if (rc) return rc;
    if (a.res && (rc = encode(&maps.res, const_cast<void*>(a.res), 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_64B,
                              CU_TENSOR_MAP_DATA_TYPE_FLOAT32)))
      return rc;
    a.tma_out = 2;
    return C3B_OK;
  }
  uint64_t dims[2] = {(uint64_t)a.N, (uint64_t)a.M};
  uint64_t str[1] = {(uint64_t)a.N * 2};
  uint32_t box[2] = {16, 32};
  int rc = encode(&maps.out, a.out, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_32B);
  if (rc) return rc;
  a.tma_out = 1;
  return C3B_OK;
}

template <int MODE, int CG = 1, bool AUX = false>
static int launch_tc_mode(const tc::TmaMaps& maps, tc::TcArgs& a, cudaStream_t s) {
  // one 128-byte K row per operand row; MODE 2 adds the packed FP4 tile and its scales
  const size_t b_stage = (size_t)(a.block_n / CG) * 128;
  if (MODE != 0 || CG != 1) a.bres = 0;
  const size_t b_res = a.bres ? (size_t)a.k_blocks * b_stage : 0;  // resident B (single CTAs)
  if ((a.aux_n != 0) != AUX) return fail(C3B_E_INVALID, "tc gemm: fused shortcut needs its kernel variant");
  const size_t aux_bytes = AUX ? (size_t)a.cblocks * a.aux_n * 128 : 0;  // fused shortcut weights
  size_t stage_bytes = (size_t)tc::BM * 128 + (a.bres ? 0 : b_stage);
  if (MODE == 2) stage_bytes += (size_t)a.block_n * (tc::BK / 2) + (size_t)a.block_n * (tc::BK / tc::W4_GROUP) * 4;
  size_t out_tiles =
      a.tma_out ? (size_t)(MODE == 2 ? 8 : 16) * (a.tma_out == 2 ? 4096 : 2048) + 1024 : 0;  // + alignment
  // with output tiles the stage ring takes what the opt-in maximum leaves, so
  // long-K convolutions keep their pipeline depth
  size_t budget = a.tma_out ? 227 * 1024 - 2048 - out_tiles - b_res - aux_bytes : 200 * 1024 - b_res - aux_bytes;
  if (a.bres && a.tma_out && budget / stage_bytes < 4) {
    // resident B and output tiles leave under four A stages: per-lane stores
    a.tma_out = 0;
    out_tiles = 0;
    budget = 227 * 1024 - 2048 - b_res - aux_bytes;
  }
  int stages = (int)(budget / stage_bytes);
  if (stages > 8) stages = 8;
  if (stages < 2) return fail(C3B_E_INVALID, "tc gemm: tile does not fit in shared memory");
  a.stages = stages;
  const size_t smem = 1024 + stages * stage_bytes + b_res + aux_bytes + out_tiles + (3 * stages + 4 + 32) * 8 + 16;
  static bool attr_set = false;
  if (!attr_set) {
    C3B_CHECK_CUDA(cudaFuncSetAttribute(tc::tc_gemm_kernel<MODE, CG, AUX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        227 * 1024));
    attr_set = true;
  }
  if (CG == 2) {
    // persistent pairs: as many clusters as can be resident at once
    static int max_clusters = 0;
    if (!max_clusters) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)sm_count());
      cfg.blockDim = dim3((unsigned)tc::HALO16_THREADS);
      cfg.dynamicSmemBytes = 227 * 1024;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = 2;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, tc::tc_gemm_kernel<MODE, CG, AUX>, &cfg) != cudaSuccess || n < 1) {
        (void)cudaGetLastError();
        n = sm_count() / 2;
      }
      max_clusters = n;
    }
    const int clusters = a.n_tiles < max_clusters ? a.n_tiles : max_clusters;
    if (clusters < 1) return C3B_OK;
    if (int rc = launch_pdl_cluster(tc::tc_gemm_kernel<MODE, CG, AUX>, 2 * clusters, 2, tc::HALO16_THREADS, smem, s, maps,
                                    a))
      return rc;
    C3B_CHECK_CUDA(cudaGetLastError());
    return C3B_OK;
  }
  int grid = a.n_tiles < sm_count() ? a.n_tiles : sm_count();
  if (grid < 1) return C3B_OK;
  if (int rc = launch_pdl(tc::tc_gemm_kernel<MODE, CG, AUX>, grid, tc::HALO16_THREADS, smem, s, maps, a)) return rc;
  C3B_CHECK_CUDA(cudaGetLastError());
  return C3B_OK;
}

// CTA pairs for bf16/fp16 GEMMs and convolutions through tc_gemm_kernel with
// 256-column tiles (128-column pairs measured no faster): B is re-encoded with half-width boxes (each CTA of a pair
// loads its half) and tiles are counted in 256 rows.  C3B200_GEMM_PAIR=0 keeps
// single-CTA tiles (A/B timing).
static int use_pairs(tc::TmaMaps& maps, tc::TcArgs& a, const void* b, uint64_t K, uint64_t N) {
  static const bool on = [] {
    const char* e = getenv("C3B200_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  a.cg = 1;
  static const int min_n = [] {
    const char* e = getenv("C3B200_GEMM_PAIR_MIN_N");
    return e ? atoi(e) : 256;
  }();
  // (short K: the pair's cross-CTA handshakes cost more than the halved B
  // traffic saves; ResNet 1x1 shortcuts with K = 128/256 measured slower)
  // (few tiles: pairs halve the tile count, and below two waves of pairs
  // the coarser quantisation cost more than the shared B saves; ResNet-18 at
  // 512 images per GPU measured 689K img/s with pairs, 705K without)
  static const int min_tiles = [] {
    const char* e = getenv("C3B200_GEMM_PAIR_MIN_TILES");
    return e ? atoi(e) : sm_count();
  }();
  const int64_t pair_tiles = (a.M + 2 * tc::BM - 1) / (2 * tc::BM) * a.n_tiles_n;
  if (!on || a.block_n < min_n || a.M < 2 * tc::BM || a.k_blocks < 8 || pair_tiles < min_tiles) return C3B_OK;
  uint64_t dims[2] = {K, N};
  uint64_t str[1] = {K * 2};
  uint32_t box[2] = {tc::BK, (uint32_t)a.block_n / 2};
  if (int rc = encode(&maps.b, const_cast<void*>(b), 2, dims, str, box)) return rc;
  a.cg = 2;
  a.n_tiles = (int)((a.M + 2 * tc::BM - 1) / (2 * tc::BM)) * a.n_tiles_n;
  return C3B_OK;
}

// Resident B for single-CTA bf16/fp16 convolutions whose B column block fits
// in shared memory beside four A stages: the weights are staged once per CTA
// instead of once per tile, which halves the shared-memory fill of each K
// block (N = 128 tiles are bound by shared-memory bandwidth: TMA fill plus
// the MMA operand reads).  A CTA's tiles all share one column block when the
// grid (the SM count) is a multiple of the column-block count.
// C3B200_GEMM_BRES=0 restages B per K block (A/B timing).
static void use_resident_b(tc::TcArgs& a) {
  static const bool on = [] {
    const char* e = getenv("C3B200_GEMM_BRES");
    return !(e && e[0] == '0');
  }();
  a.bres = 0;
  const size_t b_res = (size_t)a.k_blocks * a.block_n * 128;
  if (!on || a.cg != 1 || sm_count() % a.n_tiles_n != 0 || a.n_tiles < 2 * sm_count()) return;
  if (b_res + 4 * (size_t)tc::BM * 128 + 4096 > 227 * 1024) return;
  a.bres = 1;
}

static int launch_tc(const tc::TmaMaps& maps, tc::TcArgs& a, cudaStream_t s, int mode = 0) {
  if (mode == 0 && a.cg == 2) return launch_tc_mode<0, 2>(maps, a, s);
  if (mode == 0 && a.aux_n) return launch_tc_mode<0, 1, true>(maps, a, s);
  if (mode == 3) return launch_tc_mode<3>(maps, a, s);
  if (mode == 1) return launch_tc_mode<1>(maps, a, s);
  if (mode == 2) return launch_tc_mode<2>(maps, a, s);
  return launch_tc_mode<0>(maps, a, s);
}

static int fill_epilogue(tc::TcArgs& a, const c3b_tensor* in, int n_in, int first_extra, int bias_mode,
                         int has_residual, int64_t M, int64_t N, const c3b_tensor& out) {
  int idx = first_extra;
  a.bias = nullptr;
  a.res = nullptr;
  if (bias_mode != C3B_BIAS_NONE) {
    C3B_REQUIRE(bias_mode == C3B_BIAS_COL, "tc: only per-column bias");
    C3B_REQUIRE(idx < n_in && in[idx].dtype == C3B_F32 && numel(in[idx]) == N, "tc: bias must be f32 [N]");
    a.bias = (const float*)in[idx++].ptr;
  }
  if (has_residual) {
    C3B_REQUIRE(idx < n_in, "tc: missing residual");
    C3B_REQUIRE(in[idx].dtype == (a.h16 ? C3B_F16 : C3B_BF16) || in[idx].dtype == C3B_F32,
                a.h16 ? "tc: residual fp16/f32" : "tc: residual bf16/f32");
    C3B_REQUIRE(numel(in[idx]) >= M * N, "tc: residual too small");
    C3B_REQUIRE(((uintptr_t)in[idx].ptr & 15) == 0, "tc: residual must be 16-byte aligned");
    a.res = in[idx].ptr;
    a.dt_res = in[idx].dtype;
    idx++;
  }
  C3B_REQUIRE(idx == n_in, "tc: input count does not match bias/residual flags");
  C3B_REQUIRE(out.dtype == (a.h16 ? C3B_F16 : C3B_BF16) || out.dtype == C3B_F32,
              a.h16 ? "tc: output fp16/f32" : "tc: output bf16/f32");
  C3B_REQUIRE(numel(out) >= M * N, "tc: output too small");
  C3B_REQUIRE(((uintptr_t)out.ptr & 15) == 0, "tc: output must be 16-byte aligned");
  a.out = out.ptr;
  a.dt_out = out.dtype;
  return C3B_OK;
}

// Failure-path probe (C3B_K_WAIT_PROBE): one thread waits, through the same
// bounded mbarrier wait as every tcgen05 kernel, on a barrier that nothing
// ever arrives on.  When the limit runs out the wait sets the device status
// word to `code` and the kernel returns, leaving the context usable.  Tests
// shorten the limit (c3b_set_wait_limit_ns) so this takes about a millisecond.
__global__ void wait_probe_kernel(int code) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    tc::mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tc::mbar_wait(&bar, 0, &abort_flag, code);
  }
}

int launch_wait_probe(const c3b_wait_probe_params& p, cudaStream_t s) {
  C3B_REQUIRE(p.code > 0, "wait probe: the status code must be positive");
  wait_probe_kernel<<<1, 32, 0, s>>>(p.code);
  C3B_CHECK_CUDA(cudaGetLastError());
  return C3B_OK;
}

int launch_gemm_tc(const c3b_tensor* in, int n_in, const c3b_tensor& out, const c3b_gemm_tc_params& p,
                   cudaStream_t s) {
  C3B_REQUIRE(n_in >= 2, "tc gemm: needs A and B");
  C3B_REQUIRE((in[0].dtype == C3B_BF16 || in[0].dtype == C3B_F16) && in[1].dtype == in[0].dtype,
              "tc gemm: A and B must be both bf16 or both fp16");
  C3B_REQUIRE(p.K > 0 && p.K % 8 == 0, "tc gemm: K must be a positive multiple of 8");
  C3B_REQUIRE(p.N > 0 && p.N % 32 == 0, "tc gemm: N must be a positive multiple of 32");
  C3B_REQUIRE(p.M >= 0 && p.M < (int64_t)1 << 31, "tc gemm: M range");
  C3B_REQUIRE(numel(in[0]) >= p.M * p.K && numel(in[1]) >= p.N * p.K, "tc gemm: operand extents");
  C3B_REQUIRE(((uintptr_t)in[0].ptr & 15) == 0 && ((uintptr_t)in[1].ptr & 15) == 0, "tc gemm: 16-byte alignment");
  tc::TcArgs a;
  memset(&a, 0, sizeof(a));
  a.h16 = in[0].dtype == C3B_F16;
  int rc = fill_epilogue(a, in, n_in, 2, p.bias_mode, p.has_residual, p.M, p.N, out);
  if (rc) return rc;
  if (p.M == 0) return C3B_OK;
  a.M = p.M; a.N = p.N; a.K = p.K; a.act = p.act;
  a.block_n = pick_block_n(p.N, p.block_n);
  a.n_tiles_n = (int)((p.N + a.block_n - 1) / a.block_n);
  a.n_tiles = (int)((p.M + tc::BM - 1) / tc::BM) * a.n_tiles_n;
  a.k_blocks = (int)((p.K + tc::BK - 1) / tc::BK);
  tc::TmaMaps maps;
  memset(&maps, 0, sizeof(maps));
  {
    uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.M};
    uint64_t str[1] = {(uint64_t)p.K * 2};
    uint32_t box[2] = {tc::BK, tc::BM};
    if ((rc = encode(&maps.a[0], in[0].ptr, 2, dims, str, box))) return rc;
  }
  {
    uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.N};
    uint64_t str[1] = {(uint64_t)p.K * 2};
    uint32_t box[2] = {tc::BK, (uint32_t)a.block_n};
    if ((rc = encode(&maps.b, in[1].ptr, 2, dims, str, box))) return rc;
  }
  if ((rc = use_pairs(maps, a, in[1].ptr, (uint64_t)p.K, (uint64_t)p.N))) return rc;
  if ((rc = enable_tma_out(maps, a))) return rc;
  return launch_tc(maps, a, s);
}

// fp32 operands on the tensor cores as tf32 (the tf32 precision profile):
// kind::tf32 reads fp32 words and uses their 10 leading mantissa bits, fp32
// accumulation in TMEM, the same epilogue as the bf16 GEMM.
int launch_gemm_tf32(const c3b_tensor* in, int n_in, const c3b_tensor& out, const c3b_gemm_tc_params& p,
                     cudaStream_t s) {
  C3B_REQUIRE(n_in >= 2, "tf32 gemm: needs A and B");
  C3B_REQUIRE(in[0].dtype == C3B_F32 && in[1].dtype == C3B_F32, "tf32 gemm: A and B must be f32");
  C3B_REQUIRE(p.K > 0 && p.K % 4 == 0, "tf32 gemm: K must be a positive multiple of 4");
  C3B_REQUIRE(p.N > 0 && p.N % 32 == 0, "tf32 gemm: N must be a positive multiple of 32");
  C3B_REQUIRE(p.M >= 0 && p.M < (int64_t)1 << 31, "tf32 gemm: M range");
  C3B_REQUIRE(numel(in[0]) >= p.M * p.K && numel(in[1]) >= p.N * p.K, "tf32 gemm: operand extents");
  C3B_REQUIRE(((uintptr_t)in[0].ptr & 15) == 0 && ((uintptr_t)in[1].ptr & 15) == 0, "tf32 gemm: 16-byte alignment");
  C3B_REQUIRE(out.dtype == C3B_F32, "tf32 gemm: f32 output");
  tc::TcArgs a;
  memset(&a, 0, sizeof(a));
  int rc = fill_epilogue(a, in, n_in, 2, p.bias_mode, p.has_residual, p.M, p.N, out);
  if (rc) return rc;
  C3B_REQUIRE(!a.res || a.dt_res == C3B_F32, "tf32 gemm: f32 residual");
  if (p.M == 0) return C3B_OK;
  a.M = p.M; a.N = p.N; a.K = p.K; a.act = p.act;
  a.block_n = pick_block_n(p.N, p.block_n);
  a.n_tiles_n = (int)((p.N + a.block_n - 1) / a.block_n);
  a.n_tiles = (int)((p.M + tc::BM - 1) / tc::BM) * a.n_tiles_n;
  a.k_blocks = (int)((p.K + 31) / 32);
  tc::TmaMaps maps;
  memset(&maps, 0, sizeof(maps));
  {
    uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.M};
    uint64_t str[1] = {(uint64_t)p.K * 4};
    uint32_t box[2] = {32, tc::BM};
    if ((rc = encode(&maps.a[0], in[0].ptr, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_DATA_TYPE_FLOAT32)))
      return rc;
  }
  {
    uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.N};
    uint64_t str[1] = {(uint64_t)p.K * 4};
    uint32_t box[2] = {32, (uint32_t)a.block_n};
    if ((rc = encode(&maps.b, in[1].ptr, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_DATA_TYPE_FLOAT32)))
      return rc;
  }
  return launch_tc(maps, a, s, 3);
}

int launch_gemm_fp8(const c3b_tensor* in, int n_in, const c3b_tensor& out, const c3b_gemm_tc_params& p,
                    cudaStream_t s) {
  C3B_REQUIRE(n_in >= 4, "fp8 gemm: needs A, B, A row scales, B row scales");
  C3B_REQUIRE(in[0].dtype == C3B_U8 && in[1].dtype == C3B_U8, "fp8 gemm: A and B must be e4m3 bytes (u8)");
  C3B_REQUIRE(in[2].dtype == C3B_F32 && in[3].dtype == C3B_F32, "fp8 gemm: scales must be f32");
  C3B_REQUIRE(p.K > 0 && p.K % 16 == 0, "fp8 gemm: K must be a positive multiple of 16");
  C3B_REQUIRE(p.N > 0 && p.N % 32 == 0, "fp8 gemm: N must be a positive multiple of 32");
  C3B_REQUIRE(p.M >= 0 && p.M < (int64_t)1 << 31, "fp8 gemm: M range");
  C3B_REQUIRE(numel(in[0]) >= p.M * p.K && numel(in[1]) >= p.N * p.K, "fp8 gemm: operand extents");
  C3B_REQUIRE(numel(in[2]) >= p.M && numel(in[3]) >= p.N, "fp8 gemm: scale extents");
  C3B_REQUIRE(((uintptr_t)in[0].ptr & 15) == 0 && ((uintptr_t)in[1].ptr & 15) == 0 && ((uintptr_t)in[3].ptr & 15) == 0,
              "fp8 gemm: 16-byte alignment");
  tc::TcArgs a;
  memset(&a, 0, sizeof(a));
  a.h16 = out.dtype == C3B_F16;
  int rc = fill_epilogue(a, in, n_in, 4, p.bias_mode, p.has_residual, p.M, p.N, out);
  if (rc) return rc;
  if (p.M == 0) return C3B_OK;
  a.M = p.M; a.N = p.N; a.K = p.K; a.act = p.act;
  a.a_scale = (const float*)in[2].ptr;
  a.b_scale = (const float*)in[3].ptr;
  a.block_n = pick_block_n(p.N, p.block_n);
  a.n_tiles_n = (int)((p.N + a.block_n - 1) / a.block_n);
  a.n_tiles = (int)((p.M + tc::BM - 1) / tc::BM) * a.n_tiles_n;
  a.k_blocks = (int)((p.K + 127) / 128);
  tc::TmaMaps maps;
  memset(&maps, 0, sizeof(maps));
  {
    uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.M};
    uint64_t str[1] = {(uint64_t)p.K};
    uint32_t box[2] = {128, tc::BM};
    if ((rc = encode(&maps.a[0], in[0].ptr, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_DATA_TYPE_UINT8)))
      return rc;
  }
  {
    uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.N};
    uint64_t str[1] = {(uint64_t)p.K};
    uint32_t box[2] = {128, (uint32_t)a.block_n};
    if ((rc = encode(&maps.b, in[1].ptr, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_DATA_TYPE_UINT8)))
      return rc;
  }
  if ((rc = enable_tma_out(maps, a))) return rc;
  return launch_tc(maps, a, s, 1);
}

int launch_gemm_w4a16(const c3b_tensor* in, int n_in, const c3b_tensor& out, const c3b_gemm_tc_params& p,
                      cudaStream_t s) {
  C3B_REQUIRE(n_in >= 3, "w4a16 gemm: needs A, packed B, B scales");
  C3B_REQUIRE((in[0].dtype == C3B_BF16 || in[0].dtype == C3B_F16) && in[1].dtype == C3B_U8 &&
                  in[2].dtype == C3B_F32,
              "w4a16 gemm: A bf16 or fp16, B packed FP4 (u8), scales f32");
  C3B_REQUIRE(p.K > 0 && p.K % 64 == 0, "w4a16 gemm: K must be a positive multiple of 64");
  C3B_REQUIRE(p.N > 0 && p.N % 32 == 0, "w4a16 gemm: N must be a positive multiple of 32");
  C3B_REQUIRE(p.M >= 0 && p.M < (int64_t)1 << 31, "w4a16 gemm: M range");
  C3B_REQUIRE(numel(in[0]) >= p.M * p.K && numel(in[1]) >= p.N * p.K / 2 && numel(in[2]) >= p.N * p.K / tc::W4_GROUP,
              "w4a16 gemm: operand extents");
  C3B_REQUIRE(((uintptr_t)in[0].ptr & 15) == 0 && ((uintptr_t)in[1].ptr & 15) == 0 && ((uintptr_t)in[2].ptr & 15) == 0,
              "w4a16 gemm: 16-byte alignment");
  tc::TcArgs a;
  memset(&a, 0, sizeof(a));
  a.h16 = in[0].dtype == C3B_F16;  // the FP4 weights expand to the activations' format
  int rc = fill_epilogue(a, in, n_in, 3, p.bias_mode, p.has_residual, p.M, p.N, out);
  if (rc) return rc;
  if (p.M == 0) return C3B_OK;
  a.M = p.M; a.N = p.N; a.K = p.K; a.act = p.act;
  a.block_n = pick_block_n(p.N, p.block_n);
  a.n_tiles_n = (int)((p.N + a.block_n - 1) / a.block_n);
  a.n_tiles = (int)((p.M + tc::BM - 1) / tc::BM) * a.n_tiles_n;
  a.k_blocks = (int)(p.K / tc::BK);
  tc::TmaMaps maps;
  memset(&maps, 0, sizeof(maps));
  {
    uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.M};
    uint64_t str[1] = {(uint64_t)p.K * 2};
    uint32_t box[2] = {tc::BK, tc::BM};
    if ((rc = encode(&maps.a[0], in[0].ptr, 2, dims, str, box))) return rc;
  }
  {  // packed FP4 rows: K/2 bytes per output row, 32 bytes (64 elements) per K block
    uint64_t dims[2] = {(uint64_t)p.K / 2, (uint64_t)p.N};
    uint64_t str[1] = {(uint64_t)p.K / 2};
    uint32_t box[2] = {tc::BK / 2, (uint32_t)a.block_n};
    if ((rc = encode(&maps.a[1], in[1].ptr, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_DATA_TYPE_UINT8)))
      return rc;
  }
  {  // scales [K/64][N][4]: the four group scales of one row and K block are contiguous
    uint64_t dims[3] = {(uint64_t)(tc::BK / tc::W4_GROUP), (uint64_t)p.N, (uint64_t)p.K / tc::BK};
    uint64_t str[2] = {(uint64_t)(tc::BK / tc::W4_GROUP) * 4, (uint64_t)p.N * (tc::BK / tc::W4_GROUP) * 4};
    uint32_t box[3] = {(uint32_t)(tc::BK / tc::W4_GROUP), (uint32_t)a.block_n, 1};
    if ((rc = encode(&maps.a[2], in[2].ptr, 3, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_DATA_TYPE_FLOAT32)))
      return rc;
  }
  if ((rc = enable_tma_out(maps, a))) return rc;
  return launch_tc(maps, a, s, 2);
}

int launch_conv_tc(const c3b_tensor* in, int n_in, const c3b_tensor* outs, const c3b_conv_tc_params& p,
                   cudaStream_t s) {
  const c3b_tensor& out = outs[0];
  const int n_main = 3 + (p.has_residual ? 1 : 0);
  C3B_REQUIRE(n_in == n_main + (p.has_shortcut ? 2 : 0),
              "tc conv: inputs x, w, bias [, residual] [, shortcut w, shortcut bias]");
  C3B_REQUIRE((in[0].dtype == C3B_BF16 || in[0].dtype == C3B_F16) && in[1].dtype == in[0].dtype,
              "tc conv: activations and weights both bf16 or both fp16");
  C3B_REQUIRE(p.cin % 64 == 0, "tc conv: Cin must be a multiple of 64");
  C3B_REQUIRE(p.cout % 32 == 0, "tc conv: Cout must be a multiple of 32");
  C3B_REQUIRE(p.stride == 1 || p.stride == 2, "tc conv: stride 1 or 2");
  C3B_REQUIRE(p.ho == (p.h + 2 * p.pad - p.k) / p.stride + 1 && p.wo == (p.w + 2 * p.pad - p.k) / p.stride + 1,
              "tc conv: output extents");
  if (p.stride == 2) {
    C3B_REQUIRE(p.h % 2 == 0 && p.w % 2 == 0, "tc conv: stride 2 needs even H, W");
    C3B_REQUIRE(p.ho == p.h / 2 && p.wo == p.w / 2, "tc conv: stride-2 geometry must halve H and W");
  }
  const int pix = p.ho * p.wo;
  C3B_REQUIRE(p.wo <= 128 && 128 % p.wo == 0, "tc conv: Wo must divide 128");
  C3B_REQUIRE(pix >= 128 ? pix % 128 == 0 : 128 % pix == 0, "tc conv: Ho*Wo must divide or be a multiple of 128");
  C3B_REQUIRE(numel(in[0]) == (int64_t)p.n * p.h * p.w * p.cin, "tc conv: input extents");
  C3B_REQUIRE(numel(in[1]) == (int64_t)p.cout * p.k * p.k * p.cin, "tc conv: weight extents");
  C3B_REQUIRE(((uintptr_t)in[0].ptr & 15) == 0 && ((uintptr_t)in[1].ptr & 15) == 0, "tc conv: 16-byte alignment");
  const int64_t M = (int64_t)p.n * pix;
  tc::TcArgs a;
  memset(&a, 0, sizeof(a));
  a.h16 = in[0].dtype == C3B_F16;
  int rc = fill_epilogue(a, in, n_main, 2, C3B_BIAS_COL, p.has_residual, M, p.cout, out);
  if (rc) return rc;
  if (M == 0) return C3B_OK;
  const int64_t K = (int64_t)p.k * p.k * p.cin;
  a.M = M; a.N = p.cout; a.K = K; a.act = p.act;
  a.block_n = pick_block_n(p.cout, p.block_n);
  a.n_tiles_n = (p.cout + a.block_n - 1) / a.block_n;
  a.n_tiles = (int)((M + tc::BM - 1) / tc::BM) * a.n_tiles_n;
  a.k_blocks = (int)(K / tc::BK);
  a.conv = 1; a.cblocks = p.cin / 64; a.ksz = p.k; a.stride = p.stride; a.pad = p.pad;
  a.pix = pix; a.wo = p.wo; a.cin = p.cin;
  if (p.has_shortcut) {
    // The 1x1 stride-2 shortcut samples the centre tap's pixels: its A blocks
    // are the centre tap's, and it becomes aux_n more columns of each tile
    // (checked here, before any CUDA call).
    const c3b_tensor &ws = in[n_main], &bs = in[n_main + 1], &ys = outs[1];
    C3B_REQUIRE(p.stride == 2 && p.k % 2 == 1 && p.pad == p.k / 2, "tc conv shortcut: stride 2, pad k/2");
    C3B_REQUIRE(!p.has_residual, "tc conv shortcut: the main convolution takes no residual");
    C3B_REQUIRE(a.n_tiles_n == 1 && a.block_n == p.cout && (p.cout == 64 || p.cout == 128),
                "tc conv shortcut: Cout 64 or 128 (one column block)");
    C3B_REQUIRE(ws.dtype == in[0].dtype && numel(ws) == (int64_t)p.cout * p.cin, "tc conv shortcut: ws [Cout, Cin]");
    C3B_REQUIRE(bs.dtype == C3B_F32 && numel(bs) == p.cout, "tc conv shortcut: bs [Cout] f32");
    C3B_REQUIRE(ys.dtype == in[0].dtype && numel(ys) == M * p.cout, "tc conv shortcut: ys [N, Ho, Wo, Cout] 16-bit");
    C3B_REQUIRE(((uintptr_t)ws.ptr & 15) == 0 && ((uintptr_t)bs.ptr & 15) == 0 && ((uintptr_t)ys.ptr & 15) == 0,
                "tc conv shortcut: 16-byte alignment");
    a.aux_n = p.cout;
    a.aux_kb0 = (p.pad * p.k + p.pad) * a.cblocks;
    a.aux_w = static_cast<const uint16_t*>(ws.ptr);
    a.aux_bias = static_cast<const float*>(bs.ptr);
    a.aux_out = static_cast<uint16_t*>(ys.ptr);
  }
  const uint32_t bw = (uint32_t)p.wo;
  const uint32_t bh = pix >= 128 ? 128u / bw : (uint32_t)p.ho;
  const uint32_t bn = pix >= 128 ? 1u : 128u / (uint32_t)pix;
  a.bh = (int)bh;
  tc::TmaMaps maps;
  memset(&maps, 0, sizeof(maps));
  uint8_t* x = static_cast<uint8_t*>(in[0].ptr);
  const uint64_t C = p.cin;
  {
    uint64_t dims[2] = {(uint64_t)K, (uint64_t)p.cout};
    uint64_t str[1] = {(uint64_t)K * 2};
    uint32_t box[2] = {tc::BK, (uint32_t)a.block_n};
    if ((rc = encode(&maps.b, in[1].ptr, 2, dims, str, box))) return rc;
  }
  // Halo mode: 3x3, stride 1, pad 1, Cout <= 128 (one weight tile), two output
  // rows per super-tile.
  const int wt = p.wo < 16 ? p.wo : 16;
  // (16-bit output and residual only: their epilogues store 16-bit rows)
  const bool bf16_epi = a.dt_out != C3B_F32 && (!a.res || a.dt_res != C3B_F32);
  if (p.mode != 1 && bf16_epi && p.k == 3 && p.stride == 1 && p.pad == 1 && p.cout <= 128 && a.n_tiles_n == 1 &&
      p.wo % wt == 0 && 128 % wt == 0 && (128 / wt) >= 8 && p.ho % 2 == 0) {
    a.img = 128 / wt;
    a.wt = wt;
    a.wblocks = p.wo / wt;
    a.ho = p.ho;
    a.n_img = p.n;
    // sliding-window accumulators (tc_conv_rowslide_kernel) unless
    // C3B200_CONV_RING=1 selects the paired row-ring kernel (A/B timing)
    static const bool use_ring = [] {
      const char* e = getenv("C3B200_CONV_RING");
      return e && e[0] == '1';
    }();
    if (p.mode == 0 && !use_ring && p.cin == 64 && p.cout == 64 && a.block_n == 64 && 32 % a.img == 0) {
      // Segments split each strip's rows across CTAs.  A segment of R rows
      // issues MMAs for R + 2 input rows, so the choice minimises
      // waves x (R + 2): whole strips at large batch, shorter segments only
      // where they fill idle SMs (at 512 images the old rule, four items per
      // SM, made 4-row segments that cost 1.5x the MMA issue).
      const int strips = ((p.n + a.img - 1) / a.img) * a.wblocks;
      int segs = 1;
      long best = -1;
      for (int sg = 1; sg <= p.ho / 2 && p.ho % sg == 0; sg *= 2) {
        const long waves = ((long)strips * sg + sm_count() - 1) / sm_count();
        const long cost = waves * (p.ho / sg + 2);
        if (best < 0 || cost < best) {
          best = cost;
          segs = sg;
        }
      }
      a.segs = segs;
      a.seg_rows = p.ho / segs;
      a.n_items = strips * segs;
      a.row_bytes = 64 * a.img * (wt + 2) * 2;
      const size_t rb = ((size_t)a.row_bytes + 1023) & ~(size_t)1023;
      const size_t wbytes = (size_t)9 * 64 * tc::BK * 2;
      // residual layers: per-warp 2 x 2 KB residual / output tiles
      static const bool tiles_nores = [] {
        const char* e = getenv("C3B200_SLIDE_TILES");
        return e && e[0] == '1';
      }();
      a.rring = p.has_residual ? 1 : tiles_nores ? 2 : 0;
      const size_t fixed = 1024 + wbytes + (a.rring ? 8 * 4096 : 0) + (1 + 2 * tc::SLIDE_NL + 16) * 8 + 16;
      int ring = (int)((227 * 1024 - fixed) / (rb + 16));
      if (ring > 8) ring = 8;
      if (ring >= 4) {
        a.ring = ring;
        uint64_t dims[4] = {C, (uint64_t)p.n, (uint64_t)p.w, (uint64_t)p.h};
        uint64_t str[3] = {(uint64_t)p.h * p.w * C * 2, C * 2, (uint64_t)p.w * C * 2};
        uint32_t box[4] = {64, (uint32_t)a.img, (uint32_t)(wt + 2), 1};
        if ((rc = encode(&maps.a[0], x, 4, dims, str, box))) return rc;
        if (a.rring) {
          // residual and output: NHWC [n, ho, wo, 64]; one warp's 32 channels x 32 pixels per box
          // (rring 2: output tiles only, no residual)
          uint64_t rdims[4] = {64, (uint64_t)p.n, (uint64_t)p.wo, (uint64_t)p.ho};
          uint64_t rstr[3] = {(uint64_t)p.ho * p.wo * 64 * 2, 64 * 2, (uint64_t)p.wo * 64 * 2};
          uint32_t rbox[4] = {32, (uint32_t)a.img, (uint32_t)(32 / a.img), 1};
          if (a.res &&
              (rc = encode(&maps.res, const_cast<void*>(a.res), 4, rdims, rstr, rbox, CU_TENSOR_MAP_SWIZZLE_64B)))
            return rc;
          if ((rc = encode(&maps.out, out.ptr, 4, rdims, rstr, rbox, CU_TENSOR_MAP_SWIZZLE_64B))) return rc;
        }
        const size_t smem = fixed + ring * (rb + 16);
        static bool attr_slide = false;
        if (!attr_slide) {
          C3B_CHECK_CUDA(cudaFuncSetAttribute(tc::tc_conv_rowslide_kernel,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
          attr_slide = true;
        }
        static unsigned long long* prof_buf = [] {
          const char* e = getenv("C3B200_CONV_PROF");
          unsigned long long* b = nullptr;
          if (e && e[0] == '1' && cudaMalloc(&b, tc::RP_COUNT * sizeof(unsigned long long)) != cudaSuccess) b = nullptr;
          return b;
        }();
        if (prof_buf) {
          C3B_CHECK_CUDA(cudaMemsetAsync(prof_buf, 0, tc::RP_COUNT * sizeof(unsigned long long), s));
          a.prof = prof_buf;
        }
        int grid = a.n_items < sm_count() ? a.n_items : sm_count();
        if ((rc = launch_pdl(tc::tc_conv_rowslide_kernel, grid, tc::SLIDE_THREADS, smem, s, maps, a))) return rc;
        C3B_CHECK_CUDA(cudaGetLastError());
        if (prof_buf) {
          unsigned long long h[tc::RP_COUNT];
          C3B_CHECK_CUDA(cudaStreamSynchronize(s));
          C3B_CHECK_CUDA(cudaMemcpy(h, prof_buf, sizeof(h), cudaMemcpyDeviceToHost));
          const double rows = h[tc::RP_PAIRS] ? (double)h[tc::RP_PAIRS] : 1.0;
          fprintf(stderr,
                  "[rowslide prof] res=%d per CTA: prod %.0f (empty-wait %.0f) | mma %.0f (rfull %.0f tempty %.0f) | "
                  "per epilogue warp: %.0f (tfull %.0f) | per output row: mma %.0f rfull %.0f tempty %.0f "
                  "epi-tfull %.0f | rows/CTA %.1f ring %d\n",
                  a.res != nullptr, (double)h[tc::RP_PROD_TOTAL] / grid, (double)h[tc::RP_PROD_EMPTY] / grid,
                  (double)h[tc::RP_MMA_TOTAL] / grid, (double)h[tc::RP_MMA_RFULL] / grid,
                  (double)h[tc::RP_MMA_TEMPTY] / grid, (double)h[tc::RP_EPI_TOTAL] / (8.0 * grid),
                  (double)h[tc::RP_EPI_TFULL] / (8.0 * grid), (double)h[tc::RP_MMA_TOTAL] / rows,
                  (double)h[tc::RP_MMA_RFULL] / rows, (double)h[tc::RP_MMA_TEMPTY] / rows,
                  (double)h[tc::RP_EPI_TFULL] / (8.0 * rows), rows / grid, ring);
        }
        return C3B_OK;
      }
    }
    if ((p.mode == 0) && p.cin == 64 && p.cout == 64 && a.block_n == 64) {
      // row ring: strips of IMG images x WT columns, segments of seg_rows rows
      const int strips = ((p.n + a.img - 1) / a.img) * a.wblocks;
      int segs = 1;
      while (strips * segs < 4 * sm_count() && segs * 2 <= p.ho / 2) segs *= 2;  // ~4 items per CTA (measured best of 2, 4, 8)
      if (p.ho % (2 * segs) == 0) {
        a.segs = segs;
        a.seg_rows = p.ho / segs;
        a.n_items = strips * segs;
        a.row_bytes = 64 * a.img * (wt + 2) * 2;
        const size_t rb = ((size_t)a.row_bytes + 1023) & ~(size_t)1023;
        const size_t wbytes = (size_t)9 * 64 * tc::BK * 2;
        const size_t epi = 8 * 4096;  // per-warp epilogue tiles
        const size_t budget = 212 * 1024;
        int ring = (int)((budget - wbytes - epi) / rb);
        if (ring > 8) ring = 8;
        if (ring >= 5 && 32 % a.img == 0) {
          a.ring = ring;
          uint64_t dims[4] = {C, (uint64_t)p.n, (uint64_t)p.w, (uint64_t)p.h};
          uint64_t str[3] = {(uint64_t)p.h * p.w * C * 2, C * 2, (uint64_t)p.w * C * 2};
          uint32_t box[4] = {64, (uint32_t)a.img, (uint32_t)(wt + 2), 1};
          if ((rc = encode(&maps.a[0], x, 4, dims, str, box))) return rc;
          // residual and output: NHWC [n, ho, wo, 64], one warp's 32 pixels x 32 channels per box
          uint64_t odims[4] = {64, (uint64_t)p.n, (uint64_t)p.wo, (uint64_t)p.ho};
          uint64_t ostr[3] = {(uint64_t)p.ho * p.wo * 64 * 2, 64 * 2, (uint64_t)p.wo * 64 * 2};
          uint32_t obox[4] = {32, (uint32_t)a.img, (uint32_t)(32 / a.img), 1};
          if ((rc = encode(&maps.out, out.ptr, 4, odims, ostr, obox, CU_TENSOR_MAP_SWIZZLE_64B))) return rc;
          if (p.has_residual &&
              (rc = encode(&maps.res, const_cast<void*>(a.res), 4, odims, ostr, obox, CU_TENSOR_MAP_SWIZZLE_64B)))
            return rc;
          const size_t smem = 1024 + ring * rb + wbytes + epi + (2 * ring + 13) * 8 + 16;
          static bool attr_ring = false;
          if (!attr_ring) {
            C3B_CHECK_CUDA(cudaFuncSetAttribute(tc::tc_conv_rowring_kernel,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
            attr_ring = true;
          }
          // Wait profiler (C3B200_CONV_PROF=1, measurement runs only): cycles
          // summed over CTAs, printed after a synchronous launch.
          static unsigned long long* prof_buf = [] {
            const char* e = getenv("C3B200_CONV_PROF");
            unsigned long long* b = nullptr;
            if (e && e[0] == '1' && cudaMalloc(&b, tc::RP_COUNT * sizeof(unsigned long long)) != cudaSuccess)
              b = nullptr;
            return b;
          }();
          if (prof_buf) {
            C3B_CHECK_CUDA(cudaMemsetAsync(prof_buf, 0, tc::RP_COUNT * sizeof(unsigned long long), s));
            a.prof = prof_buf;
          }
          int grid = a.n_items < sm_count() ? a.n_items : sm_count();
          if ((rc = launch_pdl(tc::tc_conv_rowring_kernel, grid, tc::HALO_THREADS, smem, s, maps, a))) return rc;
          C3B_CHECK_CUDA(cudaGetLastError());
          if (prof_buf) {
            unsigned long long h[tc::RP_COUNT];
            C3B_CHECK_CUDA(cudaStreamSynchronize(s));
            C3B_CHECK_CUDA(cudaMemcpy(h, prof_buf, sizeof(h), cudaMemcpyDeviceToHost));
            const double pairs = h[tc::RP_PAIRS] ? (double)h[tc::RP_PAIRS] : 1.0;
            fprintf(stderr,
                    "[rowring prof] res=%d per CTA: prod %.0f (empty-wait %.0f) | mma %.0f (rfull %.0f tempty %.0f) | "
                    "per epilogue warp: %.0f (tfull %.0f res %.0f) | per pair: mma %.0f rfull %.0f tempty %.0f "
                    "epi-tfull %.0f | pairs/CTA %.1f\n",
                    a.res != nullptr, (double)h[tc::RP_PROD_TOTAL] / grid, (double)h[tc::RP_PROD_EMPTY] / grid,
                    (double)h[tc::RP_MMA_TOTAL] / grid, (double)h[tc::RP_MMA_RFULL] / grid,
                    (double)h[tc::RP_MMA_TEMPTY] / grid, (double)h[tc::RP_EPI_TOTAL] / (8.0 * grid),
                    (double)h[tc::RP_EPI_TFULL] / (8.0 * grid), (double)h[tc::RP_EPI_RES] / (8.0 * grid),
                    (double)h[tc::RP_MMA_TOTAL] / pairs, (double)h[tc::RP_MMA_RFULL] / pairs,
                    (double)h[tc::RP_MMA_TEMPTY] / pairs, (double)h[tc::RP_EPI_TFULL] / (8.0 * pairs),
                    pairs / grid);
          }
          return C3B_OK;
        }
      }
    }
    a.rows = 2;
    a.halo_bytes = 64 * a.img * (wt + 2) * (a.rows + 2) * 2;
    a.n_tiles = ((p.n + a.img - 1) / a.img) * (p.ho / a.rows) * a.wblocks;
    uint64_t dims[4] = {C, (uint64_t)p.n, (uint64_t)p.w, (uint64_t)p.h};
    uint64_t str[3] = {(uint64_t)p.h * p.w * C * 2, C * 2, (uint64_t)p.w * C * 2};
    uint32_t box[4] = {64, (uint32_t)a.img, (uint32_t)(wt + 2), (uint32_t)(a.rows + 2)};
    if ((rc = encode(&maps.a[0], x, 4, dims, str, box))) return rc;
    const size_t hb = ((size_t)a.halo_bytes + 1023) & ~(size_t)1023;
    const size_t bb = (size_t)a.block_n * tc::BK * 2;
    a.hstages = 2;
    const size_t budget = 212 * 1024;
    if (2 * hb + 2 * bb > budget) return fail(C3B_E_INVALID, "tc conv: halo tiles do not fit in shared memory");
    const size_t all_b = (size_t)9 * a.cblocks * bb;
    if (2 * hb + all_b <= budget && p.mode != 2) {
      a.bres = 1;  // weights stay resident: one load per CTA
      a.stages = 9 * a.cblocks;
    } else {
      int bst = (int)((budget - 2 * hb) / bb);
      a.stages = bst > 8 ? 8 : bst;
    }
    size_t smem = 1024 + 2 * hb + a.stages * bb + (2 * 2 + 2 * a.stages + 4) * 8 + 16;
    // bf16 output through per-warp tiles and TMA stores when 16 KB of tiles fit
    // (residual layers of stage 2: the per-lane stores scatter one 16-byte piece
    // per image)
    a.tma_out = 0;
    if (32 % a.img == 0 && smem + 1024 + 16 * 1024 <= 227 * 1024) {
      uint64_t odims[4] = {(uint64_t)p.cout, (uint64_t)p.n, (uint64_t)p.wo, (uint64_t)p.ho};
      uint64_t ostr[3] = {(uint64_t)p.ho * p.wo * p.cout * 2, (uint64_t)p.cout * 2, (uint64_t)p.wo * p.cout * 2};
      uint32_t obox[4] = {16, (uint32_t)a.img, (uint32_t)(32 / a.img), 1};
      if ((rc = encode(&maps.out, out.ptr, 4, odims, ostr, obox, CU_TENSOR_MAP_SWIZZLE_32B))) return rc;
      a.tma_out = 1;
      smem += 1024 + 16 * 1024;
    }
    static bool attr_halo = false;
    if (!attr_halo) {
      C3B_CHECK_CUDA(cudaFuncSetAttribute(tc::tc_conv_halo_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          227 * 1024));
      attr_halo = true;
    }
    int grid = a.n_tiles < sm_count() ? a.n_tiles : sm_count();
    if ((rc = launch_pdl(tc::tc_conv_halo_kernel, grid, tc::HALO16_THREADS, smem, s, maps, a))) return rc;
    C3B_CHECK_CUDA(cudaGetLastError());
    return C3B_OK;
  }
  if (p.stride == 1) {
    uint64_t dims[4] = {C, (uint64_t)p.w, (uint64_t)p.h, (uint64_t)p.n};
    uint64_t str[3] = {C * 2, (uint64_t)p.w * C * 2, (uint64_t)p.h * p.w * C * 2};
    uint32_t box[4] = {64, bw, bh, bn};
    if ((rc = encode(&maps.a[0], x, 4, dims, str, box))) return rc;
  } else {
    for (int pr = 0; pr < 2; ++pr)
      for (int ps = 0; ps < 2; ++ps) {
        uint64_t dims[4] = {C, (uint64_t)(p.w / 2), (uint64_t)(p.h / 2), (uint64_t)p.n};
        uint64_t str[3] = {2 * C * 2, 2 * (uint64_t)p.w * C * 2, (uint64_t)p.h * p.w * C * 2};
        uint32_t box[4] = {64, bw, bh, bn};
        uint8_t* base = x + ((uint64_t)pr * p.w + ps) * C * 2;
        if ((rc = encode(&maps.a[pr * 2 + ps], base, 4, dims, str, box))) return rc;
      }
  }
  if (!p.has_shortcut && (rc = use_pairs(maps, a, in[1].ptr, (uint64_t)K, (uint64_t)p.cout))) return rc;
  if ((rc = enable_tma_out(maps, a))) return rc;
  use_resident_b(a);
  return launch_tc(maps, a, s);
}

// Tensor-core stem (tc_stem_kernel): Cout 64, Cin*kh*kw <= 32, bf16 output.
// Returns false when the shape is not eligible (the caller falls back).
// C3B200_STEM=mma selects the mma.sync stem instead (A/B timing).
bool launch_stem_tc(const c3b_tensor* in, const c3b_tensor& out, const c3b_stem_conv_params& p, cudaStream_t s,
                    int* rc) {
  static const bool off = [] {
    const char* e = getenv("C3B200_STEM");
    return e && std::string(e) == "mma";
  }();
  const c3b_stem_params& g = p.geom;
  *rc = C3B_OK;
  if (off || p.cout != 64 || g.c * g.g.kh * g.g.kw > 32 || ((uintptr_t)in[2].ptr & 15)) return false;
  const int64_t M = (int64_t)g.n * g.ho * g.wo;
  if (M >= ((int64_t)1 << 31)) return false;
  tc::TmaMaps maps;
  memset(&maps, 0, sizeof(maps));
  uint64_t dims[2] = {64, (uint64_t)M};
  uint64_t str[1] = {128};
  uint32_t box[2] = {64, 32};
  if ((*rc = encode(&maps.out, out.ptr, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return true;
  // whole images through shared memory (tc_stem_kernel<true>) for the 3x3 /
  // stride 1 / pad 1 stem of 32-pixel-wide images; C3B200_STEM=gather keeps
  // the per-pixel global gathers (A/B timing)
  static const bool img_off = [] {
    const char* e = getenv("C3B200_STEM");
    return e && std::string(e) == "gather";
  }();
  const bool img = !img_off && g.g.kh == 3 && g.g.kw == 3 && g.g.sh == 1 && g.g.sw == 1 && g.g.ph0 == 1 &&
                   g.g.pw0 == 1 && g.g.dh == 1 && g.g.dw == 1 && g.w == 32 && g.wo == 32 && g.ho == g.h &&
                   (g.h * 32) % 128 == 0 && g.c >= 1 && g.c <= 3 && g.c * g.h * 32 * 4 <= tc::STEM_IMG_BYTES &&
                   ((uintptr_t)in[0].ptr & 15) == 0;
  if (img) {
    uint64_t idims[4] = {32, (uint64_t)g.h, (uint64_t)g.c, (uint64_t)g.n};
    uint64_t istr[3] = {32 * 4, (uint64_t)g.h * 32 * 4, (uint64_t)g.c * g.h * 32 * 4};
    uint32_t ibox[4] = {32, (uint32_t)g.h, (uint32_t)g.c, 1};
    if ((*rc = encode(&maps.a[0], in[0].ptr, 4, idims, istr, ibox, CU_TENSOR_MAP_SWIZZLE_NONE,
                      CU_TENSOR_MAP_DATA_TYPE_FLOAT32)))
      return true;
    uint32_t hbox[2] = {32, 32};  // 32 channels x 32 pixels per TMA store
    if ((*rc = encode(&maps.b, out.ptr, 2, dims, str, hbox, CU_TENSOR_MAP_SWIZZLE_64B))) return true;
  }
  const size_t smem = 1024 + tc::STEM_STAGES * 16384 + 8192 + (img ? 8 : 4) * 4096 + (img ? tc::STEM_IMGS * tc::STEM_IMG_BYTES : 0) +
                      32 * 16 + (2 * tc::STEM_STAGES + 8 + 2 * tc::STEM_IMGS) * 8 + 16;
  static bool attr = false;
  if (!attr) {
    for (auto k : {tc::tc_stem_kernel<false>, tc::tc_stem_kernel<true>}) {
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      if (e != cudaSuccess) {
        *rc = fail(C3B_E_CUDA, std::string("stem attribute: ") + cudaGetErrorString(e));
        return true;
      }
    }
    attr = true;
  }
  const int n_tiles = (int)((M + 127) / 128);
  // Wait profiler (C3B200_STEM_PROF=1, measurement runs only): cycles summed
  // over warps, printed after a synchronous launch.
  static unsigned long long* prof = [] {
    const char* e = getenv("C3B200_STEM_PROF");
    unsigned long long* b = nullptr;
    if (e && e[0] == '1' && cudaMalloc(&b, 8 * sizeof(unsigned long long)) != cudaSuccess) b = nullptr;
    return b;
  }();
  if (prof && cudaMemsetAsync(prof, 0, 8 * sizeof(unsigned long long), s) != cudaSuccess) {
    *rc = fail(C3B_E_CUDA, "stem profiler reset");
    return true;
  }
  auto report = [&]() {
    if (!prof) return;
    unsigned long long h[8];
    if (cudaStreamSynchronize(s) != cudaSuccess || cudaMemcpy(h, prof, sizeof(h), cudaMemcpyDeviceToHost) != cudaSuccess)
      return;
    const double tiles = h[7] ? (double)h[7] / 4.0 : 1.0;  // 4 epilogue warps per tile
    fprintf(stderr,
            "[stem prof] img=%d per tile per warp (cycles): gather aempty %.0f ifull %.0f work %.0f | epilogue tfull "
            "%.0f math %.0f read-wait %.0f store %.0f | tiles %.0f\n",
            (int)img, h[0] / (tiles * 4), h[1] / (tiles * 4), h[2] / (tiles * 4), h[3] / (tiles * 4), h[4] / (tiles * 4),
            h[5] / (tiles * 4), h[6] / (tiles * 4), tiles);
  };
  if (img) {
    const int grid = g.n < sm_count() ? g.n : sm_count();
    *rc = launch_pdl(tc::tc_stem_kernel<true>, grid, tc::STEM_IMG_THREADS, smem, s, maps, (const float*)in[0].ptr,
                     (const float*)in[1].ptr, (const float*)in[2].ptr, g, p.act, M, n_tiles,
                     (int)(out.dtype == C3B_F16), prof);
    report();
    return true;
  }
  const int grid = n_tiles < sm_count() ? n_tiles : sm_count();
  *rc = launch_pdl(tc::tc_stem_kernel<false>, grid, tc::STEM_THREADS, smem, s, maps, (const float*)in[0].ptr,
                   (const float*)in[1].ptr, (const float*)in[2].ptr, g, p.act, M, n_tiles,
                   (int)(out.dtype == C3B_F16), prof);
  report();
  return true;
}

}  // namespace c3b

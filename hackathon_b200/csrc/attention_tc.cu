// tcgen05 / TMEM causal flash attention (bf16 profile, head_dim 64).
//
// Replaces, for the bf16 precision profile, the reference's materialised
// attention: fused_attention_scores_f32 (softmax(Q K^T / divisor + mask) into a
// [B, H, S, S] tensor, c35/engine.py:1250-1380) followed by the P.V matmul_f32
// (c32/kernel_registry.py:318-358) and the head merge.  Same contract as the
// other flash kernels: qkv [B, S, 3, H, 64] bf16 -> out [B, S, H*64] bf16 (or
// fp16 in and out for the fp16 profile).
//
// Design (persistent, two CTAs per SM, 10 warps and about 100 KB of shared
// memory each).  A work item is one (batch, head, 128-row query tile); items
// run heaviest (last) tile first.  Keys are processed in 64-key sub-tiles.
//   warp 0      TMA loads: Q once per item (two buffers, so the next item's Q
//               lands early), then K_j / V_j (128 keys x 64 dims, 128-byte
//               swizzle) into 2-stage K and V rings (K is read ahead by the S
//               products, V behind by the P.V products).
//   warp 1      allocates 256 TMEM columns and issues every tcgen05.mma from
//               one thread: S = Q K_u^T (M=128, N=64, K=64) into one of two
//               64-column S buffers, and O += P V_u (M=128, N=64, K=64; P read
//               from TMEM, V an MN-major shared-memory operand) into O's 64
//               columns.  The S products run two sub-tiles ahead of the P.V
//               products, across item boundaries, so the tensor core computes
//               the next scores while the softmax runs.
//   warps 2-9   softmax.  Each query row is one TMEM lane; the two warps of a
//               lane quarter (2+q and 6+q) split the 64 keys of a sub-tile and
//               the 64 O columns, and exchange partial row maxima through
//               shared memory.  Per sub-tile: tcgen05.ld 32 scores, release the
//               S buffer, causal mask on the diagonal tile, row max (three-input
//               maxima), exponentials half on the FMA pipe (degree-3
//               polynomial) and half on the SFU, row sum, P as bf16 pairs into
//               one of two 32-column P buffers in TMEM (tcgen05.st: the A
//               operand of P.V, no shared-memory round trip).  The running
//               maximum is raised lazily: only when a row's maximum grows by
//               more than 8 (log2 units) does the warp rescale its O columns in
//               TMEM, so P <= 2^8.  After the item's last sub-tile: O / l ->
//               bf16 rows of `out`.
// The two CTAs on an SM interleave: while one softmax group computes or waits
// at an item boundary, the other's work fills the SM.  Every mbarrier wait is
// bounded; on expiry the kernel records a status code, stops, and frees TMEM.
#include <cstdio>

#include "common.cuh"
#include "exp2.cuh"
#include "tc_prims.cuh"

namespace c3b {

namespace fat {
constexpr int D = 64;
constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int SUB = 64;        // keys per sub-tile (one S / P buffer)
constexpr int HALF = SUB / 2;  // keys per softmax warp and sub-tile
constexpr int NSK = 2;         // K stages
constexpr int NSV = 2;         // V stages
constexpr int THREADS = 320;   // loader, MMA, 8 softmax warps
constexpr int CTAS_PER_SM = 2;
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t TILE_BYTES = BQ * D * 2;  // 16 KB: 128 rows x 128 bytes
// shared-memory layout (offsets from a 1024-byte-aligned base)
constexpr uint32_t OFF_Q = 0;                       // two Q buffers
constexpr uint32_t OFF_K = OFF_Q + 2 * TILE_BYTES;
constexpr uint32_t OFF_V = OFF_K + NSK * TILE_BYTES;
constexpr uint32_t DATA_BYTES = OFF_V + NSV * TILE_BYTES;
// Metadata: barriers (256 B), profiler counters (128 B), row-max exchange
// [parity][half][128] (2 KB), row sums [half][128] (1 KB).  It goes in the
// alignment slack before the 1024-byte-aligned data when that is large
// enough, else right after the data.
constexpr uint32_t META_BAR = 0, META_PROF = 256, META_XMAX = 448, META_XSUM = 448 + 2048;
constexpr uint32_t META_BYTES = META_XSUM + 1024;
constexpr uint32_t SMEM_BYTES = DATA_BYTES + META_BYTES + 1024;
static_assert(2 * (SMEM_BYTES + 1024) <= 233472, "two CTAs fit an SM's shared memory");
// TMEM columns: two 64-column S buffers, O (64 columns), two 32-column P
// buffers (64 bf16 keys per row, two per 32-bit column)
constexpr uint32_t COL_S = 0, COL_O = 128, COL_P = 192;

struct Args {
  int batch, seq, heads, qtiles, n_items, causal;
  float scale_log2;  // softmax scale x log2(e)
  uint16_t* out;
  int h16;           // 16-bit format of qkv, P and out: 0 bf16, 1 fp16
  unsigned long long* prof;  // optional wait counters (C3B200_FLASH_PROF=1), else null
};

// Wait-profiler slots (cycles summed over softmax warps / MMA threads).
enum { PF_S_FULL = 0, PF_P_FREE, PF_LOOP, PF_SUBTILES, PF_MMA_SFREE, PF_MMA_PFULL, PF_MMA_LOAD, PF_MMA_TOTAL,
       PF_COUNT };
static_assert(PF_COUNT * 8 <= 128, "profiler counters fit their block");

// Work item w: one (batch, head, query tile), heaviest tiles first.
struct Item {
  int b, h, q, n;  // n = K/V tiles the query tile needs
};
__device__ __forceinline__ Item decode(const Args& a, int w) {
  Item it;
  const int bh_count = a.batch * a.heads;
  it.q = a.qtiles - 1 - w / bh_count;
  const int bh = w % bh_count;
  it.b = bh / a.heads;
  it.h = bh % a.heads;
  it.n = a.causal ? it.q + 1 : a.qtiles;
  return it;
}

// 32 consecutive fp32 TMEM columns of this thread's lane (one load, waited).
__device__ __forceinline__ void tmem_ld32v(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 16 columns from registers into this thread's TMEM lane.
__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// D (+)= A B with A (M=128 rows x K=16, bf16 pairs) read from TMEM and B from
// shared memory.
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accum) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accum));
}



__global__ void __launch_bounds__(THREADS, CTAS_PER_SM) flash_tc_kernel(const __grid_constant__ CUtensorMap qkv_map,
                                                                       const Args a) {
  using namespace tc;
  extern __shared__ uint8_t smem_raw[];
  const uintptr_t raw = reinterpret_cast<uintptr_t>(smem_raw);
  uint8_t* sm = reinterpret_cast<uint8_t*>((raw + 1023) & ~(uintptr_t)1023);
  uint8_t* meta = (reinterpret_cast<uintptr_t>(sm) - raw >= META_BYTES) ? smem_raw : sm + DATA_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(meta + META_BAR);
  uint64_t* k_full = bars;            // [NSK]
  uint64_t* k_empty = k_full + NSK;   // [NSK]
  uint64_t* v_full = k_empty + NSK;   // [NSV]
  uint64_t* v_empty = v_full + NSV;   // [NSV]
  uint64_t* q_full = v_empty + NSV;   // [item parity]
  uint64_t* q_empty = q_full + 2;     // [item parity]
  uint64_t* s_full = q_empty + 2;     // [buffer]
  uint64_t* s_free = s_full + 2;      // [buffer]
  uint64_t* p_full = s_free + 2;      // [buffer]
  uint64_t* p_free = p_full + 2;      // [buffer]
  uint64_t* o_free = p_free + 2;      // 1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_free + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  unsigned long long* prof_sm = reinterpret_cast<unsigned long long*>(meta + META_PROF);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool prof = a.prof != nullptr;
  if (threadIdx.x < PF_COUNT) prof_sm[threadIdx.x] = 0;
#define PROF_T0 const long long _t0 = prof ? clock64() : 0
#define PROF_ADD(slot) \
  do { if (prof && lane == 0) atomicAdd(&prof_sm[slot], (unsigned long long)(clock64() - _t0)); } while (0)
  if (threadIdx.x == 0) {
    for (int i = 0; i < NSK; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < NSV; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 8);
      mbar_init(&p_full[i], 8);
      mbar_init(&p_free[i], 1);
    }
    mbar_init(o_free, 8);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0 && lane == 0) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&qkv_map)));
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // every CTA of this persistent grid is resident: the next kernel may launch
  // onto SMs as they free up (it waits on griddepcontrol before its activations)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  const int H = a.heads;
  if (warp == 0) {
    // ------------------------------------------------ TMA loads
    if (lane == 0) {
      uint32_t kv = 0;  // global K/V tile counter
      int it_count = 0;
      for (int w = blockIdx.x; w < a.n_items; w += gridDim.x, ++it_count) {
        const Item it = decode(a, w);
        const int row0 = it.b * a.seq;
        const uint32_t qb = it_count & 1;
        // Q buffer qb is free once item it_count - 2 has issued every product reading it
        if (it_count > 1 && !mbar_wait(&q_empty[qb], (uint32_t)(((it_count - 2) >> 1) & 1), abort_flag, 21))
          goto load_done;
        mbar_arrive_tx(&q_full[qb], TILE_BYTES);
        tma_load_2d(sm + OFF_Q + qb * TILE_BYTES, &qkv_map, &q_full[qb], it.h * D, row0 + it.q * BQ);
        for (int j = 0; j < it.n; ++j, ++kv) {
          if (!mbar_wait(&k_empty[kv % NSK], ((kv / NSK) & 1) ^ 1, abort_flag, 22)) goto load_done;
          mbar_arrive_tx(&k_full[kv % NSK], TILE_BYTES);
          tma_load_2d(sm + OFF_K + (kv % NSK) * TILE_BYTES, &qkv_map, &k_full[kv % NSK], (H + it.h) * D,
                      row0 + j * BKV);
          if (!mbar_wait(&v_empty[kv % NSV], ((kv / NSV) & 1) ^ 1, abort_flag, 22)) goto load_done;
          mbar_arrive_tx(&v_full[kv % NSV], TILE_BYTES);
          tma_load_2d(sm + OFF_V + (kv % NSV) * TILE_BYTES, &qkv_map, &v_full[kv % NSV], (2 * H + it.h) * D,
                      row0 + j * BKV);
        }
      }
    load_done:;
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issue (one thread)
    // Sub-tile u of an item = keys 64u .. 64u+63 = half u&1 of K/V tile u>>1.
    // S of global sub-tile t goes to S buffer t&1, P to P buffer t&1.
    if (lane == 0) {
      const uint32_t id_s = instr_desc_h(BQ, SUB, a.h16);
      const uint32_t id_pv = instr_desc_h(BQ, D, a.h16) | (1u << 16);  // B (V) is MN-major
      const uint64_t q_desc0 = smem_desc(smem_u32(sm + OFF_Q));
      const uint64_t k_desc0 = smem_desc(smem_u32(sm + OFF_K));
      const uint64_t v_desc0 = smem_desc(smem_u32(sm + OFF_V));
      const long long t_mma0 = prof ? clock64() : 0;
      struct Stream {
        int k;        // item index in this CTA's sequence
        int w;        // work item
        int total;    // sub-tiles of the item
        int u;        // next sub-tile
        uint32_t kv;  // global K/V tile index of the item's first tile
      };
      Stream S{0, (int)blockIdx.x, 0, 0, 0}, P{0, (int)blockIdx.x, 0, 0, 0};
      if (S.w < a.n_items) S.total = P.total = 2 * decode(a, S.w).n;
      uint32_t ts = 0, tp = 0;
      bool ok = true;
      // issue the next S product of the S stream (false: stream done or failure)
      auto issue_s = [&]() -> bool {
        if (S.w >= a.n_items) return false;
        const uint32_t qb = S.k & 1;
        const uint32_t tile = S.kv + (uint32_t)(S.u >> 1);
        {
          PROF_T0;
          if (S.u == 0 && !mbar_wait(&q_full[qb], (uint32_t)((S.k >> 1) & 1), abort_flag, 23)) { ok = false; return false; }
          if ((S.u & 1) == 0 && !mbar_wait(&k_full[tile % NSK], (tile / NSK) & 1, abort_flag, 27)) { ok = false; return false; }
          PROF_ADD(PF_MMA_LOAD);
        }
        const uint32_t b = ts & 1;
        {
          PROF_T0;
          if (!mbar_wait(&s_free[b], ((ts >> 1) & 1) ^ 1, abort_flag, 24)) { ok = false; return false; }
          PROF_ADD(PF_MMA_SFREE);
        }
        tc_fence_after();
        const uint64_t qd = q_desc0 + (uint64_t)((qb * TILE_BYTES) >> 4);
        const uint64_t kd = k_desc0 + (uint64_t)(((tile % NSK) * TILE_BYTES + (S.u & 1) * (SUB * 128)) >> 4);
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          tc::mma_bf16(tmem + COL_S + 64u * b, qd + (uint64_t)(2 * k), kd + (uint64_t)(2 * k), id_s, k > 0);
        mma_commit(&s_full[b]);
        if (S.u & 1) mma_commit(&k_empty[tile % NSK]);  // both halves of the K tile consumed
        ++ts;
        if (++S.u == S.total) {  // every product reading this item's Q is issued
          mma_commit(&q_empty[qb]);
          S.kv += (uint32_t)(S.total >> 1);
          ++S.k;
          S.w += gridDim.x;
          S.u = 0;
          S.total = S.w < a.n_items ? 2 * decode(a, S.w).n : 0;
        }
        return true;
      };
      while (ok && P.w < a.n_items) {
        // keep S two sub-tiles ahead of the P.V about to be issued
        while (ok && ts < tp + 3 && issue_s()) {
        }
        if (!ok) break;
        const uint32_t b = tp & 1;
        const uint32_t tile = P.kv + (uint32_t)(P.u >> 1);
        {
          PROF_T0;
          if (!mbar_wait(&p_full[b], (tp >> 1) & 1, abort_flag, 25)) break;
          PROF_ADD(PF_MMA_PFULL);
        }
        // the softmax has read the previous item's O; the V tile has landed
        if (P.u == 0 && P.k > 0 && !mbar_wait(o_free, (uint32_t)((P.k - 1) & 1), abort_flag, 26)) break;
        if ((P.u & 1) == 0 && !mbar_wait(&v_full[tile % NSV], (tile / NSV) & 1, abort_flag, 27)) break;
        tc_fence_after();
        const uint64_t vd = v_desc0 + (uint64_t)(((tile % NSV) * TILE_BYTES + (P.u & 1) * (SUB * 128)) >> 4);
#pragma unroll
        for (int k = 0; k < SUB / 16; ++k)  // A = P from TMEM: 16 keys = 8 packed columns per step
          mma_ts(tmem + COL_O, tmem + COL_P + 32u * b + 8u * k, vd + (uint64_t)(k * (16 * 128 / 16)), id_pv,
                 (P.u > 0 || k > 0));
        mma_commit(&p_free[b]);
        if (P.u & 1) mma_commit(&v_empty[tile % NSV]);  // both halves of the V tile consumed
        ++tp;
        if (++P.u == P.total) {
          P.kv += (uint32_t)(P.total >> 1);
          ++P.k;
          P.w += gridDim.x;
          P.u = 0;
          P.total = P.w < a.n_items ? 2 * decode(a, P.w).n : 0;
        }
      }
      if (prof) atomicAdd(&prof_sm[PF_MMA_TOTAL], (unsigned long long)(clock64() - t_mma0));
    }
  } else {
    // ------------------------------------------------ softmax (warps 2-9)
    // Warp 2+q takes keys 0..31 of every sub-tile and O columns 0..31 of rows
    // 32q..32q+31, warp 6+q keys and O columns 32..63.  The pair exchanges
    // partial row maxima through shared memory (named barrier 1+q, 64
    // threads) so both use the same running maximum; the row sums are
    // combined once, at the epilogue.
    const int quarter = warp & 3;       // TMEM lanes 32*quarter .. +31
    const int half = (warp - 2) >> 2;   // which 32 keys / O columns
    const int r = quarter * 32 + lane;  // query row within the tile
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t taddr_o = tmem + lane_base + COL_O + 32u * half;
    float* xmax = reinterpret_cast<float*>(meta + META_XMAX);  // [parity][half][128]
    float* xsum = reinterpret_cast<float*>(meta + META_XSUM);  // [half][128]
    const uint32_t pair_bar = 1 + quarter;
    uint32_t t = 0;  // sub-tiles processed, across items
    float sa[HALF];  // this warp's 32 scores of the current sub-tile
    const float2 sc2 = make_float2(a.scale_log2, a.scale_log2);
    bool ok = true;
    const long long t_sm0 = prof ? clock64() : 0;
    for (int w = blockIdx.x; w < a.n_items && ok; w += gridDim.x) {
      const Item it = decode(a, w);
      if (prof && lane == 0) atomicAdd(&prof_sm[PF_SUBTILES], (unsigned long long)(2 * it.n));
      float m = -INFINITY, l = 0.f;
      for (int u = 0; u < 2 * it.n; ++u, ++t) {
        const uint32_t b = t & 1;
        {
          PROF_T0;
          if (!mbar_wait(&s_full[b], (t >> 1) & 1, abort_flag, 28)) { ok = false; break; }
          PROF_ADD(PF_S_FULL);
        }
        tc_fence_after();
        tmem_ld32v(tmem + lane_base + COL_S + 64u * b + 32u * half, sa);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[b]);
        if (a.causal && (u >> 1) == it.q) {  // diagonal K/V tile: keys past the row are masked
          const int k0 = (u & 1) * SUB + half * HALF;
#pragma unroll
          for (int c = 0; c < HALF; ++c)
            if (k0 + c > r) sa[c] = -INFINITY;
        }
        // partial row max over 32 keys, then the pair's
        static_assert(HALF == 32, "the max tree covers 32 scores");
        float mx8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx8[i] = fmax3f(sa[i], sa[i + 8], sa[i + 16]);
#pragma unroll
        for (int i = 0; i < 8; ++i) mx8[i] = fmaxf(mx8[i], sa[i + 24]);
        float mx = fmax3f(fmax3f(mx8[0], mx8[1], mx8[2]), fmax3f(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
        xmax[(b * 2 + half) * 128 + r] = mx;
        asm volatile("bar.sync %0, 64;" ::"r"(pair_bar) : "memory");
        mx = fmaxf(mx, xmax[(b * 2 + (half ^ 1)) * 128 + r]);
        mx *= a.scale_log2;
        const bool grow = mx > m + 8.0f;
        if (__any_sync(0xffffffffu, grow)) {
          const float mn = grow ? fmaxf(m, mx) : m;
          const float f = exp2_sfu(m - mn);  // 0 when m = -inf
          l *= f;
          m = mn;
          if (u > 0) {
            // every earlier P.V has landed in O; rescale this warp's 32 columns
            if (!mbar_wait(&p_free[(t - 1) & 1], ((t - 1) >> 1) & 1, abort_flag, 29)) { ok = false; break; }
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < 32; c += 16) {
              float o[16];
              tmem_ld16(taddr_o + (uint32_t)c, o);
              uint32_t ou[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) ou[i] = __float_as_uint(o[i] * f);
              tmem_st16u(taddr_o + (uint32_t)c, ou);
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
          }
        }
        {
          // P buffer b is free once the P.V of sub-tile t-2 has completed
          PROF_T0;
          if (!mbar_wait(&p_free[b], ((t >> 1) & 1) ^ 1, abort_flag, 30)) { ok = false; break; }
          PROF_ADD(PF_P_FREE);
        }
        // P = 2^(s * scale_log2 - m) -> bf16 pairs: this warp's 16 columns of P buffer b
        float2 sum2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        const float2 negm = make_float2(-m, -m);
        uint32_t pk[HALF / 2];
#pragma unroll
        for (int ch = 0; ch < HALF / 8; ++ch) {
          float2 e[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 z = __ffma2_rn(make_float2(sa[8 * ch + 2 * q], sa[8 * ch + 2 * q + 1]), sc2, negm);
            if (q < 2) {
              e[q] = exp2_fma2_p3(z);
            } else {
              e[q] = make_float2(exp2_sfu(z.x), exp2_sfu(z.y));
            }
            pk[4 * ch + q] = pack2h(e[q], a.h16);
          }
          sum2[ch & 1] = __fadd2_rn(sum2[ch & 1], __fadd2_rn(__fadd2_rn(e[0], e[1]), __fadd2_rn(e[2], e[3])));
        }
        const float2 sumv = __fadd2_rn(sum2[0], sum2[1]);
        l += sumv.x + sumv.y;
        tmem_st16u(tmem + lane_base + COL_P + 32u * b + 16u * half, pk);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[b]);
      }
      if (!ok) break;
      // epilogue: wait for the item's last P.V, read this warp's 32 O columns,
      // combine the pair's row sums, normalise, store
      if (!mbar_wait(&p_free[(t - 1) & 1], ((t - 1) >> 1) & 1, abort_flag, 31)) break;
      tc_fence_after();
      float* o = sa;  // the scores are dead here: reuse their registers for O's 32 columns
      tmem_ld32v(taddr_o, o);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free);
      xsum[half * 128 + r] = l;
      asm volatile("bar.sync %0, 64;" ::"r"(pair_bar) : "memory");
      const float inv = 1.0f / (l + xsum[(half ^ 1) * 128 + r]);
      asm volatile("bar.sync %0, 64;" ::"r"(pair_bar) : "memory");  // xsum is rewritten by the next item
      const int64_t token = (int64_t)it.b * a.seq + (int64_t)it.q * BQ + r;
      uint4* dst = reinterpret_cast<uint4*>(a.out + token * (int64_t)H * D + (int64_t)it.h * D + 32 * half);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint4 v;
        v.x = pack2h(make_float2(o[8 * c] * inv, o[8 * c + 1] * inv), a.h16);
        v.y = pack2h(make_float2(o[8 * c + 2] * inv, o[8 * c + 3] * inv), a.h16);
        v.z = pack2h(make_float2(o[8 * c + 4] * inv, o[8 * c + 5] * inv), a.h16);
        v.w = pack2h(make_float2(o[8 * c + 6] * inv, o[8 * c + 7] * inv), a.h16);
        dst[c] = v;
      }
    }
    if (prof && lane == 0) atomicAdd(&prof_sm[PF_LOOP], (unsigned long long)(clock64() - t_sm0));
  }

  tc_fence_before();
  __syncthreads();
  if (prof && threadIdx.x < PF_COUNT) atomicAdd(&a.prof[threadIdx.x], prof_sm[threadIdx.x]);
#undef PROF_T0
#undef PROF_ADD
  if (*abort_flag) {
    for (int i = 0; i < 1000; ++i) __nanosleep(1000);
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

}  // namespace fat

// The tcgen05 kernel takes bf16, head_dim 64 and whole 128-row tiles; other
// shapes keep the mma.sync kernel.
bool flash_tc_supported(const c3b_flash_params& p) {
  static const bool off = [] {
    const char* e = getenv("C3B200_FLASH_TC");
    return e && e[0] == '0';
  }();
  return !off && p.head_dim == fat::D && p.seq % fat::BQ == 0 && p.seq > 0;
}

int launch_flash_tc(const c3b_tensor& qkv, const c3b_tensor& out, const c3b_flash_params& p, cudaStream_t s) {
  C3B_REQUIRE((qkv.dtype == C3B_BF16 || qkv.dtype == C3B_F16) && out.dtype == qkv.dtype,
              "flash tc: bf16 or fp16, the same in and out");
  C3B_REQUIRE(((uintptr_t)qkv.ptr & 15) == 0 && ((uintptr_t)out.ptr & 15) == 0, "flash tc: 16-byte alignment");
  fat::Args a;
  a.batch = p.batch;
  a.seq = p.seq;
  a.heads = p.heads;
  a.qtiles = p.seq / fat::BQ;
  a.n_items = p.batch * p.heads * a.qtiles;
  a.causal = p.causal;
  a.scale_log2 = p.scale * 1.4426950408889634f;
  a.out = (uint16_t*)out.ptr;
  a.h16 = qkv.dtype == C3B_F16;
  a.prof = nullptr;
  if (a.n_items == 0) return C3B_OK;
  // Wait profiler (C3B200_FLASH_PROF=1, measurement runs only): cycles summed
  // over the softmax warps and MMA threads, printed after a synchronous launch.
  static unsigned long long* prof_buf = [] {
    const char* e = getenv("C3B200_FLASH_PROF");
    unsigned long long* p = nullptr;
    if (e && e[0] == '1' && cudaMalloc(&p, fat::PF_COUNT * sizeof(unsigned long long)) != cudaSuccess) p = nullptr;
    return p;
  }();
  if (prof_buf) {
    C3B_CHECK_CUDA(cudaMemsetAsync(prof_buf, 0, fat::PF_COUNT * sizeof(unsigned long long), s));
    a.prof = prof_buf;
  }
  CUtensorMap map;
  const uint64_t tokens = (uint64_t)p.batch * p.seq;
  const uint64_t width = (uint64_t)3 * p.heads * fat::D;
  uint64_t dims[2] = {width, tokens};
  uint64_t str[1] = {width * 2};
  uint32_t box[2] = {(uint32_t)fat::D, (uint32_t)fat::BQ};
  if (int rc = encode(&map, qkv.ptr, 2, dims, str, box)) return rc;
  static bool attr = false;
  if (!attr) {
    C3B_CHECK_CUDA(cudaFuncSetAttribute(fat::flash_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)fat::SMEM_BYTES));
    attr = true;
  }
  const int slots = fat::CTAS_PER_SM * sm_count();
  const int grid = a.n_items < slots ? a.n_items : slots;
  if (int rc = launch_pdl(fat::flash_tc_kernel, grid, fat::THREADS, (size_t)fat::SMEM_BYTES, s, map, a)) return rc;
  C3B_CHECK_CUDA(cudaGetLastError());
  if (prof_buf) {
    unsigned long long h[fat::PF_COUNT];
    C3B_CHECK_CUDA(cudaStreamSynchronize(s));
    C3B_CHECK_CUDA(cudaMemcpy(h, prof_buf, sizeof(h), cudaMemcpyDeviceToHost));
    const double warps = 8.0 * grid;
    const double sub = h[fat::PF_SUBTILES] ? (double)h[fat::PF_SUBTILES] : 1.0;  // summed over warps
    fprintf(stderr,
            "[flash_tc prof] per sub-tile per softmax warp (cycles): s_full %.0f p_free %.0f loop %.0f | "
            "per CTA: mma total %.0f (s_free %.0f p_full %.0f loads %.0f) | CTAs %d, sub-tiles/warp %.0f\n",
            h[fat::PF_S_FULL] / sub, h[fat::PF_P_FREE] / sub, h[fat::PF_LOOP] / sub,
            (double)h[fat::PF_MMA_TOTAL] / grid, (double)h[fat::PF_MMA_SFREE] / grid,
            (double)h[fat::PF_MMA_PFULL] / grid, (double)h[fat::PF_MMA_LOAD] / grid, grid, sub / warps);
  }
  return C3B_OK;
}

}  // namespace c3b

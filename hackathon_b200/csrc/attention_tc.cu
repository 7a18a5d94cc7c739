// tcgen05 / TMEM causal flash attention (bf16 profile, head_dim 64).
//
// Replaces, for the bf16 precision profile, the reference's materialised
// attention: fused_attention_scores_f32 (softmax(Q K^T / divisor + mask) into a
// [B, H, S, S] tensor, c35/engine.py:1250-1380) followed by the P.V matmul_f32
// (c32/kernel_registry.py:318-358) and the head merge.  Same contract as the
// other flash kernels: qkv [B, S, 3, H, 64] bf16 -> out [B, S, H*64] bf16.
//
// Design (persistent, one CTA per SM, 10 warps).  A work item is one
// (batch, head) and a pair of adjacent 128-row query tiles A = 2p, B = 2p + 1
// that share every K/V tile they both need; items run heaviest first.  The
// softmax works through 64-key sub-tiles (64 scores in registers per thread).
//   warp 0      TMA loads: Q_A, Q_B once per item, then K_j / V_j (128 keys x
//               64 dims, 128-byte swizzle) into a 3-stage ring.
//   warp 1      allocates 512 TMEM columns and issues every tcgen05.mma from
//               one thread: S_X = Q_X K_u^T (M=128, N=64, K=64) into one of
//               S_X's two 64-column buffers, and O_X += P_X V_u (M=128, N=64,
//               K=64, V as an MN-major operand) into O_X's 64 columns.  It
//               issues S of sub-tile u+2 before P.V of sub-tile u, so the tensor
//               core computes the next scores while the softmax runs.
//   warps 2-5   softmax of query tile A, warps 6-9 of tile B: thread = one
//               query row (its TMEM lane).  Per sub-tile: tcgen05.ld the 64
//               scores, release the S buffer, causal mask on the diagonal tile,
//               row max, exponentials half on the FMA pipe (polynomial) and half
//               on the SFU, row sum, P as bf16 into one of two shared-memory P
//               buffers (K-major, swizzled: the A operand of P.V).  The running
//               maximum is raised lazily: only when a row's maximum grows by
//               more than 8 (log2 units) does the warp rescale O in TMEM (ld,
//               scale, st), so P <= 2^8.  After the item's last sub-tile:
//               O / l -> bf16 rows of `out`.
// The two query tiles ping-pong: while one softmax group computes, the tensor
// core runs the other's products.  Every mbarrier wait is bounded; on expiry the
// kernel records a status code, stops, and frees TMEM.
#include <cstdio>

#include "common.cuh"
#include "exp2.cuh"
#include "tc_prims.cuh"

namespace c3b {

namespace fat {
constexpr int D = 64;
constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int NS = 3;
constexpr int THREADS = 320;
constexpr uint32_t TMEM_COLS = 512;
constexpr int SUB = 64;                      // keys per softmax step (one S / P buffer)
constexpr uint32_t TILE_BYTES = BQ * D * 2;  // 16 KB: 128 rows x 128 bytes
constexpr uint32_t P_SUB_BYTES = BQ * SUB * 2;  // 16 KB: 128 rows x 64 keys, K-major
constexpr uint32_t P_BYTES = 2 * P_SUB_BYTES;   // two P buffers per query tile
// shared-memory layout (offsets from a 1024-byte-aligned base)
constexpr uint32_t OFF_Q = 0;
constexpr uint32_t OFF_K = OFF_Q + 4 * TILE_BYTES;  // Q_A, Q_B of two items (double-buffered)
constexpr uint32_t OFF_V = OFF_K + NS * TILE_BYTES;
constexpr uint32_t OFF_P = OFF_V + NS * TILE_BYTES;
constexpr uint32_t OFF_BAR = OFF_P + 2 * P_BYTES;
constexpr uint32_t SMEM_BYTES = OFF_BAR + 256 + 1024;  // barriers + alignment slack

struct Args {
  int batch, seq, heads, qtiles, n_pairs, n_items, causal;
  float scale_log2;  // softmax scale x log2(e)
  __nv_bfloat16* out;
  unsigned long long* prof;  // optional per-role cycle counters (C3B200_FLASH_PROF=1), else null
};

// Cycle counters of the wait profiler (slot indices).
enum {
  PF_SM_SFULL = 0, PF_SM_LANDED, PF_SM_PFREE, PF_SM_RESCALE, PF_SM_TOTAL, PF_SM_EPI,
  PF_MMA_SFREE, PF_MMA_PFULL, PF_MMA_KV, PF_MMA_OFREE, PF_MMA_QFULL, PF_MMA_TOTAL,
  PF_LD_KVEMPTY, PF_LD_QEMPTY, PF_LD_TOTAL, PF_SUBTILES, PF_COUNT
};

// TMEM columns: S buffers of query tile x at 128x + 64b (64 fp32 columns each),
// O of query tile x at 256 + 64x.
__device__ __forceinline__ uint32_t tmem_col_s(int x, uint32_t b) { return (uint32_t)(x * 128) + 64u * b; }
__device__ __forceinline__ uint32_t tmem_col_o(int x) { return (uint32_t)(256 + x * 64); }

// Decode work item w: heaviest (last) query-tile pairs first.
struct Item {
  int b, h, qa, n[2];  // query tile A = qa, B = qa + 1; n[X] = key tiles of X (0: absent)
};
__device__ __forceinline__ Item decode(const Args& a, int w) {
  Item it;
  const int bh_count = a.batch * a.heads;
  const int p = a.n_pairs - 1 - w / bh_count;
  const int bh = w % bh_count;
  it.b = bh / a.heads;
  it.h = bh % a.heads;
  it.qa = 2 * p;
  const bool has_b = it.qa + 1 < a.qtiles;
  it.n[0] = a.causal ? it.qa + 1 : a.qtiles;
  it.n[1] = has_b ? (a.causal ? it.qa + 2 : a.qtiles) : 0;
  return it;
}

// 64 consecutive fp32 TMEM columns of this thread's lane (2 loads, one wait).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* v) {
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint32_t* r = reinterpret_cast<uint32_t*>(v + 32 * c);
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
          "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
          "=r"(r[30]), "=r"(r[31])
        : "r"(taddr + 32u * c));
  }
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Issue a 64-column load without waiting (tcgen05.wait::ld completes it).
__device__ __forceinline__ void tmem_ld64_nowait(uint32_t taddr, float* v) {
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint32_t* r = reinterpret_cast<uint32_t*>(v + 32 * c);
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
          "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
          "=r"(r[30]), "=r"(r[31])
        : "r"(taddr + 32u * c));
  }
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

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__global__ void __launch_bounds__(THREADS, 1) flash_tc_kernel(const __grid_constant__ CUtensorMap qkv_map,
                                                             const Args a) {
  using namespace tc;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* kv_full = bars;            // [NS]
  uint64_t* kv_empty = bars + NS;      // [NS]
  uint64_t* q_full = bars + 2 * NS;    // [item parity]
  uint64_t* q_empty = q_full + 2;      // [item parity]
  uint64_t* s_full = q_full + 4;       // [X][buffer]
  uint64_t* s_free = s_full + 4;       // [X][buffer]
  uint64_t* p_full = s_free + 4;       // [X][buffer]
  uint64_t* p_free = p_full + 4;       // [X][buffer]
  uint64_t* o_free = p_free + 4;       // [X]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_free + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  __shared__ unsigned long long prof_sm[PF_COUNT];
  const bool prof = a.prof != nullptr;
  if (threadIdx.x < PF_COUNT) prof_sm[threadIdx.x] = 0;
#define PROF_T0 const long long _t0 = prof ? clock64() : 0
#define PROF_ADD(slot) \
  do { if (prof && lane == 0) atomicAdd(&prof_sm[slot], (unsigned long long)(clock64() - _t0)); } while (0)
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&p_free[i], 1);
    }
    mbar_init(&o_free[0], 4);
    mbar_init(&o_free[1], 4);
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

  const int H = a.heads;
  if (warp == 0) {
    // ------------------------------------------------ TMA loads
    if (lane == 0) {
      uint32_t kv = 0;
      int it_count = 0;
      for (int w = blockIdx.x; w < a.n_items; w += gridDim.x, ++it_count) {
        const Item it = decode(a, w);
        const int row0 = it.b * a.seq;
        // Q buffer set it_count & 1 is free once item it_count - 2 has issued all its S products
        const uint32_t qb = it_count & 1;
        {
          PROF_T0;
          if (it_count > 1 && !mbar_wait(&q_empty[qb], (uint32_t)(((it_count - 2) >> 1) & 1), abort_flag, 21))
            goto load_done;
          PROF_ADD(PF_LD_QEMPTY);
        }
        mbar_arrive_tx(&q_full[qb], TILE_BYTES * (it.n[1] ? 2u : 1u));
        tma_load_2d(sm + OFF_Q + qb * 2 * TILE_BYTES, &qkv_map, &q_full[qb], it.h * D, row0 + it.qa * BQ);
        if (it.n[1])
          tma_load_2d(sm + OFF_Q + (qb * 2 + 1) * TILE_BYTES, &qkv_map, &q_full[qb], it.h * D,
                      row0 + (it.qa + 1) * BQ);
        const int nkv = it.n[1] > it.n[0] ? it.n[1] : it.n[0];
        for (int j = 0; j < nkv; ++j, ++kv) {
          const uint32_t st = kv % NS, ph = (kv / NS) & 1;
          {
            PROF_T0;
            if (!mbar_wait(&kv_empty[st], ph ^ 1, abort_flag, 22)) goto load_done;
            PROF_ADD(PF_LD_KVEMPTY);
          }
          mbar_arrive_tx(&kv_full[st], 2 * TILE_BYTES);
          tma_load_2d(sm + OFF_K + st * TILE_BYTES, &qkv_map, &kv_full[st], (H + it.h) * D, row0 + j * BKV);
          tma_load_2d(sm + OFF_V + st * TILE_BYTES, &qkv_map, &kv_full[st], (2 * H + it.h) * D, row0 + j * BKV);
        }
      }
    load_done:;
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issue (one thread)
    // Per query tile X the softmax works through 64-key sub-tiles u = 0, 1, ...
    // (sub-tile u = keys 64u .. 64u+63 = half u&1 of K/V tile u>>1).  S of
    // sub-tile u goes to S buffer u&1 (64 columns), P of sub-tile u to P
    // buffer u&1; counters t_s / t_p run across items so barrier parities do.
    if (lane == 0) {
      const uint32_t id_s = instr_desc(BQ, SUB);
      const uint32_t id_pv = instr_desc(BQ, D) | (1u << 16);  // B (V) is MN-major
      const uint64_t q_desc0 = smem_desc(smem_u32(sm + OFF_Q));
      const uint64_t p_desc0 = smem_desc(smem_u32(sm + OFF_P));
      const uint64_t k_desc0 = smem_desc(smem_u32(sm + OFF_K));
      const uint64_t v_desc0 = smem_desc(smem_u32(sm + OFF_V));
      const long long t_mma0 = prof ? clock64() : 0;
      uint32_t kv = 0, t_s[2] = {0, 0}, t_p[2] = {0, 0}, items_x[2] = {0, 0};
      int it_count = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < a.n_items && ok; w += gridDim.x, ++it_count) {
        const Item it = decode(a, w);
        const int nkv = it.n[1] > it.n[0] ? it.n[1] : it.n[0];
        const int n_s_total = 2 * (it.n[0] + it.n[1]);
        {
          PROF_T0;
          if (!mbar_wait(&q_full[it_count & 1], (uint32_t)((it_count >> 1) & 1), abort_flag, 23)) break;
          PROF_ADD(PF_MMA_QFULL);
        }
        tc_fence_after();
        const uint32_t qb = it_count & 1;
        const uint64_t q_desc[2] = {q_desc0 + (uint64_t)((qb * 2 * TILE_BYTES) >> 4),
                                    q_desc0 + (uint64_t)(((qb * 2 + 1) * TILE_BYTES) >> 4)};
        // Event loop: for each query tile, issue its next S product as soon as
        // an S buffer is free and its K/V tile has landed, and its next P.V as
        // soon as its P is written; neither tile waits for the other.
        int s_next[2] = {0, 0}, pv_next[2] = {0, 0};
        const int total[2] = {2 * it.n[0], 2 * it.n[1]};
        int kv_ready = 0, kv_released = 0, s_issued = 0;
        uint64_t idle_since = 0;
        while (pv_next[0] < total[0] || pv_next[1] < total[1]) {
          bool progress = false;
          while (kv_ready < nkv && mbar_test(&kv_full[(kv + kv_ready) % NS], ((kv + kv_ready) / NS) & 1)) {
            ++kv_ready;
            progress = true;
          }
          for (int x = 0; x < 2; ++x) {
            // S of the next sub-tile u (keys 64u .. 64u+63) into S buffer t&1
            const int u = s_next[x];
            if (u < total[x] && (u >> 1) < kv_ready) {
              const uint32_t t = t_s[x], b = t & 1;
              if (mbar_test(&s_free[2 * x + b], ((t >> 1) & 1) ^ 1)) {
                tc_fence_after();
                const uint32_t st = (kv + (u >> 1)) % NS;
                const uint64_t kd = k_desc0 + (uint64_t)((st * TILE_BYTES + (u & 1) * (SUB * 128)) >> 4);
#pragma unroll
                for (int k = 0; k < D / 16; ++k)
                  tc::mma_bf16(tmem + tmem_col_s(x, b), q_desc[x] + (uint64_t)(2 * k), kd + (uint64_t)(2 * k), id_s,
                               k > 0);
                mma_commit(&s_full[2 * x + b]);
                ++t_s[x];
                ++s_next[x];
                if (++s_issued == n_s_total) mma_commit(&q_empty[qb]);  // every product reading Q is issued
                progress = true;
              }
            }
            // P.V of the next sub-tile v once its P is written
            const int v = pv_next[x];
            if (v < s_next[x]) {
              const uint32_t t = t_p[x], b = t & 1;
              if (mbar_test(&p_full[2 * x + b], (t >> 1) & 1) &&
                  (v > 0 || items_x[x] == 0 || mbar_test(&o_free[x], (items_x[x] - 1) & 1))) {
                tc_fence_after();
                const uint32_t st = (kv + (v >> 1)) % NS;
                const uint64_t vd = v_desc0 + (uint64_t)((st * TILE_BYTES + (v & 1) * (SUB * 128)) >> 4);
                const uint64_t pd = p_desc0 + (uint64_t)(((2 * x + b) * P_SUB_BYTES) >> 4);
#pragma unroll
                for (int k = 0; k < SUB / 16; ++k)
                  tc::mma_bf16(tmem + tmem_col_o(x), pd + (uint64_t)(2 * k), vd + (uint64_t)(k * (16 * 128 / 16)),
                               id_pv, (v > 0 || k > 0));
                mma_commit(&p_free[2 * x + b]);
                ++t_p[x];
                ++pv_next[x];
                progress = true;
              }
            }
          }
          // K/V tile j is consumed once every query tile that needs it has
          // issued the P.V products of both its halves
          while (kv_released < nkv) {
            const int need = 2 * kv_released + 2;
            if ((it.n[0] > kv_released && pv_next[0] < need) || (it.n[1] > kv_released && pv_next[1] < need)) break;
            mma_commit(&kv_empty[(kv + kv_released) % NS]);
            ++kv_released;
            progress = true;
          }
          if (progress) {
            idle_since = 0;
          } else {
            // bounded like every other wait: nothing became ready for the limit
            __nanosleep(32);
            const uint64_t now = gtimer();
            if (idle_since == 0) {
              idle_since = now;
            } else if (now - idle_since > g_wait_limit_ns || *abort_flag) {
              *abort_flag = 1;
              atomicExch(&g_status, 24);
              ok = false;
              break;
            }
          }
        }
        kv += nkv;
        for (int x = 0; x < 2; ++x)
          if (it.n[x] > 0) ++items_x[x];
      }
      if (prof) atomicAdd(&prof_sm[PF_MMA_TOTAL], (unsigned long long)(clock64() - t_mma0));
    }
  } else {
    // ------------------------------------------------ softmax (warps 2-5: A, 6-9: B)
    const int x = (warp - 2) >> 2;
    const int quarter = warp & 3;            // TMEM lanes 32*quarter .. +31
    const int r = quarter * 32 + lane;       // query row within the tile
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t taddr_o = tmem + lane_base + tmem_col_o(x);
    uint32_t t = 0;  // sub-tiles processed by this query tile, across items
    float sa[SUB];  // the 64 scores of the current sub-tile
    const float2 sc2 = make_float2(a.scale_log2, a.scale_log2);
    bool ok = true;
    // Issue the TMEM load of sub-tile tt's scores (waits until they exist).
    auto fetch = [&](float* dst, uint32_t tt) -> bool {
      PROF_T0;
      if (!mbar_wait(&s_full[2 * x + (tt & 1)], (tt >> 1) & 1, abort_flag, 28)) return false;
      PROF_ADD(PF_SM_SFULL);
      tc_fence_after();
      tmem_ld64_nowait(tmem + lane_base + tmem_col_s(x, tt & 1), dst);
      return true;
    };
    // The scores of sub-tile tt are in registers: hand its S buffer back.
    auto landed = [&](uint32_t tt) {
      PROF_T0;
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      PROF_ADD(PF_SM_LANDED);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[2 * x + (tt & 1)]);
    };
    const long long t_sm0 = prof ? clock64() : 0;
    for (int w = blockIdx.x; w < a.n_items && ok; w += gridDim.x) {
      const Item it = decode(a, w);
      const int n = it.n[x];
      if (n == 0) continue;
      if (prof && lane == 0) atomicAdd(&prof_sm[PF_SUBTILES], (unsigned long long)(2 * n));
      const int qtile = it.qa + x;
      float m = -INFINITY, l = 0.f;
      // softmax of one 64-key sub-tile u (global index tt) held in s
      auto process = [&](float* s, int u, uint32_t tt) -> bool {
        const uint32_t b = tt & 1;
        if (a.causal && (u >> 1) == qtile) {  // diagonal K/V tile: keys past the row are masked
          const int k0 = (u & 1) * SUB;
#pragma unroll
          for (int c = 0; c < SUB; ++c)
            if (k0 + c > r) s[c] = -INFINITY;
        }
        // row max as a tree (eight independent chains, not one 63-deep chain)
        float mx8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx8[i] = fmaxf(s[i], s[i + 8]);
#pragma unroll
        for (int c = 16; c < SUB; c += 8) {
#pragma unroll
          for (int i = 0; i < 8; ++i) mx8[i] = fmaxf(mx8[i], s[c + i]);
        }
        float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                         fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        mx *= a.scale_log2;
        const bool grow = mx > m + 8.0f;
        if (__any_sync(0xffffffffu, grow)) {
          PROF_T0;
          const float mn = grow ? fmaxf(m, mx) : m;
          const float f = exp2_sfu(m - mn);  // 0 when m = -inf
          l *= f;
          m = mn;
          if (u > 0) {
            // every earlier P.V has landed in O; rescale it 16 columns at a time
            if (!mbar_wait(&p_free[2 * x + ((tt - 1) & 1)], ((tt - 1) >> 1) & 1, abort_flag, 29)) return false;
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < 64; c += 16) {
              float o[16];
              tmem_ld16(taddr_o + (uint32_t)c, o);
#pragma unroll
              for (int i = 0; i < 16; ++i) o[i] *= f;
              tmem_st16(taddr_o + (uint32_t)c, o);
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
          }
          PROF_ADD(PF_SM_RESCALE);
        }
        // P buffer b is free once the P.V of sub-tile tt-2 has completed
        {
          PROF_T0;
          if (!mbar_wait(&p_free[2 * x + b], ((tt >> 1) & 1) ^ 1, abort_flag, 30)) return false;
          PROF_ADD(PF_SM_PFREE);
        }
        // P = 2^(s * scale_log2 - m) -> bf16, K-major 64 keys (one 128-byte swizzled row)
        uint8_t* prow = sm + OFF_P + (2 * x + b) * P_SUB_BYTES + (r >> 3) * 1024 + (r & 7) * 128;
        float2 sum2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        const float2 negm = make_float2(-m, -m);
#pragma unroll
        for (int ch = 0; ch < SUB / 8; ++ch) {
          float2 e[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 z = __ffma2_rn(make_float2(s[8 * ch + 2 * q], s[8 * ch + 2 * q + 1]), sc2, negm);
            if (q < 2) {
              e[q] = exp2_fma2(z);
            } else {
              e[q] = make_float2(exp2_sfu(z.x), exp2_sfu(z.y));
            }
          }
          sum2[ch & 1] = __fadd2_rn(sum2[ch & 1], __fadd2_rn(__fadd2_rn(e[0], e[1]), __fadd2_rn(e[2], e[3])));
          uint4 pk;
          pk.x = pack2(e[0].x, e[0].y);
          pk.y = pack2(e[1].x, e[1].y);
          pk.z = pack2(e[2].x, e[2].y);
          pk.w = pack2(e[3].x, e[3].y);
          *reinterpret_cast<uint4*>(prow + ((ch ^ (r & 7)) << 4)) = pk;
        }
        const float2 sumv = __fadd2_rn(sum2[0], sum2[1]);
        l += sumv.x + sumv.y;
        fence_proxy_async();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[2 * x + b]);
        return true;
      };
      for (int u = 0; u < 2 * n; ++u, ++t) {
        if (!fetch(sa, t)) { ok = false; break; }
        landed(t);
        if (!process(sa, u, t)) { ok = false; break; }
      }
      if (!ok) break;
      // epilogue: wait for the item's last P.V, read O, normalise, store
      if (!mbar_wait(&p_free[2 * x + ((t - 1) & 1)], ((t - 1) >> 1) & 1, abort_flag, 31)) break;
      tc_fence_after();
      {
        float* o = sa;  // the scores are dead here: reuse their registers for O's 64 columns
        tmem_ld64(taddr_o, o);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_free[x]);
        const float inv = 1.0f / l;
        const int64_t token = (int64_t)it.b * a.seq + (int64_t)qtile * BQ + r;
        uint4* dst = reinterpret_cast<uint4*>(a.out + token * (int64_t)H * D + (int64_t)it.h * D);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4 v;
          v.x = pack2(o[8 * c] * inv, o[8 * c + 1] * inv);
          v.y = pack2(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
          v.z = pack2(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
          v.w = pack2(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
          dst[c] = v;
        }
      }
    }
    if (prof && lane == 0) atomicAdd(&prof_sm[PF_SM_TOTAL], (unsigned long long)(clock64() - t_sm0));
  soft_done:;
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
  C3B_REQUIRE(qkv.dtype == C3B_BF16 && out.dtype == C3B_BF16, "flash tc: bf16 in and out");
  C3B_REQUIRE(((uintptr_t)qkv.ptr & 15) == 0 && ((uintptr_t)out.ptr & 15) == 0, "flash tc: 16-byte alignment");
  fat::Args a;
  a.batch = p.batch;
  a.seq = p.seq;
  a.heads = p.heads;
  a.qtiles = p.seq / fat::BQ;
  a.n_pairs = (a.qtiles + 1) / 2;
  a.n_items = p.batch * p.heads * a.n_pairs;
  a.causal = p.causal;
  a.scale_log2 = p.scale * 1.4426950408889634f;
  a.out = (__nv_bfloat16*)out.ptr;
  a.prof = nullptr;
  if (a.n_items == 0) return C3B_OK;
  // Wait profiler (C3B200_FLASH_PROF=1, measurement builds only): per-role
  // cycles summed over CTAs, printed to stderr after a synchronous launch.
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
  const int grid = a.n_items < sm_count() ? a.n_items : sm_count();
  if (int rc = launch_pdl(fat::flash_tc_kernel, grid, fat::THREADS, (size_t)fat::SMEM_BYTES, s, map, a)) return rc;
  C3B_CHECK_CUDA(cudaGetLastError());
  if (prof_buf) {
    unsigned long long h[fat::PF_COUNT];
    C3B_CHECK_CUDA(cudaStreamSynchronize(s));
    C3B_CHECK_CUDA(cudaMemcpy(h, prof_buf, sizeof(h), cudaMemcpyDeviceToHost));
    const double sub = (double)(h[fat::PF_SUBTILES] ? h[fat::PF_SUBTILES] : 1);
    fprintf(stderr,
            "[flash_tc prof] per sub-tile per softmax warp (cycles): s_full %.0f landed %.0f p_free %.0f rescale %.0f "
            "loop %.0f (sum over the item loop) | per CTA: mma total %.0f (s_free %.0f p_full %.0f kv %.0f o_free %.0f q_full %.0f) "
            "loader total %.0f (kv_empty %.0f q_empty %.0f) | sub-tiles %.0f, CTAs %d\n",
            h[0] / sub, h[1] / sub, h[2] / sub, h[3] / sub, h[4] / sub, (double)h[11] / grid, (double)h[6] / grid,
            (double)h[7] / grid, (double)h[8] / grid, (double)h[9] / grid, (double)h[10] / grid,
            (double)h[14] / grid, (double)h[12] / grid, (double)h[13] / grid, sub, grid);
  }
  return C3B_OK;
}

}  // namespace c3b

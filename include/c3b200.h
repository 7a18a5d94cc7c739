/*
 * c3b200 — B200-native C-ABI for the C3.5 numerical hot path.
 *
 * This library replaces two things in the reference (zhenlu1936/Hackathon):
 *
 *  1. Every kernel of the C3.2 kernel registry.  The reference ABI is the
 *     Python call  kernel(inputs, outputs, params, tuning)
 *     (c32/kernel_registry.py:6-16, 42-67), dispatched from
 *     PlannedGraphExecutor._execute_planned_node (c35/executor.py:514-604).
 *     Here it is one entry point, c3b_launch(), taking raw device pointers and
 *     an explicit stream (the reference used CuPy's implicit current stream,
 *     c35/executor.py:843-846).
 *
 *  2. The C3.4 timeline interpreter PlannedGraphExecutor.run_planned
 *     (c35/executor.py:723-903).  The c3b_plan_* entry points take a flattened
 *     timeline (arena offsets, H2D / KERNEL / EVENT_RECORD / EVENT_WAIT / D2H
 *     actions on logical streams) and execute it natively on real CUDA streams
 *     and events, optionally replayed as one CUDA graph.
 *
 * Conventions: every function returns 0 on success or a negative C3B_E* code;
 * c3b_last_error() returns the calling thread's last message.  Tensors are
 * dense row-major (C-contiguous).  No function aborts the process.
 */
#ifndef C3B200_H
#define C3B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define C3B_MAX_RANK 8

/* status codes */
#define C3B_OK 0
#define C3B_E_INVALID (-1)   /* bad argument / shape / dtype */
#define C3B_E_UNKNOWN (-2)   /* unknown kernel name or id (kernel_registry.py:65-67) */
#define C3B_E_CUDA (-3)      /* CUDA runtime error */
#define C3B_E_DEVICE (-4)    /* a kernel reported an error through the device status word */
#define C3B_E_UNSUPPORTED (-5)

typedef enum {
  C3B_F32 = 0,
  C3B_BF16 = 1,
  C3B_F16 = 2,
  C3B_I64 = 3,
  C3B_I32 = 4,
  C3B_U8 = 5
} c3b_dtype;

/* A dense tensor.  In plan records (c3b_plan_add_kernel) `ptr` holds a byte
 * offset into the plan arena when (flags & C3B_TENSOR_ARENA). */
#define C3B_TENSOR_ARENA 1
typedef struct {
  void* ptr;
  int32_t dtype;
  int32_t ndim;
  int64_t shape[C3B_MAX_RANK];
  int32_t flags;
  int32_t _pad;
} c3b_tensor;

/* ------------------------------------------------------------------ kernels
 * Kernel ids.  Names of the reference registry map onto these through
 * c3b_kernel_id() (name + the _f32/_fp32 alias rules of
 * c32/kernel_registry.py:42-67); the Python registry supplies the parameter
 * block built from the reference's operator_params. */
enum {
  C3B_K_EW = 1,          /* broadcasting elementwise program            */
  C3B_K_COPY = 2,        /* strided gather copy with dtype cast          */
  C3B_K_IM2COL = 3,      /* NCHW -> [N*Ho*Wo, C*kh*kw]                   */
  C3B_K_REDUCE = 4,      /* [outer, R, inner] mean / sum / max            */
  C3B_K_GEMM = 5,        /* SIMT GEMM (fp32 math), batched, epilogue     */
  C3B_K_LAYERNORM = 6,   /* LayerNorm (+residual) over the last axis      */
  C3B_K_SOFTMAX = 7,     /* softmax over one axis                         */
  C3B_K_ATTN_SCORES = 8, /* softmax(QK^T/div + mask), materialised         */
  C3B_K_GATHER = 9,      /* np.take along one axis                        */
  C3B_K_CONV = 10,       /* SIMT implicit-GEMM conv, NCHW or NHWC, epilogue */
  C3B_K_GEMM_TC = 11,    /* tcgen05/TMEM bf16 GEMM, TMA-fed, epilogue    */
  C3B_K_CONV_TC = 12,    /* tcgen05/TMEM bf16 implicit-GEMM conv, NHWC   */
  C3B_K_FLASH_ATTN = 13, /* causal flash attention on packed QKV          */
  C3B_K_EMBED = 14,      /* token-row gather + position add               */
  C3B_K_STEM_IM2COL = 15,/* NCHW f32 -> bf16 [N*Ho*Wo, Kpad] patch matrix */
  C3B_K_GAP_NHWC = 16,   /* NHWC mean over H,W -> [N, C]                  */
  C3B_K_STEM_CONV = 17,  /* direct small-Cin conv NCHW f32 -> NHWC bf16    */
  C3B_K_QUANT_E4M3 = 18, /* rowwise e4m3 quantisation (fp8 precision path) */
  C3B_K_GEMM_FP8 = 19,   /* e4m3 x e4m3 tcgen05 GEMM, scaled epilogue      */
  C3B_K_QUANT_FP4 = 20,  /* FP4 E2M1 weight quantisation (W4A16 path)      */
  C3B_K_GEMM_W4A16 = 21, /* bf16 x FP4-weight tcgen05 GEMM (W4A16)         */
  C3B_K_DEQUANT_FP4 = 22,/* FP4 weights -> bf16 (W4A16 at large M)         */
  C3B_K_WAIT_PROBE = 23, /* failure-path probe: a bounded wait that expires */
  C3B_K_GEMM_TF32 = 24,  /* fp32 x fp32 tcgen05 GEMM as tf32 (kind::tf32) */
  C3B_K_COUNT = 25
};

/* --- C3B_K_EW: out = program(in0..in5) with NumPy broadcasting.
 * Each op: code, a, b.  Operand encoding: v >= 0 → input v; v < 0 → result of
 * op (-v - 1); for C3B_OP_*_IMM the second operand is imm[b]. */
enum {
  C3B_OP_ADD = 0, C3B_OP_SUB, C3B_OP_MUL, C3B_OP_DIV, C3B_OP_RELU, C3B_OP_ERF,
  C3B_OP_ERF_AS, C3B_OP_SQRT, C3B_OP_EXP, C3B_OP_RECIP, C3B_OP_ADD_IMM,
  C3B_OP_MUL_IMM, C3B_OP_MAX_IMM, C3B_OP_COPY
};
#define C3B_EW_MAX_OPS 12
#define C3B_EW_MAX_IN 6
typedef struct {
  int32_t n_ops;
  int32_t _pad;
  int32_t op[C3B_EW_MAX_OPS];
  int32_t a[C3B_EW_MAX_OPS];
  int32_t b[C3B_EW_MAX_OPS];
  float imm[C3B_EW_MAX_OPS];
} c3b_ew_params;

/* --- C3B_K_COPY: out[idx] = cast(in[offset + sum_k coord_k(idx) * in_stride[k]])
 * over out's shape (rank = out.ndim).  Covers transpose, split slices,
 * NHWO->NCHW reshapes, layout changes and dtype casts. */
typedef struct {
  int64_t in_offset;
  int64_t in_stride[C3B_MAX_RANK];
} c3b_copy_params;

/* --- C3B_K_IM2COL (c32/kernel_registry.py:399-453) and conv geometry. */
typedef struct {
  int32_t kh, kw, sh, sw, ph0, pw0, ph1, pw1, dh, dw;
} c3b_conv_geom;

/* --- C3B_K_REDUCE */
enum { C3B_RED_MEAN = 0, C3B_RED_SUM = 1, C3B_RED_MAX = 2 };
typedef struct {
  int64_t outer, reduce, inner;
  int32_t op;
  int32_t _pad;
} c3b_reduce_params;

/* --- epilogue shared by GEMM / conv kernels */
enum { C3B_ACT_NONE = 0, C3B_ACT_RELU = 1, C3B_ACT_GELU = 2 };
enum {
  C3B_BIAS_NONE = 0, C3B_BIAS_COL = 1 /* [N] */, C3B_BIAS_ROW = 2 /* [M] */,
  C3B_BIAS_FULL = 3 /* [M,N] */, C3B_BIAS_SCALAR = 4
};

/* --- C3B_K_GEMM: C[b] = act(alpha * op(A[b]) op(B[b]) + beta * bias + residual)
 * A is [M,K] (or [K,M] when trans_a), B is [K,N] (or [N,K] when trans_b).
 * batch strides in elements; 0 broadcasts one operand across the batch.
 * inputs: A, B, [bias if bias_mode], [residual if has_residual] ; output: C. */
typedef struct {
  int64_t M, N, K, batch;
  int64_t stride_a, stride_b, stride_c;
  int32_t trans_a, trans_b;
  float alpha, beta;
  int32_t bias_mode, act, has_residual, _pad;
} c3b_gemm_params;

/* --- C3B_K_LAYERNORM: rows x cols, optional residual (LN(x + r)), bias.
 * inputs: x, [residual], scale, [bias] ; outputs: y, [x+r when write_sum].
 * fp8 path: when outputs[0] is u8 the outputs are E4M3 bytes [rows, cols] and
 * f32 row scales [rows] with C3B_K_QUANT_E4M3's rowwise scheme applied to the
 * fp32 normalised values (cols 128, 256, 512, 1024 or 2048). */
typedef struct {
  int64_t rows, cols;
  float epsilon;
  int32_t has_residual, has_bias, write_sum;
} c3b_layernorm_params;

/* --- C3B_K_SOFTMAX: [outer, axis, inner] */
typedef struct {
  int64_t outer, axis, inner;
} c3b_softmax_params;

/* --- C3B_K_ATTN_SCORES (c35/engine.py:1250-1380); inputs q, kT, divisor, mask.
 * Broadcast extents follow the reference kernel's argument list. */
typedef struct {
  int32_t q0, q1, k0, k1, rows, cols, inner, out0, out1;
  int32_t m[4];
  int32_t _pad;
} c3b_attn_scores_params;

/* --- C3B_K_GATHER: out[o, j, i] = data[o, idx[j], i] (idx int64 or int32,
 * negative indices wrap as in np.take). */
typedef struct {
  int64_t outer, axis_len, n_idx, inner;
} c3b_gather_params;

/* --- C3B_K_CONV: SIMT implicit-GEMM convolution with fused epilogue.
 * inputs: x, w [Cout, Cin, kh, kw] (layout 0) or [Cout, kh, kw, Cin] (layout 1),
 * [bias [Cout]], [residual shaped like out] ; output y.
 * layout 0 = NCHW activations, 1 = NHWC. */
typedef struct {
  int32_t n, c, h, w, cout, ho, wo, layout;
  c3b_conv_geom g;
  int32_t has_bias, has_residual, act, _pad;
} c3b_conv_params;

/* --- C3B_K_GEMM_TC: bf16 x bf16 -> fp32 accumulate in TMEM.
 * A [M,K] bf16 row-major, B [N,K] bf16 row-major (i.e. both K-major).
 * inputs: A, B, [bias f32 [N]], [residual [M,N] f32|bf16] ; output C [M,N] f32|bf16.
 * K % 8 == 0, N % 32 == 0; M arbitrary. */
typedef struct {
  int64_t M, N, K;
  int32_t bias_mode, act, has_residual, block_n;
} c3b_gemm_tc_params;

/* --- C3B_K_CONV_TC: NHWC bf16 implicit GEMM, K ordered (kh, kw, Cin).
 * inputs: x [N,H,W,Cin] bf16, w [Cout, kh, kw, Cin] bf16, bias f32 [Cout],
 * [residual [N,Ho,Wo,Cout] bf16] ; output y [N,Ho,Wo,Cout] bf16.
 * Cin % 64 == 0, Cout % 32 == 0, stride 1 or 2 (H, W even for stride 2),
 * square kernel, symmetric padding.
 * has_shortcut = 1 (stride 2, pad = k / 2, Cout 64 or 128, no residual): the launch also
 * computes the 1x1 stride-2 convolution of the same input (a residual block's
 * downsampling shortcut), which samples exactly the pixels of the centre tap.
 * Two more inputs follow: ws [Cout, Cin] bf16, bs [Cout] f32; and a second
 * output ys [N,Ho,Wo,Cout] bf16 = conv1x1(x) + bs with no activation. */
typedef struct {
  int32_t n, h, w, cin, cout, ho, wo, k, stride, pad;
  int32_t has_residual, act, block_n;
  int32_t mode; /* 0: fastest eligible path: row-ring halo (3x3 s1 p1, Cin = Cout = 64), halo
                   tiles (3x3 s1 p1, Cout <= 128, weights resident when they fit), else one TMA
                   window per tap; 1: one TMA window per tap; 2: halo tiles, streamed weights;
                   3: halo tiles, resident weights, no row ring */
  int32_t has_shortcut;
} c3b_conv_tc_params;

/* --- C3B_K_FLASH_ATTN: qkv [B, S, 3, H, D] (f32 or bf16) -> out [B, S, H*D].
 * causal softmax(q k^T * scale) v. */
typedef struct {
  int32_t batch, seq, heads, head_dim;
  float scale;
  int32_t causal;
} c3b_flash_params;

/* --- C3B_K_EMBED: out[b,s,:] = tok[ids[b,s],:] + pos[s,:] */
typedef struct {
  int64_t batch, seq, dim, vocab;
} c3b_embed_params;

/* --- C3B_K_STEM_IM2COL: x NCHW f32 [N,C,H,W] -> [N*Ho*Wo, kpad] bf16 with
 * K ordered (kh, kw, C) and zero padding from kh*kw*C to kpad. */
typedef struct {
  int32_t n, c, h, w, ho, wo, kpad, _pad;
  c3b_conv_geom g;
  int32_t _pad2[2];
} c3b_stem_params;

/* --- C3B_K_STEM_CONV: inputs x NCHW f32, w [K][Cout] f32 (K ordered c, kh, kw;
 * K <= 64), bias f32 [Cout]; output [N*Ho*Wo, Cout] bf16 = act(conv + bias).
 * Cout in {16, 32, 64}. */
typedef struct {
  c3b_stem_params geom;
  int32_t cout, act;
} c3b_stem_conv_params;

/* --- C3B_K_QUANT_E4M3: x [M,K] f32|bf16 -> q [M,K] u8 (OCP E4M3 bytes) and
 * scale [M] f32: scale[m] = max|x[m,:]| / 448 (1 for an all-zero row),
 * q[m,k] = e4m3(x[m,k] / scale[m]) rounded to nearest even, saturating.
 * K % 16 == 0.  No reference counterpart: the reference policy names fp8
 * (c32/strategy.py:124-160) but has no fp8 kernel. */
typedef struct {
  int64_t M, K;
} c3b_quant_params;

/* --- C3B_K_GEMM_FP8: C = (A·Bᵀ) * a_scale[m] * b_scale[n] (+ bias[n]) (+ residual)
 * then act, with A [M,K] and B [N,K] e4m3 bytes (both K-major) from
 * C3B_K_QUANT_E4M3, fp32 accumulation in TMEM.  inputs: A, B, a_scale f32 [M],
 * b_scale f32 [N], [bias f32 [N]], [residual [M,N] f32|bf16]; output f32|bf16.
 * Parameters: c3b_gemm_tc_params.  K % 16 == 0, N % 32 == 0.  Executes the
 * reference's "matmul_f8" name (which the reference cannot run). */

/* --- C3B_K_QUANT_FP4: w [N,K] f32|bf16 -> q [N,K/2] u8 (two FP4 E2M1 codes per
 * byte, element 2i in the low nibble) and scale f32 laid out [K/64][N][4]:
 * scale of group g (16 K elements) of row n at ((g/4)*N + n)*4 + g%4;
 * scale = max|group| / 6 (1 for an all-zero group), code = E2M1(w / scale)
 * round-to-nearest-even, saturating.  K % 64 == 0.  Parameters:
 * c3b_quant_params, with M = N rows.  No reference counterpart: the reference
 * policy names fp4 as W4A16 (c32/strategy.py:98-119, 150-154) without a kernel.
 *
 * --- C3B_K_GEMM_W4A16: C = A · dequant(B)ᵀ (+ bias) (+ residual), act, with A
 * [M,K] bf16 and B the output of C3B_K_QUANT_FP4; dequant(B)[n,k] =
 * bf16(E2M1 value × group scale); fp32 accumulation in TMEM.  inputs: A, q, scale,
 * [bias f32 [N]], [residual]; output f32|bf16.  Parameters: c3b_gemm_tc_params.
 * K % 64 == 0, N % 32 == 0.  Executes the reference's "matmul_f4" name.
 *
 * --- C3B_K_DEQUANT_FP4: (q, scale) from C3B_K_QUANT_FP4 -> w [N,K] bf16, the
 * same effective weights the W4A16 GEMM expands next to its MMA.  With many
 * rows per call (M in the thousands) expanding once and running C3B_K_GEMM_TC
 * costs less than re-expanding the weights for every 128-row tile.
 * Parameters: c3b_quant_params, with M = N rows.  No reference counterpart. */

/* --- C3B_K_GEMM_TF32: C = act(A B^T + bias [+ residual]) with A [M,K] and
 * B [N,K] f32 read by the tensor cores as tf32 (10-bit mantissa), fp32
 * accumulation in TMEM, f32 output; c3b_gemm_tc_params, K % 4 == 0,
 * N % 32 == 0.  The tf32 precision profile's contraction (the fp32 C3.5
 * contractions, c35/engine.py:722-849, at tensor-core rate). */

/* --- C3B_K_WAIT_PROBE: no tensors.  One thread waits on an mbarrier that is
 * never armed, through the bounded wait every tcgen05 kernel uses; when the
 * limit expires it writes `code` to the device status word and returns.  No
 * counterpart in the reference: it exists to test the failure path
 * (c3b_plan_sync / c3b_device_status report C3B_E_DEVICE) without a fault. */
typedef struct { int32_t code; } c3b_wait_probe_params;

/* --- C3B_K_GAP_NHWC: x [N, HW, C] -> y [N, C] f32.  With two or three inputs
 * (x bf16/fp16, w [classes, C] f32, optional b [classes] f32; C a multiple of
 * 256 up to 1024) the classifier follows in the same launch:
 * y [N, classes] = mean_hw(x) w^T + b (GlobalAveragePool -> Flatten -> Gemm). */
typedef struct {
  int64_t n, hw, c;
} c3b_gap_params;

/* ------------------------------------------------------------- entry points */

/* Library / device info.  c3b_version returns the ABI version (1). */
int c3b_version(void);
const char* c3b_last_error(void);
/* Resolve a reference kernel name (c32/kernel_registry.py:42-67 alias rules)
 * to the id of the kernel family that implements it; C3B_E_UNKNOWN if none. */
int c3b_kernel_id(const char* name);
/* Launch one kernel on `stream` (a cudaStream_t; NULL = legacy default).
 * Replaces kernel(inputs, outputs, params, tuning) (c35/executor.py:576-581). */
int c3b_launch(int kernel_id, const c3b_tensor* in, int n_in, const c3b_tensor* out, int n_out,
               const void* params, size_t params_len, void* stream);
/* Read and clear the device-side status word set by kernels whose bounded
 * waits expired (0 = none).  Synchronises the device. */
int c3b_device_status(int* status);
/* Number of streaming multiprocessors of the current device. */
int c3b_sm_count(void);
/* Limit of every bounded device wait (mbarrier waits of the tcgen05 kernels),
 * in ns, for the current device; default 2 s, accepted range [1 us, 60 s].
 * Synchronises the device.  Tests shorten it to make a wait expire on purpose. */
int c3b_set_wait_limit_ns(uint64_t ns);

/* Stem convolution that allocates nothing: the same computation as
 * C3B_K_STEM_IM2COL followed by C3B_K_GEMM_TC (out = act(patches(x) * w^T + bias),
 * x NCHW f32, w [Cout, kpad] bf16, bias f32 [Cout], out [N*Ho*Wo, Cout] bf16),
 * but the bf16 patch matrix lives in a fixed 16 MiB device array inside this
 * library instead of caller-allocated memory.  No counterpart in the reference:
 * it exists for callers that cannot call cudaMalloc (they run inside a memory
 * budget owned by someone else, or on a hot path where allocation would
 * synchronise the device).  Limit: N*Ho*Wo*kpad*2 <= 16 MiB, otherwise
 * C3B_E_INVALID with a message.  The first call on each device looks up the
 * array's device address (cudaGetSymbolAddress), so make that first call
 * before any stream capture; the cached address is per device and safe to
 * fill from several host threads, but it does not survive cudaDeviceReset.
 * Every argument is validated before any work is queued, so a rejected call
 * launches nothing.  All calls share the one array: calls that overlap on the
 * GPU (different streams, or different host threads) race. */
int c3b_stem_conv_noalloc(const c3b_tensor* x, const c3b_tensor* w, const c3b_tensor* bias,
                          const c3b_tensor* out, const c3b_stem_params* p, int act, void* stream);

/* ------------------------------------------------------------------ plans
 * Native replacement for PlannedGraphExecutor.run_planned
 * (c35/executor.py:723-903).  Arena = plan.pool_stats.peak_reserved_bytes
 * (executor.py:757-765); resident model tensors are uploaded once
 * (executor.py:805-839); pinned staging is allocated once per input/output slot
 * instead of once per copy (executor.py:489-505). */
typedef struct c3b_plan c3b_plan;

int c3b_plan_create(c3b_plan** out, uint64_t arena_bytes, int n_streams, int n_events);
int c3b_plan_destroy(c3b_plan* plan);
void* c3b_plan_arena(c3b_plan* plan);
/* Synchronous upload of a resident tensor (weights) into the arena; waits
 * first for every pass already launched on the plan. */
int c3b_plan_upload(c3b_plan* plan, uint64_t arena_offset, const void* host, uint64_t bytes);
/* Synchronous read of arena bytes back to host memory. */
int c3b_plan_download(c3b_plan* plan, uint64_t arena_offset, void* host, uint64_t bytes);
/* Pinned host staging for graph inputs / outputs (slots are plan-owned). */
int c3b_plan_add_input_slot(c3b_plan* plan, uint64_t bytes);
int c3b_plan_add_output_slot(c3b_plan* plan, uint64_t bytes);
void* c3b_plan_slot_ptr(c3b_plan* plan, int is_output, int slot);
/* Timeline actions, appended in order. */
int c3b_plan_add_h2d(c3b_plan* plan, int stream, int slot, uint64_t slot_offset,
                     uint64_t arena_offset, uint64_t bytes);
int c3b_plan_add_d2h(c3b_plan* plan, int stream, int slot, uint64_t slot_offset,
                     uint64_t arena_offset, uint64_t bytes);
int c3b_plan_add_record(c3b_plan* plan, int stream, int event);
int c3b_plan_add_wait(c3b_plan* plan, int stream, int event);
int c3b_plan_add_kernel(c3b_plan* plan, int stream, int kernel_id, const c3b_tensor* in, int n_in,
                        const c3b_tensor* out, int n_out, const void* params, size_t params_len);
/* Freeze the timeline; use_graph != 0 captures it as one CUDA graph. */
int c3b_plan_finalize(c3b_plan* plan, int use_graph);
/* Enqueue one pass (graph launch or action replay) on the plan's origin
 * stream; c3b_plan_sync waits for it with a deadline (cudaStreamQuery polling). */
int c3b_plan_launch(c3b_plan* plan);
int c3b_plan_sync(c3b_plan* plan, double timeout_s);
int c3b_plan_run(c3b_plan* plan);
/* Replay the timeline eagerly with CUDA events around every kernel action;
 * ms[i] receives the i-th kernel action's device time.  n = capacity. */
int c3b_plan_run_timed(c3b_plan* plan, float* ms, int n);
/* Run n_steps passes back to back with the host copies overlapped: the
 * inputs of pass k+1 are copied (on a separate copy stream, into a device
 * staging buffer) while pass k computes, and each pass's outputs leave through
 * a staging buffer of their own.  in_host[k * n_in + i] is pass k's source for
 * input slot i, out_host[k * n_out + j] its destination for output slot j
 * (pinned memory for full overlap; the plan's own slots qualify).  Each pass
 * runs the plan's timeline with its h2d / d2h actions reading and writing the
 * staging buffers.  *ms (optional) = device time from the first copy to the
 * last read-back.  No reference counterpart: the reference's run_planned
 * executes one pass at a time (streaming extension of the plan executor). */
int c3b_plan_stream(c3b_plan* plan, int n_steps, const void* const* in_host, void* const* out_host, float* ms);
int c3b_plan_kernel_count(c3b_plan* plan);
void* c3b_plan_origin_stream(c3b_plan* plan);

#ifdef __cplusplus
}
#endif

#endif /* C3B200_H */

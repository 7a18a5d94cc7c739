// C-ABI: kernel dispatch, name resolution, and the native plan executor.
//
// c3b_launch            replaces kernel(inputs, outputs, params, tuning)
//                       (c32/kernel_registry.py:6-16; called from
//                       c35/executor.py:576-581).
// c3b_kernel_id         replaces lookup(name) and its alias rules
//                       (c32/kernel_registry.py:42-67), fail-closed.
// c3b_plan_*            replace the timeline interpreter of
//                       PlannedGraphExecutor.run_planned (c35/executor.py:723-903):
//                       one arena per plan, H2D/KERNEL/EVENT/D2H actions on real
//                       CUDA streams and events, pinned staging allocated once,
//                       optional capture of the whole pass as one CUDA graph.
#include <chrono>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"

namespace c3b {

__device__ int g_status = 0;
__device__ unsigned long long g_wait_limit_ns = 2000000000ull;

static thread_local std::string t_error;

void set_error(const std::string& msg) { t_error = msg; }
int fail(int code, const std::string& msg) {
  t_error = msg;
  return code;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cached[dev] = v;
  }
  return cached[dev];
}

struct NameEntry {
  const char* name;
  int id;
};

// Every kernel name the reference registry defines (c32/kernel_registry.py:200-759)
// plus the names of the fused B200 kernels the backend's lowering emits.
static const NameEntry kNames[] = {
    {"add", C3B_K_EW}, {"add_f32", C3B_K_EW}, {"mul", C3B_K_EW}, {"mul_f32", C3B_K_EW},
    {"div", C3B_K_EW}, {"div_f32", C3B_K_EW}, {"sub", C3B_K_EW}, {"sub_f32", C3B_K_EW},
    {"relu_f32", C3B_K_EW}, {"erf_f32", C3B_K_EW}, {"exp", C3B_K_EW}, {"exp_f32", C3B_K_EW},
    {"sqrt", C3B_K_EW}, {"sqrt_f32", C3B_K_EW}, {"reciprocal", C3B_K_EW}, {"reciprocal_f32", C3B_K_EW},
    {"add_bias_f32", C3B_K_EW}, {"batchnorm_f32", C3B_K_EW}, {"fused_ew_f32", C3B_K_EW},
    {"fused_residual_relu_f32", C3B_K_EW},
    {"reduce_max", C3B_K_REDUCE}, {"reduce_max_f32", C3B_K_REDUCE}, {"reduce_sum", C3B_K_REDUCE},
    {"reduce_sum_f32", C3B_K_REDUCE}, {"reduce_mean", C3B_K_REDUCE}, {"reduce_mean_f32", C3B_K_REDUCE},
    {"matmul_f32", C3B_K_GEMM}, {"fused_matmul_bias_f32", C3B_K_GEMM}, {"fused_gemm_epilogue_f32", C3B_K_GEMM},
    {"conv_reshape_f32", C3B_K_COPY}, {"reshape", C3B_K_COPY}, {"transpose", C3B_K_COPY},
    {"flatten", C3B_K_COPY}, {"split", C3B_K_COPY}, {"fused_transpose_reshape_f32", C3B_K_COPY},
    {"im2col_f32", C3B_K_IM2COL}, {"winograd_forward_f32", C3B_K_CONV},
    {"fused_layer_norm_f32", C3B_K_LAYERNORM}, {"fused_residual_norm_f32", C3B_K_LAYERNORM},
    {"fused_softmax_f32", C3B_K_SOFTMAX}, {"fused_attention_scores_f32", C3B_K_ATTN_SCORES},
    {"gather", C3B_K_GATHER}, {"constant", 0},
    // backend kernels
    {"conv2d_bias_act_f32", C3B_K_CONV}, {"conv2d_bias_act_bf16", C3B_K_CONV_TC},
    {"gemm_bias_act_bf16", C3B_K_GEMM_TC}, {"flash_attention_f32", C3B_K_FLASH_ATTN},
    {"flash_attention_bf16", C3B_K_FLASH_ATTN}, {"embed_positions", C3B_K_EMBED},
    {"stem_im2col_bf16", C3B_K_STEM_IM2COL}, {"global_avgpool_nhwc", C3B_K_GAP_NHWC},
    {"stem_conv_bias_act_bf16", C3B_K_STEM_CONV},
    {"layout_copy", C3B_K_COPY},
    // fp8 precision path (names the reference's policy emits but cannot execute)
    {"quantize_e4m3_rows", C3B_K_QUANT_E4M3}, {"matmul_f8", C3B_K_GEMM_FP8},
    {"gemm_bias_act_f8", C3B_K_GEMM_FP8},
    // W4A16 path (the policy's fp4 for constant-weight GEMMs)
    {"quantize_fp4_groups", C3B_K_QUANT_FP4}, {"matmul_f4", C3B_K_GEMM_W4A16},
    {"gemm_bias_act_w4a16", C3B_K_GEMM_W4A16}, {"dequantize_fp4_groups", C3B_K_DEQUANT_FP4},
    // tf32 profile and the fused nodes of the backend's extra C3.3 passes
    {"gemm_bias_act_tf32", C3B_K_GEMM_TF32},
    {"b200convbiasact_f32", C3B_K_CONV}, {"b200convbiasact_bf16", C3B_K_CONV_TC},
    {"b200convbiasact_fp16", C3B_K_CONV_TC}, {"b200linearepilogue_f32", C3B_K_GEMM},
    {"b200linearepilogue_bf16", C3B_K_GEMM_TC}, {"b200linearepilogue_fp16", C3B_K_GEMM_TC},
    {"b200flashattention_f32", C3B_K_FLASH_ATTN}, {"b200flashattention_bf16", C3B_K_FLASH_ATTN},
    {"b200flashattention_fp16", C3B_K_FLASH_ATTN},
};

static int find_name(const std::string& n) {
  for (const auto& e : kNames)
    if (n == e.name) return e.id;
  return -1;
}

static int resolve_name(const char* cname) {
  if (!cname) return -1;
  std::string n(cname);
  int id = find_name(n);
  if (id >= 0) return id;
  if ((id = find_name(n + "_f32")) >= 0) return id;
  auto ends = [&](const std::string& suf) { return n.size() >= suf.size() && n.compare(n.size() - suf.size(), suf.size(), suf) == 0; };
  if (ends("_f32")) {
    if ((id = find_name(n.substr(0, n.size() - 4))) >= 0) return id;
  }
  if (ends("_fp32")) {
    std::string bare = n.substr(0, n.size() - 5);
    if ((id = find_name(bare + "_f32")) >= 0) return id;
    if ((id = find_name(bare)) >= 0) return id;
  }
  return -1;
}

template <typename P>
static int get_params(const void* params, size_t len, P& out) {
  if (!params || len != sizeof(P))
    return fail(C3B_E_INVALID, "parameter block size " + std::to_string(len) + " != expected " +
                                   std::to_string(sizeof(P)));
  memcpy(&out, params, sizeof(P));
  return C3B_OK;
}

static int check_tensors(const c3b_tensor* t, int n) {
  for (int i = 0; i < n; ++i) {
    if (t[i].ndim < 0 || t[i].ndim > C3B_MAX_RANK) return fail(C3B_E_INVALID, "tensor rank out of range");
    if (dtype_size(t[i].dtype) == 0) return fail(C3B_E_INVALID, "unknown dtype");
    for (int d = 0; d < t[i].ndim; ++d)
      if (t[i].shape[d] < 0) return fail(C3B_E_INVALID, "negative extent");
    if (!t[i].ptr && numel(t[i]) > 0) return fail(C3B_E_INVALID, "null data pointer");
  }
  return C3B_OK;
}

int dispatch(int kid, const c3b_tensor* in, int n_in, const c3b_tensor* out, int n_out, const void* params,
             size_t len, cudaStream_t s) {
  int rc;
  if ((rc = check_tensors(in, n_in))) return rc;
  if ((rc = check_tensors(out, n_out))) return rc;
  switch (kid) {
    case 0:
      return C3B_OK;
    case C3B_K_EW: {
      c3b_ew_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_out == 1, "ew: one output");
      return launch_ew(in, n_in, out[0], p, s);
    }
    case C3B_K_COPY: {
      c3b_copy_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_in == 1 && n_out == 1, "copy: one input, one output");
      return launch_copy(in[0], out[0], p, s);
    }
    case C3B_K_IM2COL: {
      c3b_conv_geom p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_in == 1 && n_out == 1, "im2col: one input, one output");
      return launch_im2col(in[0], out[0], p, s);
    }
    case C3B_K_REDUCE: {
      c3b_reduce_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_in == 1 && n_out == 1, "reduce: one input, one output");
      return launch_reduce(in[0], out[0], p, s);
    }
    case C3B_K_GEMM: {
      c3b_gemm_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_out == 1, "gemm: one output");
      return launch_gemm_simt(in, n_in, out[0], p, s);
    }
    case C3B_K_LAYERNORM: {
      c3b_layernorm_params p;
      if ((rc = get_params(params, len, p))) return rc;
      return launch_layernorm(in, n_in, out, n_out, p, s);
    }
    case C3B_K_SOFTMAX: {
      c3b_softmax_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_in == 1 && n_out == 1, "softmax: one input, one output");
      return launch_softmax(in[0], out[0], p, s);
    }
    case C3B_K_ATTN_SCORES: {
      c3b_attn_scores_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_in == 4 && n_out == 1, "attention scores: q, kT, divisor, mask -> scores");
      return launch_attn_scores(in, out[0], p, s);
    }
    case C3B_K_GATHER: {
      c3b_gather_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_in == 2 && n_out == 1, "gather: data, indices -> out");
      return launch_gather(in[0], in[1], out[0], p, s);
    }
    case C3B_K_CONV: {
      c3b_conv_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_out == 1, "conv: one output");
      return launch_conv_simt(in, n_in, out[0], p, s);
    }
    case C3B_K_GEMM_TC: {
      c3b_gemm_tc_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_out == 1, "tc gemm: one output");
      return launch_gemm_tc(in, n_in, out[0], p, s);
    }
    case C3B_K_CONV_TC: {
      c3b_conv_tc_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_out == (p.has_shortcut ? 2 : 1), "tc conv: one output, two with the fused shortcut");
      return launch_conv_tc(in, n_in, out, p, s);
    }
    case C3B_K_FLASH_ATTN: {
      c3b_flash_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_in == 1 && n_out == 1, "flash attention: qkv -> out");
      return launch_flash_attn(in[0], out[0], p, s);
    }
    case C3B_K_EMBED: {
      c3b_embed_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_in == 3 && n_out == 1, "embed: ids, tok, pos -> out");
      return launch_embed(in, out[0], p, s);
    }
    case C3B_K_STEM_IM2COL: {
      c3b_stem_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_in == 1 && n_out == 1, "stem im2col: one input, one output");
      return launch_stem_im2col(in[0], out[0], p, s);
    }
    case C3B_K_STEM_CONV: {
      c3b_stem_conv_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_out == 1, "stem conv: one output");
      return launch_stem_conv(in, n_in, out[0], p, s);
    }
    case C3B_K_QUANT_E4M3: {
      c3b_quant_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_in == 1 && n_out == 2, "quantize e4m3: x -> q, scale");
      return launch_quant_e4m3(in[0], out[0], out[1], p, s);
    }
    case C3B_K_GEMM_FP8: {
      c3b_gemm_tc_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_out == 1, "fp8 gemm: one output");
      return launch_gemm_fp8(in, n_in, out[0], p, s);
    }
    case C3B_K_QUANT_FP4: {
      c3b_quant_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_in == 1 && n_out == 2, "quantize fp4: w -> q, scale");
      return launch_quant_fp4(in[0], out[0], out[1], p, s);
    }
    case C3B_K_DEQUANT_FP4: {
      c3b_quant_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_in == 2 && n_out == 1, "dequantize fp4: q, scale -> w");
      return launch_dequant_fp4(in[0], in[1], out[0], p, s);
    }
    case C3B_K_GEMM_W4A16: {
      c3b_gemm_tc_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_out == 1, "w4a16 gemm: one output");
      return launch_gemm_w4a16(in, n_in, out[0], p, s);
    }
    case C3B_K_GEMM_TF32: {
      c3b_gemm_tc_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_out == 1, "tf32 gemm: one output");
      return launch_gemm_tf32(in, n_in, out[0], p, s);
    }
    case C3B_K_WAIT_PROBE: {
      c3b_wait_probe_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_in == 0 && n_out == 0, "wait probe: no tensors");
      return launch_wait_probe(p, s);
    }
    case C3B_K_GAP_NHWC: {
      c3b_gap_params p;
      if ((rc = get_params(params, len, p))) return rc;
      C3B_REQUIRE(n_in >= 1 && n_in <= 3 && n_out == 1, "gap: x [, w [, b]] in, one output");
      return launch_gap_nhwc(in, n_in, out[0], p, s);
    }
  }
  return fail(C3B_E_UNKNOWN, "unknown kernel id " + std::to_string(kid));
}

}  // namespace c3b

using namespace c3b;

// ======================================================================= plans

namespace {

enum ActKind { A_KERNEL = 0, A_H2D, A_D2H, A_RECORD, A_WAIT };

struct Action {
  int kind = 0;
  int stream = 0;
  int event = 0;
  int kernel = 0;
  std::vector<c3b_tensor> in, out;
  std::vector<uint8_t> params;
  int slot = 0;
  uint64_t slot_off = 0, arena_off = 0, bytes = 0;
};

}  // namespace

struct c3b_plan {
  int device = 0;
  uint8_t* arena = nullptr;
  uint64_t arena_bytes = 0;
  std::vector<cudaStream_t> streams;
  std::vector<cudaEvent_t> events;
  std::vector<cudaEvent_t> joins;
  cudaEvent_t fork = nullptr;
  cudaStream_t origin = nullptr;
  std::vector<void*> in_slots, out_slots;
  std::vector<uint64_t> in_bytes, out_bytes;
  std::vector<Action> actions;
  bool finalized = false;
  bool use_graph = false;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int n_kernels = 0;
  // streaming (c3b_plan_stream): device staging copies of the slots, one
  // graph of the device pass per staging parity, a copy stream and its events
  uint64_t in_total = 0, out_total = 0;
  std::vector<uint64_t> in_base, out_base;
  uint8_t* stg_in[2] = {nullptr, nullptr};
  uint8_t* stg_out[2] = {nullptr, nullptr};
  cudaGraphExec_t sexec[2] = {nullptr, nullptr};
  cudaStream_t cstream = nullptr;
  cudaEvent_t in_ready[2] = {nullptr, nullptr}, pass_done[2] = {nullptr, nullptr}, out_read[2] = {nullptr, nullptr};
  cudaEvent_t t_begin = nullptr, t_end = nullptr, c_end = nullptr;
};

// Device staging for one streamed pass: slot copies read and write device
// buffers (parity `par`) instead of the pinned host slots.
struct Staging {
  const c3b_plan* p;
  int par;
};

static int plan_enqueue(c3b_plan* p, std::vector<cudaEvent_t>* timers, const Staging* stg = nullptr) {
  C3B_CHECK_CUDA(cudaEventRecord(p->fork, p->origin));
  for (auto s : p->streams) C3B_CHECK_CUDA(cudaStreamWaitEvent(s, p->fork, 0));
  int k = 0;
  for (const Action& a : p->actions) {
    cudaStream_t s = p->streams[a.stream];
    switch (a.kind) {
      case A_KERNEL: {
        if (timers) C3B_CHECK_CUDA(cudaEventRecord((*timers)[2 * k], s));
        int rc = dispatch(a.kernel, a.in.data(), (int)a.in.size(), a.out.data(), (int)a.out.size(),
                          a.params.data(), a.params.size(), s);
        if (rc) return rc;
        if (timers) C3B_CHECK_CUDA(cudaEventRecord((*timers)[2 * k + 1], s));
        ++k;
        break;
      }
      case A_H2D:
        if (stg)
          C3B_CHECK_CUDA(cudaMemcpyAsync(p->arena + a.arena_off, p->stg_in[stg->par] + p->in_base[a.slot] + a.slot_off,
                                         a.bytes, cudaMemcpyDeviceToDevice, s));
        else
          C3B_CHECK_CUDA(cudaMemcpyAsync(p->arena + a.arena_off, (uint8_t*)p->in_slots[a.slot] + a.slot_off, a.bytes,
                                         cudaMemcpyHostToDevice, s));
        break;
      case A_D2H:
        if (stg)
          C3B_CHECK_CUDA(cudaMemcpyAsync(p->stg_out[stg->par] + p->out_base[a.slot] + a.slot_off, p->arena + a.arena_off,
                                         a.bytes, cudaMemcpyDeviceToDevice, s));
        else
          C3B_CHECK_CUDA(cudaMemcpyAsync((uint8_t*)p->out_slots[a.slot] + a.slot_off, p->arena + a.arena_off, a.bytes,
                                         cudaMemcpyDeviceToHost, s));
        break;
      case A_RECORD:
        C3B_CHECK_CUDA(cudaEventRecord(p->events[a.event], s));
        break;
      case A_WAIT:
        C3B_CHECK_CUDA(cudaStreamWaitEvent(s, p->events[a.event], 0));
        break;
    }
  }
  for (size_t i = 0; i < p->streams.size(); ++i) {
    C3B_CHECK_CUDA(cudaEventRecord(p->joins[i], p->streams[i]));
    C3B_CHECK_CUDA(cudaStreamWaitEvent(p->origin, p->joins[i], 0));
  }
  return C3B_OK;
}

// [off, off + bytes) inside [0, cap), written so that huge offsets cannot wrap.
static inline bool in_range(uint64_t off, uint64_t bytes, uint64_t cap) {
  return bytes <= cap && off <= cap - bytes;
}

extern "C" {

int c3b_version(void) { return 1; }

const char* c3b_last_error(void) { return t_error.c_str(); }

int c3b_kernel_id(const char* name) {
  int id = resolve_name(name);
  if (id < 0)
    return fail(C3B_E_UNKNOWN, std::string("Unknown kernel: '") + (name ? name : "(null)") + "'");
  return id;
}

int c3b_launch(int kernel_id, const c3b_tensor* in, int n_in, const c3b_tensor* out, int n_out, const void* params,
               size_t params_len, void* stream) {
  if (n_in < 0 || n_out < 0 || (n_in && !in) || (n_out && !out)) return fail(C3B_E_INVALID, "bad tensor lists");
  return dispatch(kernel_id, in, n_in, out, n_out, params, params_len, (cudaStream_t)stream);
}

int c3b_device_status(int* status) {
  C3B_CHECK_CUDA(cudaDeviceSynchronize());
  int v = 0, zero = 0;
  C3B_CHECK_CUDA(cudaMemcpyFromSymbol(&v, g_status, sizeof(int)));
  C3B_CHECK_CUDA(cudaMemcpyToSymbol(g_status, &zero, sizeof(int)));
  if (status) *status = v;
  return C3B_OK;
}

int c3b_sm_count(void) { return sm_count(); }

int c3b_set_wait_limit_ns(uint64_t ns) {
  if (ns < 1000ull || ns > 60000000000ull) return fail(C3B_E_INVALID, "wait limit must be within [1 us, 60 s]");
  unsigned long long v = ns;
  C3B_CHECK_CUDA(cudaDeviceSynchronize());
  C3B_CHECK_CUDA(cudaMemcpyToSymbol(g_wait_limit_ns, &v, sizeof(v)));
  return C3B_OK;
}

int c3b_plan_create(c3b_plan** out, uint64_t arena_bytes, int n_streams, int n_events) {
  if (!out || n_streams < 1 || n_streams > 64 || n_events < 0) return fail(C3B_E_INVALID, "plan_create: arguments");
  c3b_plan* p = new c3b_plan();
  cudaGetDevice(&p->device);
  p->arena_bytes = arena_bytes ? arena_bytes : 256;
  cudaError_t e = cudaMalloc(&p->arena, p->arena_bytes);
  if (e != cudaSuccess) {
    delete p;
    return fail(C3B_E_CUDA, std::string("arena cudaMalloc: ") + cudaGetErrorString(e));
  }
  auto bad = [&](cudaError_t err) {
    c3b_plan_destroy(p);
    return fail(C3B_E_CUDA, std::string("plan_create: ") + cudaGetErrorString(err));
  };
  for (int i = 0; i < n_streams; ++i) {
    cudaStream_t s;
    if ((e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking)) != cudaSuccess) return bad(e);
    p->streams.push_back(s);
    cudaEvent_t j;
    if ((e = cudaEventCreateWithFlags(&j, cudaEventDisableTiming)) != cudaSuccess) return bad(e);
    p->joins.push_back(j);
  }
  for (int i = 0; i < n_events; ++i) {
    cudaEvent_t ev;
    if ((e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming)) != cudaSuccess) return bad(e);
    p->events.push_back(ev);
  }
  if ((e = cudaEventCreateWithFlags(&p->fork, cudaEventDisableTiming)) != cudaSuccess) return bad(e);
  if ((e = cudaStreamCreateWithFlags(&p->origin, cudaStreamNonBlocking)) != cudaSuccess) return bad(e);
  *out = p;
  return C3B_OK;
}

int c3b_plan_destroy(c3b_plan* p) {
  if (!p) return C3B_OK;
  if (p->origin) cudaStreamSynchronize(p->origin);
  if (p->exec) cudaGraphExecDestroy(p->exec);
  if (p->cstream) cudaStreamSynchronize(p->cstream);
  for (int i = 0; i < 2; ++i) {
    if (p->sexec[i]) cudaGraphExecDestroy(p->sexec[i]);
    if (p->stg_in[i]) cudaFree(p->stg_in[i]);
    if (p->stg_out[i]) cudaFree(p->stg_out[i]);
    for (cudaEvent_t e : {p->in_ready[i], p->pass_done[i], p->out_read[i]})
      if (e) cudaEventDestroy(e);
  }
  for (cudaEvent_t e : {p->t_begin, p->t_end, p->c_end})
    if (e) cudaEventDestroy(e);
  if (p->cstream) cudaStreamDestroy(p->cstream);
  if (p->graph) cudaGraphDestroy(p->graph);
  for (auto s : p->streams) cudaStreamDestroy(s);
  for (auto e : p->events) cudaEventDestroy(e);
  for (auto e : p->joins) cudaEventDestroy(e);
  if (p->fork) cudaEventDestroy(p->fork);
  if (p->origin) cudaStreamDestroy(p->origin);
  for (auto h : p->in_slots) cudaFreeHost(h);
  for (auto h : p->out_slots) cudaFreeHost(h);
  if (p->arena) cudaFree(p->arena);
  delete p;
  return C3B_OK;
}

void* c3b_plan_arena(c3b_plan* p) { return p ? p->arena : nullptr; }

void* c3b_plan_origin_stream(c3b_plan* p) { return p ? (void*)p->origin : nullptr; }

int c3b_plan_upload(c3b_plan* p, uint64_t off, const void* host, uint64_t bytes) {
  if (!p || !host) return fail(C3B_E_INVALID, "plan_upload: arguments");
  if (!in_range(off, bytes, p->arena_bytes)) return fail(C3B_E_INVALID, "plan_upload: range exceeds the arena");
  // ordered after every pass already launched on this plan (they read the arena)
  C3B_CHECK_CUDA(cudaStreamSynchronize(p->origin));
  C3B_CHECK_CUDA(cudaMemcpy(p->arena + off, host, bytes, cudaMemcpyHostToDevice));
  return C3B_OK;
}

int c3b_plan_download(c3b_plan* p, uint64_t off, void* host, uint64_t bytes) {
  if (!p || !host) return fail(C3B_E_INVALID, "plan_download: arguments");
  if (!in_range(off, bytes, p->arena_bytes)) return fail(C3B_E_INVALID, "plan_download: range exceeds the arena");
  C3B_CHECK_CUDA(cudaStreamSynchronize(p->origin));
  C3B_CHECK_CUDA(cudaMemcpy(host, p->arena + off, bytes, cudaMemcpyDeviceToHost));
  return C3B_OK;
}

static int add_slot(std::vector<void*>& v, std::vector<uint64_t>& b, uint64_t bytes) {
  void* h = nullptr;
  C3B_CHECK_CUDA(cudaMallocHost(&h, bytes ? bytes : 16));
  memset(h, 0, bytes ? bytes : 16);
  v.push_back(h);
  b.push_back(bytes);
  return (int)v.size() - 1;
}

int c3b_plan_add_input_slot(c3b_plan* p, uint64_t bytes) {
  if (!p || p->finalized) return fail(C3B_E_INVALID, "plan_add_input_slot: plan finalized");
  return add_slot(p->in_slots, p->in_bytes, bytes);
}

int c3b_plan_add_output_slot(c3b_plan* p, uint64_t bytes) {
  if (!p || p->finalized) return fail(C3B_E_INVALID, "plan_add_output_slot: plan finalized");
  return add_slot(p->out_slots, p->out_bytes, bytes);
}

void* c3b_plan_slot_ptr(c3b_plan* p, int is_output, int slot) {
  if (!p) return nullptr;
  auto& v = is_output ? p->out_slots : p->in_slots;
  if (slot < 0 || slot >= (int)v.size()) return nullptr;
  return v[slot];
}

static int check_stream(c3b_plan* p, int stream) {
  if (!p || p->finalized) return fail(C3B_E_INVALID, "plan is null or finalized");
  if (stream < 0 || stream >= (int)p->streams.size()) return fail(C3B_E_INVALID, "stream id out of range");
  return C3B_OK;
}

int c3b_plan_add_h2d(c3b_plan* p, int stream, int slot, uint64_t slot_off, uint64_t arena_off, uint64_t bytes) {
  int rc = check_stream(p, stream);
  if (rc) return rc;
  if (slot < 0 || slot >= (int)p->in_slots.size() || !in_range(slot_off, bytes, p->in_bytes[slot]))
    return fail(C3B_E_INVALID, "h2d: slot range");
  if (!in_range(arena_off, bytes, p->arena_bytes)) return fail(C3B_E_INVALID, "h2d: arena range");
  Action a;
  a.kind = A_H2D; a.stream = stream; a.slot = slot; a.slot_off = slot_off; a.arena_off = arena_off; a.bytes = bytes;
  p->actions.push_back(std::move(a));
  return C3B_OK;
}

int c3b_plan_add_d2h(c3b_plan* p, int stream, int slot, uint64_t slot_off, uint64_t arena_off, uint64_t bytes) {
  int rc = check_stream(p, stream);
  if (rc) return rc;
  if (slot < 0 || slot >= (int)p->out_slots.size() || !in_range(slot_off, bytes, p->out_bytes[slot]))
    return fail(C3B_E_INVALID, "d2h: slot range");
  if (!in_range(arena_off, bytes, p->arena_bytes)) return fail(C3B_E_INVALID, "d2h: arena range");
  Action a;
  a.kind = A_D2H; a.stream = stream; a.slot = slot; a.slot_off = slot_off; a.arena_off = arena_off; a.bytes = bytes;
  p->actions.push_back(std::move(a));
  return C3B_OK;
}

static int add_event_action(c3b_plan* p, int kind, int stream, int event) {
  int rc = check_stream(p, stream);
  if (rc) return rc;
  if (event < 0 || event >= (int)p->events.size()) return fail(C3B_E_INVALID, "event id out of range");
  Action a;
  a.kind = kind; a.stream = stream; a.event = event;
  p->actions.push_back(std::move(a));
  return C3B_OK;
}

int c3b_plan_add_record(c3b_plan* p, int stream, int event) { return add_event_action(p, A_RECORD, stream, event); }
int c3b_plan_add_wait(c3b_plan* p, int stream, int event) { return add_event_action(p, A_WAIT, stream, event); }

int c3b_plan_add_kernel(c3b_plan* p, int stream, int kernel_id, const c3b_tensor* in, int n_in, const c3b_tensor* out,
                        int n_out, const void* params, size_t params_len) {
  int rc = check_stream(p, stream);
  if (rc) return rc;
  Action a;
  a.kind = A_KERNEL; a.stream = stream; a.kernel = kernel_id;
  auto resolve = [&](const c3b_tensor* t, int n, std::vector<c3b_tensor>& dst) -> int {
    for (int i = 0; i < n; ++i) {
      c3b_tensor x = t[i];
      if (x.flags & C3B_TENSOR_ARENA) {
        uint64_t off = (uint64_t)(uintptr_t)x.ptr;
        uint64_t bytes = (uint64_t)numel(x) * dtype_size(x.dtype);
        if (!in_range(off, bytes, p->arena_bytes)) return fail(C3B_E_INVALID, "kernel tensor exceeds the arena");
        x.ptr = p->arena + off;
        x.flags &= ~C3B_TENSOR_ARENA;
      }
      dst.push_back(x);
    }
    return C3B_OK;
  };
  if ((rc = resolve(in, n_in, a.in))) return rc;
  if ((rc = resolve(out, n_out, a.out))) return rc;
  if (params_len) a.params.assign((const uint8_t*)params, (const uint8_t*)params + params_len);
  p->actions.push_back(std::move(a));
  p->n_kernels++;
  return C3B_OK;
}

int c3b_plan_kernel_count(c3b_plan* p) { return p ? p->n_kernels : 0; }

int c3b_plan_finalize(c3b_plan* p, int use_graph) {
  if (!p || p->finalized) return fail(C3B_E_INVALID, "plan_finalize: plan is null or finalized");
  p->finalized = true;
  // One eager pass validates every action and sets per-kernel attributes
  // outside of stream capture.
  int rc = plan_enqueue(p, nullptr);
  if (rc) return rc;
  C3B_CHECK_CUDA(cudaStreamSynchronize(p->origin));
  C3B_CHECK_CUDA(cudaGetLastError());
  if (use_graph) {
    C3B_CHECK_CUDA(cudaStreamBeginCapture(p->origin, cudaStreamCaptureModeThreadLocal));
    rc = plan_enqueue(p, nullptr);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(p->origin, &g);
    if (rc) {
      if (g) cudaGraphDestroy(g);
      return rc;
    }
    if (e != cudaSuccess) return fail(C3B_E_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
    p->graph = g;
    C3B_CHECK_CUDA(cudaGraphInstantiate(&p->exec, g, 0));
    p->use_graph = true;
  }
  return C3B_OK;
}

int c3b_plan_launch(c3b_plan* p) {
  if (!p || !p->finalized) return fail(C3B_E_INVALID, "plan_launch: plan not finalized");
  if (p->use_graph) {
    C3B_CHECK_CUDA(cudaGraphLaunch(p->exec, p->origin));
    return C3B_OK;
  }
  return plan_enqueue(p, nullptr);
}

int c3b_plan_sync(c3b_plan* p, double timeout_s) {
  if (!p) return fail(C3B_E_INVALID, "plan_sync: null plan");
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t e = cudaStreamQuery(p->origin);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) return fail(C3B_E_CUDA, std::string("plan_sync: ") + cudaGetErrorString(e));
    double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (timeout_s > 0 && dt > timeout_s) return fail(C3B_E_CUDA, "plan_sync: deadline exceeded");
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  int v = 0;
  C3B_CHECK_CUDA(cudaMemcpyFromSymbol(&v, g_status, sizeof(int)));
  if (v) {
    int zero = 0;
    cudaMemcpyToSymbol(g_status, &zero, sizeof(int));
    return fail(C3B_E_DEVICE, "a kernel reported device status " + std::to_string(v));
  }
  return C3B_OK;
}

int c3b_plan_run(c3b_plan* p) {
  int rc = c3b_plan_launch(p);
  if (rc) return rc;
  return c3b_plan_sync(p, 600.0);
}

// Lazily set up the streaming state: staging buffers, the two device-pass
// graphs (captured like c3b_plan_finalize's), the copy stream and events.
static int stream_setup(c3b_plan* p) {
  if (p->sexec[0]) return C3B_OK;
  p->in_base.clear();
  p->out_base.clear();
  p->in_total = p->out_total = 0;
  for (uint64_t b : p->in_bytes) { p->in_base.push_back(p->in_total); p->in_total += (b + 255) & ~255ull; }
  for (uint64_t b : p->out_bytes) { p->out_base.push_back(p->out_total); p->out_total += (b + 255) & ~255ull; }
  for (int i = 0; i < 2; ++i) {
    C3B_CHECK_CUDA(cudaMalloc(&p->stg_in[i], p->in_total ? p->in_total : 256));
    C3B_CHECK_CUDA(cudaMalloc(&p->stg_out[i], p->out_total ? p->out_total : 256));
    C3B_CHECK_CUDA(cudaEventCreateWithFlags(&p->in_ready[i], cudaEventDisableTiming));
    C3B_CHECK_CUDA(cudaEventCreateWithFlags(&p->pass_done[i], cudaEventDisableTiming));
    C3B_CHECK_CUDA(cudaEventCreateWithFlags(&p->out_read[i], cudaEventDisableTiming));
  }
  C3B_CHECK_CUDA(cudaEventCreate(&p->t_begin));
  C3B_CHECK_CUDA(cudaEventCreate(&p->t_end));
  C3B_CHECK_CUDA(cudaEventCreateWithFlags(&p->c_end, cudaEventDisableTiming));
  C3B_CHECK_CUDA(cudaStreamCreateWithFlags(&p->cstream, cudaStreamNonBlocking));
  for (int par = 0; par < 2; ++par) {
    Staging st{p, par};
    C3B_CHECK_CUDA(cudaStreamBeginCapture(p->origin, cudaStreamCaptureModeThreadLocal));
    int rc = plan_enqueue(p, nullptr, &st);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(p->origin, &g);
    if (rc) {
      if (g) cudaGraphDestroy(g);
      return rc;
    }
    if (e != cudaSuccess) return fail(C3B_E_CUDA, std::string("stream capture: ") + cudaGetErrorString(e));
    e = cudaGraphInstantiate(&p->sexec[par], g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return fail(C3B_E_CUDA, std::string("stream instantiate: ") + cudaGetErrorString(e));
  }
  return C3B_OK;
}

int c3b_plan_stream(c3b_plan* p, int n_steps, const void* const* in_host, void* const* out_host, float* ms) {
  if (!p || !p->finalized) return fail(C3B_E_INVALID, "plan_stream: plan not finalized");
  if (n_steps < 0) return fail(C3B_E_INVALID, "plan_stream: n_steps < 0");
  const int n_in = (int)p->in_slots.size(), n_out = (int)p->out_slots.size();
  if ((n_in && !in_host) || (n_out && !out_host)) return fail(C3B_E_INVALID, "plan_stream: host pointer lists");
  for (int64_t i = 0; i < (int64_t)n_steps * n_in; ++i)
    if (!in_host[i]) return fail(C3B_E_INVALID, "plan_stream: null input pointer");
  for (int64_t i = 0; i < (int64_t)n_steps * n_out; ++i)
    if (!out_host[i]) return fail(C3B_E_INVALID, "plan_stream: null output pointer");
  int rc = stream_setup(p);
  if (rc) return rc;
  if (n_steps == 0) {
    if (ms) *ms = 0.f;
    return C3B_OK;
  }
  cudaStream_t cs = p->cstream, os = p->origin;
  auto h2d = [&](int k) -> int {
    uint8_t* dst = p->stg_in[k & 1];
    for (int i = 0; i < n_in; ++i)
      C3B_CHECK_CUDA(cudaMemcpyAsync(dst + p->in_base[i], in_host[(int64_t)k * n_in + i], p->in_bytes[i],
                                     cudaMemcpyHostToDevice, cs));
    C3B_CHECK_CUDA(cudaEventRecord(p->in_ready[k & 1], cs));
    return C3B_OK;
  };
  C3B_CHECK_CUDA(cudaEventRecord(p->t_begin, os));
  C3B_CHECK_CUDA(cudaStreamWaitEvent(cs, p->t_begin, 0));
  if ((rc = h2d(0))) return rc;
  for (int k = 0; k < n_steps; ++k) {
    const int par = k & 1;
    // device pass k: waits for its staged inputs and for the read-back of the
    // outputs staged two passes ago (same parity)
    C3B_CHECK_CUDA(cudaStreamWaitEvent(os, p->in_ready[par], 0));
    if (k >= 2) C3B_CHECK_CUDA(cudaStreamWaitEvent(os, p->out_read[par], 0));
    C3B_CHECK_CUDA(cudaGraphLaunch(p->sexec[par], os));
    C3B_CHECK_CUDA(cudaEventRecord(p->pass_done[par], os));
    // copies: next inputs (their staging buffer was consumed by pass k-1),
    // then this pass's outputs
    if (k + 1 < n_steps) {
      if (k >= 1) C3B_CHECK_CUDA(cudaStreamWaitEvent(cs, p->pass_done[par ^ 1], 0));
      if ((rc = h2d(k + 1))) return rc;
    }
    C3B_CHECK_CUDA(cudaStreamWaitEvent(cs, p->pass_done[par], 0));
    for (int i = 0; i < n_out; ++i)
      C3B_CHECK_CUDA(cudaMemcpyAsync(out_host[(int64_t)k * n_out + i], p->stg_out[par] + p->out_base[i], p->out_bytes[i],
                                     cudaMemcpyDeviceToHost, cs));
    C3B_CHECK_CUDA(cudaEventRecord(p->out_read[par], cs));
  }
  C3B_CHECK_CUDA(cudaEventRecord(p->c_end, cs));
  C3B_CHECK_CUDA(cudaStreamWaitEvent(os, p->c_end, 0));
  C3B_CHECK_CUDA(cudaEventRecord(p->t_end, os));
  rc = c3b_plan_sync(p, 600.0);
  if (rc) return rc;
  if (ms) C3B_CHECK_CUDA(cudaEventElapsedTime(ms, p->t_begin, p->t_end));
  return C3B_OK;
}

int c3b_plan_run_timed(c3b_plan* p, float* ms, int n) {
  if (!p || !p->finalized) return fail(C3B_E_INVALID, "plan_run_timed: plan not finalized");
  std::vector<cudaEvent_t> ev(2 * (size_t)p->n_kernels);
  for (auto& e : ev) C3B_CHECK_CUDA(cudaEventCreate(&e));
  int rc = plan_enqueue(p, &ev);
  if (!rc) rc = c3b_plan_sync(p, 600.0);
  if (!rc) {
    for (int k = 0; k < p->n_kernels && k < n; ++k) {
      float t = 0.f;
      if (cudaEventElapsedTime(&t, ev[2 * k], ev[2 * k + 1]) != cudaSuccess) t = -1.f;
      ms[k] = t;
    }
  }
  for (auto& e : ev) cudaEventDestroy(e);
  return rc;
}

}  // extern "C"

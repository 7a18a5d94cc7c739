// Allocation-free variant of the stem convolution.
//
// The regular stem path (C3B_K_STEM_IM2COL followed by C3B_K_GEMM_TC) needs a
// bf16 patch matrix in global memory that the caller must allocate.  Some
// callers cannot allocate device memory at the point where they run: code that
// executes inside a pre-sized memory budget (an arena owned by someone else),
// plugins called from a host runtime that forbids cudaMalloc on its hot path
// because it would synchronise the device, and embedders that only hand over
// input and output buffers.  c3b_stem_conv_noalloc serves them: the patch
// matrix lives in a fixed, file-scope device array that every GPU loading this
// library holds until the process exits.
#include <atomic>

#include "common.cuh"

namespace c3b {

// 16 MiB: the patch matrix of up to 131072 output pixels at 64 bf16 columns
// (128 CIFAR images of 32x32).
constexpr size_t kStemScratchBytes = 16u << 20;
static __device__ __align__(256) uint8_t g_stem_scratch[kStemScratchBytes];

// Device address of g_stem_scratch per device, looked up on the first call
// made with that device current.  In host code the symbol itself is only a
// stand-in and must never be handed to a kernel.  The slots are atomics, so
// two host threads making their first call on one device at the same time
// both store the same address without a data race.  The address belongs to the
// device's primary context: a process that calls cudaDeviceReset must not use
// this entry point again afterwards.
static std::atomic<void*> g_scratch_addr[64];

static int scratch_address(void** out) {
  int dev = 0;
  C3B_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(C3B_E_UNSUPPORTED, "stem_conv_noalloc: device index out of range");
  void* p = g_scratch_addr[dev].load(std::memory_order_acquire);
  if (!p) {
    C3B_CHECK_CUDA(cudaGetSymbolAddress(&p, g_stem_scratch));
    g_scratch_addr[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return C3B_OK;
}

}  // namespace c3b

using namespace c3b;

extern "C" int c3b_stem_conv_noalloc(const c3b_tensor* x, const c3b_tensor* w, const c3b_tensor* bias,
                                     const c3b_tensor* out, const c3b_stem_params* p, int act, void* stream) {
  if (!x || !w || !bias || !out || !p) return fail(C3B_E_INVALID, "stem_conv_noalloc: null argument");
  const int64_t M = (int64_t)p->n * p->ho * p->wo;
  const uint64_t need = (uint64_t)M * (uint64_t)p->kpad * 2;
  if (p->kpad <= 0 || M <= 0) return fail(C3B_E_INVALID, "stem_conv_noalloc: empty problem");
  if (need > kStemScratchBytes)
    return fail(C3B_E_INVALID, "stem_conv_noalloc: patch matrix needs " + std::to_string(need) +
                                   " bytes, the fixed scratch holds " + std::to_string(kStemScratchBytes) +
                                   " (at most " + std::to_string(kStemScratchBytes / (2 * (uint64_t)p->kpad)) +
                                   " output pixels); split the batch");
  // Every argument is checked here, before anything is queued: a rejected
  // call launches nothing and leaves the shared scratch untouched.
  if (x->dtype != C3B_F32 || numel(*x) != (int64_t)p->n * p->c * p->h * p->w)
    return fail(C3B_E_INVALID, "stem_conv_noalloc: x must be f32 [n, c, h, w]");
  if (p->kpad % 8 != 0 || p->kpad < p->g.kh * p->g.kw * p->c)
    return fail(C3B_E_INVALID, "stem_conv_noalloc: kpad must be a multiple of 8 covering c*kh*kw");
  if (w->dtype != C3B_BF16 || w->ndim != 2 || w->shape[1] != p->kpad)
    return fail(C3B_E_INVALID, "stem_conv_noalloc: w must be bf16 [Cout, kpad]");
  const int64_t cout = w->shape[0];
  if (cout <= 0 || cout % 32 != 0) return fail(C3B_E_INVALID, "stem_conv_noalloc: Cout must be a positive multiple of 32");
  if (((uintptr_t)w->ptr & 15) != 0) return fail(C3B_E_INVALID, "stem_conv_noalloc: w must be 16-byte aligned");
  if (bias->dtype != C3B_F32 || numel(*bias) != cout)
    return fail(C3B_E_INVALID, "stem_conv_noalloc: bias must be f32 [Cout]");
  if ((out->dtype != C3B_BF16 && out->dtype != C3B_F32) || numel(*out) < M * cout)
    return fail(C3B_E_INVALID, "stem_conv_noalloc: out must be bf16 or f32 with at least n*ho*wo*Cout elements");
  if (((uintptr_t)out->ptr & 15) != 0) return fail(C3B_E_INVALID, "stem_conv_noalloc: out must be 16-byte aligned");
  if (act != C3B_ACT_NONE && act != C3B_ACT_RELU && act != C3B_ACT_GELU)
    return fail(C3B_E_INVALID, "stem_conv_noalloc: unknown activation");
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  c3b_tensor cols;
  memset(&cols, 0, sizeof(cols));
  cols.ptr = scratch;
  cols.dtype = C3B_BF16;
  cols.ndim = 2;
  cols.shape[0] = M;
  cols.shape[1] = p->kpad;
  // Every element of the patch matrix (zero padding columns included) is
  // rewritten on each call, so the previous call's contents never leak in.
  rc = launch_stem_im2col(*x, cols, *p, s);
  if (rc) return rc;
  c3b_gemm_tc_params g;
  memset(&g, 0, sizeof(g));
  g.M = M;
  g.N = w->shape[0];
  g.K = p->kpad;
  g.bias_mode = C3B_BIAS_COL;
  g.act = act;
  c3b_tensor ins[3] = {cols, *w, *bias};
  return launch_gemm_tc(ins, 3, *out, g, s);
}

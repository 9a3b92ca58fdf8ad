// lb_linear_noalloc: the quantized product without a caller-supplied workspace and without allocating.
//
// Who needs it: callers that cannot allocate device memory at the point of the call.  A serving engine that
// reserved all free HBM for its KV-cache pool at start-up has nothing left for cudaMalloc; a decode loop that
// must not stall on the implicit device synchronisation of cudaMalloc/cudaFree; and host bindings (ctypes,
// cgo, JNI) that have no device allocator of their own to hand a workspace pointer over.  lb_linear needs a
// workspace only on the prefill path (M > 16), for the fp16 copy of the activations and the per-token
// factors; here that scratch is a file-scope device array, so the call allocates nothing.
//
// Limits and rules:
//   * the scratch holds LB_NOALLOC_SCRATCH_BYTES; larger prefill shapes are rejected with LB_E_WORKSPACE
//     (the decode path, M <= 16, uses no scratch and takes any shape lb_linear takes);
//   * nothing in the scratch has to start at zero: prep_x_kernel writes every byte the GEMM reads first;
//   * there is ONE scratch per device: two calls whose prefill kernels overlap in time on one device (two
//     streams, or two host threads) race on it and corrupt each other's outputs.  Calls in order on one
//     stream are safe;
//   * host code cannot use the array's name as a device address: the address is looked up with
//     cudaGetSymbolAddress on the first call in each CUDA context of a device (the primary context, a context
//     made current through the driver API, or a new primary context after cudaDeviceReset: the cache is keyed
//     by the context's unique id) and reused after that; make that first call outside any stream capture.
#include <cuda.h>
#include <mutex>

#include "../../include/apsi_lowbit.h"
#include "lb_common.cuh"
#include "lb_kernels.h"

namespace lb {

static __device__ __align__(256) unsigned char g_noalloc_scratch[LB_NOALLOC_SCRATCH_BYTES];

namespace {
struct ScratchSlot {
  unsigned long long ctx_id = 0;  // unique id of the context the address belongs to (0: none yet)
  void* ptr = nullptr;
};
ScratchSlot g_scratch[64];        // per device
std::mutex g_scratch_mu;

typedef CUresult (*PFN_ctxGetCurrent)(CUcontext*);
typedef CUresult (*PFN_ctxGetId)(CUcontext, unsigned long long*);

// Unique id of the calling thread's current context (0 when it cannot be read).
unsigned long long current_ctx_id() {
  static PFN_ctxGetCurrent get_cur = nullptr;
  static PFN_ctxGetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* a = nullptr;
    void* b = nullptr;
    cudaDriverEntryPointQueryResult q1, q2;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &a, cudaEnableDefault, &q1) == cudaSuccess &&
        q1 == cudaDriverEntryPointSuccess &&
        cudaGetDriverEntryPoint("cuCtxGetId", &b, cudaEnableDefault, &q2) == cudaSuccess &&
        q2 == cudaDriverEntryPointSuccess) {
      get_cur = reinterpret_cast<PFN_ctxGetCurrent>(a);
      get_id = reinterpret_cast<PFN_ctxGetId>(b);
    }
  });
  if (!get_cur || !get_id) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_cur(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

int scratch_for_device(int dev, void** out) {
  if (dev < 0 || dev >= 64) return fail(LB_E_DEVICE, "device %d out of range", dev);
  const unsigned long long id = current_ctx_id();
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  ScratchSlot& s = g_scratch[dev];
  if (!s.ptr || id == 0 || s.ctx_id != id) {   // unknown context id: look the address up every time
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);   // this context's copy of the array
    if (e != cudaSuccess || !p)
      return fail(LB_E_DEVICE, "lb_linear_noalloc: cudaGetSymbolAddress of the scratch failed on device %d: %s",
                  dev, cudaGetErrorString(e));
    s.ptr = p;
    s.ctx_id = id;
  }
  *out = s.ptr;
  return LB_OK;
}
}  // namespace

}  // namespace lb

extern "C" int lb_linear_noalloc(int fmt, const void* x, int64_t M, int64_t K, const void* codes, const void* scales,
                                 int64_t N, const void* bias, int accumulate, void* y, int64_t ldy, void* stream) {
  using namespace lb;
  const bool fp6 = (fmt == LB_FMT_FP6_E3M2 || fmt == LB_FMT_FP6_E2M3);
  if (fmt != LB_FMT_INT8_ROW && fmt != LB_FMT_INT4_G128 && fmt != LB_FMT_FP8_E4M3 && fmt != LB_FMT_FP8_E5M2 &&
      fmt != LB_FMT_FP4_E2M1 && !(fp6 && (M <= 16 || K % 64 == 0)))
    return fail(LB_E_UNSUPPORTED, "lb_linear_noalloc: format %d has no product kernel for M = %lld in this build", fmt,
                (long long)M);
  if (M <= 0 || N <= 0 || K <= 0) return fail(LB_E_ARG, "lb_linear_noalloc: M, N, K must be positive");
  if (M > (1LL << 31) || K > (1LL << 31)) return fail(LB_E_ARG, "lb_linear_noalloc: M and K must be below 2^31");
  if (M <= 16)   // decode path: no scratch at all
    return lb_linear_ex(fmt, x, M, K, codes, scales, N, bias, accumulate, y, ldy, nullptr, 0, 0u, stream);
  const size_t need = gemm_workspace_bytes(M, N, K);
  if (need > static_cast<size_t>(LB_NOALLOC_SCRATCH_BYTES))
    return fail(LB_E_WORKSPACE,
                "lb_linear_noalloc: M=%lld, K=%lld needs %zu bytes of scratch, above the fixed %d "
                "(use lb_linear with a workspace)", (long long)M, (long long)K, need, LB_NOALLOC_SCRATCH_BYTES);
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(LB_E_DEVICE, "lb_linear_noalloc: no CUDA device: %s", cudaGetErrorString(e));
  DevInfo* d;
  int r = init_device(dev, &d);
  if (r) return r;
  void* scratch = nullptr;
  r = scratch_for_device(dev, &scratch);
  if (r) return r;
  return lb_linear_ex(fmt, x, M, K, codes, scales, N, bias, accumulate, y, ldy, scratch,
                      static_cast<size_t>(LB_NOALLOC_SCRATCH_BYTES), 0u, stream);
}

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
//   * the first call on a device looks the array's address up (cudaGetSymbolAddress); make that first call
//     outside any stream capture.
#include "../../include/apsi_lowbit.h"
#include "lb_common.cuh"
#include "lb_kernels.h"

namespace lb {

static __device__ __align__(256) unsigned char g_noalloc_scratch[LB_NOALLOC_SCRATCH_BYTES];

namespace {
void* g_scratch_ptr[64];          // per device; set once
std::mutex g_scratch_mu;

int scratch_for_device(int dev, void** out) {
  if (dev < 0 || dev >= 64) return fail(LB_E_DEVICE, "device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);   // the current device's copy
    if (e != cudaSuccess || !p)
      return fail(LB_E_DEVICE, "lb_linear_noalloc: cudaGetSymbolAddress of the scratch failed on device %d: %s",
                  dev, cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return LB_OK;
}
}  // namespace

}  // namespace lb

extern "C" int lb_linear_noalloc(int fmt, const void* x, int64_t M, int64_t K, const void* codes, const void* scales,
                                 int64_t N, const void* bias, int accumulate, void* y, int64_t ldy, void* stream) {
  using namespace lb;
  const bool fp6 = (fmt == LB_FMT_FP6_E3M2 || fmt == LB_FMT_FP6_E2M3);
  if (fmt != LB_FMT_INT8_ROW && fmt != LB_FMT_INT4_G128 && fmt != LB_FMT_FP8_E4M3 && fmt != LB_FMT_FP8_E5M2 &&
      fmt != LB_FMT_FP4_E2M1 && !(fp6 && M <= 16))
    return fail(LB_E_UNSUPPORTED, "lb_linear_noalloc: format %d has no product kernel for M = %lld in this build", fmt,
                (long long)M);
  if (M <= 0 || N <= 0 || K <= 0) return fail(LB_E_ARG, "lb_linear_noalloc: M, N, K must be positive");
  if (M > (1LL << 31) || K > (1LL << 31)) return fail(LB_E_ARG, "lb_linear_noalloc: M and K must be below 2^31");
  if (M <= 16)   // decode path: no scratch at all
    return lb_linear_ex(fmt, x, M, K, codes, scales, N, bias, accumulate, y, ldy, nullptr, 0, 0u, stream);
  const size_t need = gemm_workspace_bytes(M, K);
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

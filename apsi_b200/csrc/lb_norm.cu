// RMSNorm of activation rows, the prologue of a normalised projection:
//   out[m, k] = bf16( x[m, k] * (1 / sqrt(mean_k(x[m, :]^2) + eps)) * (w[k] + off) )     (float32 arithmetic)
// as hub_gpu's rms op and the norm prologue of its gemvq*n kernels compute it (apsi/hub_gpu.py:1690-1693,
// 837-870; launched by _Base.linear with ln=..., apsi/hub_gpu.py:1305-1315).  The normalised rows are rounded
// to bfloat16 once, because the product kernels take bf16 activations.  One CTA per row; the sum of squares
// uses a fixed reduction tree (the same bits on every launch).  HBM-bound: 2 bytes read + 2 written per value.
#include "../../include/apsi_lowbit.h"
#include "lb_common.cuh"
#include "lb_kernels.h"

namespace lb {

template <int WDT>   // LB_DT_F32 or LB_DT_BF16 weights
__global__ void __launch_bounds__(256) rmsnorm_kernel(const uint16_t* __restrict__ x, int64_t K,
                                                      const void* __restrict__ wv, float eps, float off,
                                                      uint16_t* __restrict__ out) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const uint16_t* xr = x + row * K;
  uint16_t* orow = out + row * K;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  auto bf = [](uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); };
  float ss = 0.f;
  for (int64_t k = tid; k < K; k += 256) {
    const float v = bf(xr[k]);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float fac = 1.0f / sqrtf(tot / static_cast<float>(K) + eps);
  for (int64_t k = tid; k < K; k += 256) {
    const float w = (WDT == LB_DT_F32) ? static_cast<const float*>(wv)[k] : bf(static_cast<const uint16_t*>(wv)[k]);
    const float y = bf(xr[k]) * fac * (w + off);
    __nv_bfloat16 h = __float2bfloat16_rn(y);
    orow[k] = *reinterpret_cast<uint16_t*>(&h);
  }
}

}  // namespace lb

using namespace lb;

extern "C" int lb_rmsnorm(const void* x, int64_t M, int64_t K, const void* w, int w_dtype, float eps, float off,
                          void* out, void* stream) {
  if (!x || !w || !out) return fail(LB_E_ARG, "lb_rmsnorm: x, w and out are required");
  if (M <= 0 || K <= 0 || M > (1LL << 31)) return fail(LB_E_ARG, "lb_rmsnorm: M and K must be positive");
  if (w_dtype != LB_DT_F32 && w_dtype != LB_DT_BF16) return fail(LB_E_ARG, "lb_rmsnorm: w_dtype must be F32 or BF16");
  if (!aligned(x, 2) || !aligned(out, 2) || !aligned(w, w_dtype == LB_DT_F32 ? 4 : 2))
    return fail(LB_E_ALIGN, "lb_rmsnorm: pointers must be element aligned");
  DevInfo* d;
  int r = current(&d);
  if (r) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint16_t* xb = static_cast<const uint16_t*>(x);
  uint16_t* ob = static_cast<uint16_t*>(out);
  if (w_dtype == LB_DT_F32)
    rmsnorm_kernel<LB_DT_F32><<<static_cast<unsigned>(M), 256, 0, st>>>(xb, K, w, eps, off, ob);
  else
    rmsnorm_kernel<LB_DT_BF16><<<static_cast<unsigned>(M), 256, 0, st>>>(xb, K, w, eps, off, ob);
  return launched(cudaGetLastError(), "rmsnorm");
}

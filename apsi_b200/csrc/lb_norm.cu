// RMSNorm of activation rows, the prologue of a normalised projection:
//   out[m, k] = bf16( x[m, k] * (1 / sqrt(mean_k(x[m, :]^2) + eps)) * (w[k] + off) )     (float32 arithmetic)
// as hub_gpu's rms op and the norm prologue of its gemvq*n kernels compute it (apsi/hub_gpu.py:1690-1693,
// 837-870; launched by _Base.linear with ln=..., apsi/hub_gpu.py:1305-1315).  The normalised rows are rounded
// to bfloat16 once, because the product kernels take bf16 activations.  One CTA per row; the sum of squares
// uses the fixed reduction order of rms_chunk_fma / rms_butterfly (lb_common.cuh), the same one the decode
// GEMV's norm prologue uses, so lb_linear_rms gives the bits of lb_rmsnorm + lb_linear.  HBM-bound: 2 bytes
// read + 2 written per value.
#include "../../include/apsi_lowbit.h"
#include "lb_common.cuh"
#include "lb_kernels.h"

namespace lb {

template <int WDT>   // LB_DT_F32 or LB_DT_BF16 weights
__global__ void __launch_bounds__(RMS_VT) rmsnorm_kernel(const uint16_t* __restrict__ x, int64_t K,
                                                         const void* __restrict__ wv, float eps, float off,
                                                         uint16_t* __restrict__ out, int vec, int wvec) {
  __shared__ float red[RMS_VT / 32];
  pdl_launch_dependents();   // a following static-weight GEMV may start streaming its weights now (it waits for
                             // this grid before it reads the normalised rows)
  const int64_t row = blockIdx.x;
  const uint16_t* xr = x + row * K;
  uint16_t* orow = out + row * K;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t nc = (K + 7) / 8;
  float ss = 0.f;
  for (int64_t j = tid; j < nc; j += RMS_VT) ss = rms_chunk_fma(rms_load_chunk(xr, K, j, vec), ss);
  ss = rms_butterfly(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < RMS_VT / 32; ++i) tot += red[i];
  const float fac = rms_factor(tot, K, eps);
  for (int64_t j = tid; j < nc; j += RMS_VT) {
    const RmsW w = rms_load_w(wv, WDT == LB_DT_F32, 8 * j, K, wvec);
    const uint4 y = rms_apply_chunk(rms_load_chunk(xr, K, j, vec), fac, w, WDT == LB_DT_F32, off);
    if (vec) {
      *reinterpret_cast<uint4*>(orow + 8 * j) = y;
    } else {
      const uint32_t r[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (8 * j + e < K) orow[8 * j + e] = static_cast<uint16_t>(r[e >> 1] >> (16 * (e & 1)));
    }
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
  const int vec = (K % 8 == 0 && aligned(x, 16) && aligned(out, 16)) ? 1 : 0;
  const int wvec = (vec && aligned(w, 16)) ? 1 : 0;
  if (w_dtype == LB_DT_F32)
    rmsnorm_kernel<LB_DT_F32><<<static_cast<unsigned>(M), RMS_VT, 0, st>>>(xb, K, w, eps, off, ob, vec, wvec);
  else
    rmsnorm_kernel<LB_DT_BF16><<<static_cast<unsigned>(M), RMS_VT, 0, st>>>(xb, K, w, eps, off, ob, vec, wvec);
  return launched(cudaGetLastError(), "rmsnorm");
}

// The element-wise steps between a decoder's projections, as the reference's ops object defines them:
//
//   lb_qkv_prep  split the fused QKV projection into heads, optionally RMSNorm each q / k head, rotate the
//                first `rot` values of every q and k head (half-split pairs: [a cos - b sin, b cos + a sin]
//                with a = v[:rot/2], b = v[rot/2:rot], cos / sin from the caller's tables at the token's
//                position), write q to its output and k, v into the KV cache at the token's position
//                (apsi/hub_gpu.py:1701-1723, the host restatement of its qkv_prep kernel, 1547-1552);
//   lb_act_mul   out = act(g) * u for the fused [g | u] gate/up projection, act = silu (g / (1 + exp(-g))) or
//                the tanh form of gelu (apsi/hub_gpu.py:1755-1762, 1598-1600).
//
// Arithmetic is float32 on bf16 inputs, rounded once to bf16 on store.  Positions come from a device scalar
// (pos0 + t) when one is given, so a captured CUDA graph can advance them, else from `start`.  Memory-bound:
// one pass over the inputs, no intermediate buffers.
#include "../../include/apsi_lowbit.h"
#include "lb_common.cuh"
#include "lb_kernels.h"

namespace lb {

struct QkvPrepParams {
  const uint16_t* qkv;      // [B * T, (nh + 2 kvh) * dh]
  const float* cos;         // [cap, rot / 2]
  const float* sin;
  const uint16_t* qn;       // [dh] or null
  const uint16_t* kn;
  const int64_t* pos0;      // device scalar or null
  int64_t start;
  uint16_t* q;              // q[b, h, t, d] at b * qsb + t * qst + h * qsh + d
  uint16_t* kc;             // cache[b, h, p, d] at b * csb + h * csh + p * dh + d
  uint16_t* vc;
  int64_t qsb, qst, qsh, csb, csh;
  int B, T, nh, kvh, dh, rot;
  float eps;
};

__device__ __forceinline__ float bfv(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }
__device__ __forceinline__ uint16_t tobf(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}

// One CTA per (token, head of q / k / v); blockDim = 128 >= dh / 2 (one thread per rotated pair).
__global__ void __launch_bounds__(128) qkv_prep_kernel(const QkvPrepParams p) {
  pdl_launch_dependents();
  const int per = p.nh + 2 * p.kvh;
  const int64_t bt = blockIdx.x / per;
  const int hh = blockIdx.x % per;
  const int b = static_cast<int>(bt / p.T), t = static_cast<int>(bt % p.T);
  const int64_t pos = (p.pos0 ? *p.pos0 : p.start) + t;
  const uint16_t* src = p.qkv + bt * static_cast<int64_t>(per) * p.dh + static_cast<int64_t>(hh) * p.dh;
  const int half = p.rot / 2;
  const int tid = threadIdx.x;
  if (hh >= p.nh + p.kvh) {                       // v: copied into the cache
    uint16_t* dst = p.vc + b * p.csb + (hh - p.nh - p.kvh) * p.csh + pos * p.dh;
    for (int d = tid; d < p.dh; d += blockDim.x) dst[d] = src[d];
    return;
  }
  const bool isq = hh < p.nh;
  const uint16_t* w = isq ? p.qn : p.kn;
  float fac = 1.f;
  if (w) {                                        // per-head RMSNorm over dh values
    __shared__ float red[4];
    float ss = 0.f;
    for (int d = tid; d < p.dh; d += blockDim.x) { const float v = bfv(src[d]); ss = fmaf(v, v, ss); }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    const float tot = (red[0] + red[1]) + (red[2] + red[3]);
    fac = 1.0f / sqrtf(tot / static_cast<float>(p.dh) + p.eps);
  }
  auto val = [&](int d) { const float v = bfv(src[d]) * fac; return w ? v * bfv(w[d]) : v; };
  uint16_t* dst = isq ? p.q + b * p.qsb + t * p.qst + static_cast<int64_t>(hh) * p.qsh
                      : p.kc + b * p.csb + (hh - p.nh) * p.csh + pos * p.dh;
  for (int i = tid; i < half; i += blockDim.x) {  // rotated pairs (i, i + half)
    const float c = p.cos[pos * half + i], s = p.sin[pos * half + i];
    const float a = val(i), bb = val(i + half);
    dst[i] = tobf(a * c - bb * s);
    dst[i + half] = tobf(bb * c + a * s);
  }
  for (int d = p.rot + tid; d < p.dh; d += blockDim.x) dst[d] = tobf(val(d));   // the unrotated rest
}

// out[m, i] = act(gu[m, i]) * gu[m, I + i]; 8 values per thread when rows allow 16-byte access.
template <int KIND>
__device__ __forceinline__ float act(float g) {
  if (KIND == 0) return g / (1.0f + expf(-g));
  const float k0 = 0.7978845608028654f;            // sqrt(2 / pi)
  return 0.5f * g * (1.0f + tanhf(k0 * (g + 0.044715f * g * g * g)));
}

template <int KIND>
__global__ void __launch_bounds__(256) act_mul_kernel(const uint16_t* __restrict__ gu, int64_t M, int64_t I,
                                                      uint16_t* __restrict__ out, int vec) {
  pdl_launch_dependents();   // the down projection's GEMV may start streaming its weights (it waits for this grid)
  if (vec) {
    const int64_t n8 = M * (I / 8);
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < n8;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const int64_t m = e / (I / 8), j = (e % (I / 8)) * 8;
      const uint4 g4 = *reinterpret_cast<const uint4*>(gu + m * 2 * I + j);
      const uint4 u4 = *reinterpret_cast<const uint4*>(gu + m * 2 * I + I + j);
      const uint32_t gw[4] = {g4.x, g4.y, g4.z, g4.w}, uw[4] = {u4.x, u4.y, u4.z, u4.w};
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float lo = act<KIND>(__uint_as_float(gw[q] << 16)) * __uint_as_float(uw[q] << 16);
        const float hi = act<KIND>(__uint_as_float(gw[q] & 0xFFFF0000u)) * __uint_as_float(uw[q] & 0xFFFF0000u);
        o[q] = static_cast<uint32_t>(tobf(lo)) | (static_cast<uint32_t>(tobf(hi)) << 16);
      }
      *reinterpret_cast<uint4*>(out + m * I + j) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  } else {
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < M * I;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const int64_t m = e / I, i = e % I;
      out[e] = tobf(act<KIND>(bfv(gu[m * 2 * I + i])) * bfv(gu[m * 2 * I + I + i]));
    }
  }
}

}  // namespace lb

using namespace lb;

extern "C" {

int lb_qkv_prep(const void* qkv, int B, int T, int nh, int kvh, int dh, int rot, const float* cos, const float* sin,
                const void* qn, const void* kn, float eps, const int64_t* pos0, int64_t start, void* q,
                int64_t q_sb, int64_t q_st, int64_t q_sh, void* k_cache, void* v_cache, int64_t c_sb, int64_t c_sh,
                void* stream) {
  if (!qkv || !cos || !sin || !q || !k_cache || !v_cache) return fail(LB_E_ARG, "lb_qkv_prep: NULL pointer");
  if (B <= 0 || T <= 0 || nh <= 0 || kvh <= 0 || dh <= 0 || dh > 256 || rot < 0 || rot > dh || rot % 2)
    return fail(LB_E_ARG, "lb_qkv_prep: bad sizes (dh <= 256, rot even and <= dh)");
  if (nh % kvh) return fail(LB_E_ARG, "lb_qkv_prep: nh (%d) must be a multiple of kvh (%d)", nh, kvh);
  QkvPrepParams p;
  p.qkv = static_cast<const uint16_t*>(qkv);
  p.cos = cos; p.sin = sin;
  p.qn = static_cast<const uint16_t*>(qn);
  p.kn = static_cast<const uint16_t*>(kn);
  p.pos0 = pos0; p.start = start;
  p.q = static_cast<uint16_t*>(q);
  p.kc = static_cast<uint16_t*>(k_cache);
  p.vc = static_cast<uint16_t*>(v_cache);
  p.qsb = q_sb; p.qst = q_st; p.qsh = q_sh; p.csb = c_sb; p.csh = c_sh;
  p.B = B; p.T = T; p.nh = nh; p.kvh = kvh; p.dh = dh; p.rot = rot; p.eps = eps;
  DevInfo* d;
  int r = current(&d);
  if (r) return r;
  const int64_t blocks = static_cast<int64_t>(B) * T * (nh + 2 * kvh);
  if (blocks > 0x7FFFFFFF) return fail(LB_E_ARG, "lb_qkv_prep: too many tokens");
  qkv_prep_kernel<<<static_cast<unsigned>(blocks), 128, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return launched(cudaGetLastError(), "qkv_prep");
}

int lb_act_mul(const void* gu, int64_t M, int64_t I, int kind, void* out, void* stream) {
  if (!gu || !out) return fail(LB_E_ARG, "lb_act_mul: NULL pointer");
  if (M <= 0 || I <= 0) return fail(LB_E_ARG, "lb_act_mul: sizes must be positive");
  if (kind != 0 && kind != 1) return fail(LB_E_ARG, "lb_act_mul: kind must be 0 (silu) or 1 (gelu, tanh form)");
  DevInfo* d;
  int r = current(&d);
  if (r) return r;
  const int vec = (I % 8 == 0 && aligned(gu, 16) && aligned(out, 16));
  const int64_t work = vec ? M * (I / 8) : M * I;
  int64_t blocks = (work + 255) / 256;
  if (blocks > static_cast<int64_t>(d->sms) * 16) blocks = static_cast<int64_t>(d->sms) * 16;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint16_t* g = static_cast<const uint16_t*>(gu);
  uint16_t* o = static_cast<uint16_t*>(out);
  if (kind == 0) act_mul_kernel<0><<<static_cast<unsigned>(blocks), 256, 0, st>>>(g, M, I, o, vec);
  else act_mul_kernel<1><<<static_cast<unsigned>(blocks), 256, 0, st>>>(g, M, I, o, vec);
  return launched(cudaGetLastError(), "act_mul");
}

}  // extern "C"

// Quantisation / packing and dequantisation kernels (bandwidth-bound).
//
// Numerics follow apsi/precision.py:205-246 exactly:
//   scale = float32(absmax / qmax) computed in float64 (absmax > 0), else 1.0.  absmax of float32 values is a
//   float32 value and float64 -> float32 double rounding of a quotient of float32 numbers is innocuous
//   (53 >= 2*24 + 2), so the correctly rounded float32 division gives the same bits.
//   code  = clip(rint(float64(w) / float64(scale)), -qmax, qmax) with round half to even.  For float32 w and
//   scale the quotient can only round onto a half-integer in float64 when it IS that half-integer (a quotient
//   of two 24-bit significands is at least 2^-34 relative away from any other 9-bit number), so
//   rint(float64 quotient) == round-half-even of the exact quotient; the kernel computes that exactly:
//   a cheap float32 estimate away from half-integers, an exact side test (fma residual) near them.
// The ggml-style g32 formats follow apsi/hub_gpu.py:1215-1241 (float32 arithmetic) and the word packing of
// the quant8 / quant4 kernels (apsi/hub_gpu.py:786-800).
#include "lb_common.cuh"
#include "lb_kernels.h"

namespace lb {

template <int DT>
__device__ __forceinline__ float load_w(const void* w, int64_t i) {
  if (DT == 0) return __ldg(reinterpret_cast<const float*>(w) + i);
  uint16_t b = __ldg(reinterpret_cast<const unsigned short*>(w) + i);
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// Eight consecutive weights starting at element i (i multiple of 8).
template <int DT>
__device__ __forceinline__ void load_w8(const void* w, int64_t i, float (&v)[8]) {
  if (DT == 0) {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(w) + i);
    float4 a = __ldg(p), b = __ldg(p + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    uint4 u = ldg_nc_v4(reinterpret_cast<const unsigned short*>(w) + i);
    uint32_t r[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = __uint_as_float(r[j] << 16);
      v[2 * j + 1] = __uint_as_float(r[j] & 0xFFFF0000u);
    }
  }
}

// round-half-even(v / s) for s > 0, exactly.
__device__ __forceinline__ float round_quot(float v, float s, float inv) {
  float qf = v * inv;
  float r = rintf(qf);
  if (!(fabsf(qf - r) <= 0.4990234375f)) {  // near a half-integer (or inv overflowed): decide exactly
    if (s < 1e-30f) {                       // keep the residual below clear of underflow (exact 2^64 scaling)
      v *= 18446744073709551616.0f;
      s *= 18446744073709551616.0f;
    }
    float qe = __fdiv_rn(v, s);
    r = rintf(qe);
    float fl = floorf(qe);
    if (qe - fl == 0.5f) {                  // float32 quotient sits on a half-integer: which side is exact?
      float e = fmaf(qe, s, -v);            // sign(qe * s - v), exact
      if (e > 0.f) r = fl;
      else if (e < 0.f) r = fl + 1.f;       // e == 0: a true tie, rintf already rounded to even
    }
  }
  return r;
}

__device__ __forceinline__ float absmax_scale(float m, float qmax) {
  return m > 0.f ? __fdiv_rn(m, qmax) : 1.0f;
}

// ------------------------------------------------------------------------------------------- int4, g128
// 8 threads per group of 128 values (16 each: two 8-value loads), so a warp quantises four groups per step and
// the per-group work (absmax tree, scale division, reciprocal) is shared by 16 values per thread.  The kernel is
// bound by its instruction stream, not by HBM, at 8 values per thread.  The reciprocal only feeds round_quot's
// estimate, which is checked against a margin (2^-10) far wider than the estimate's error and decided exactly
// otherwise, so the fast approximate division gives the same codes.  Shuffles name only the lanes of their own
// group: the groups of a warp may leave the loop at different steps.
template <int DT>
__global__ void __launch_bounds__(256) quant_int4_g128_kernel(const void* __restrict__ w, int64_t ngroups,
                                                              uint32_t* __restrict__ packed,
                                                              __half* __restrict__ scale16,
                                                              float* __restrict__ scale32) {
  const int sub = threadIdx.x & 7;
  const unsigned gmask = 0xFFu << (threadIdx.x & 24);
  int64_t g = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 3;
  const int64_t gstride = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 3;
  for (; g < ngroups; g += gstride) {  // uniform per 8-lane group
    float v[2][8];
    load_w8<DT>(w, g * 128 + sub * 16, v[0]);
    load_w8<DT>(w, g * 128 + sub * 16 + 8, v[1]);
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) m = fmaxf(m, fabsf(v[j >> 3][j & 7]));
#pragma unroll
    for (int o = 4; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(gmask, m, o, 8));
    const float s = absmax_scale(m, 7.0f);
    const float inv = __fdividef(1.0f, s);
    uint32_t word[2] = {0u, 0u};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float q = fminf(fmaxf(round_quot(v[j >> 3][j & 7], s, inv), -7.f), 7.f);
      word[j >> 3] |= (static_cast<uint32_t>(static_cast<int>(q)) & 0xFu) << (4 * (j & 7));
    }
    *reinterpret_cast<uint2*>(packed + g * 16 + sub * 2) = make_uint2(word[0], word[1]);
    if (sub == 0) {
      scale16[g] = __float2half_rn(s);
      if (scale32) scale32[g] = s;
    }
  }
}

// ------------------------------------------------------------------------------------------- int8, per row
// One block per row: pass 1 absmax, pass 2 codes (the row is re-read from L2).
template <int DT>
__global__ void __launch_bounds__(256) quant_int8_rows_kernel(const void* __restrict__ w, int64_t N, int64_t K,
                                                              int8_t* __restrict__ codes,
                                                              __half* __restrict__ scale16,
                                                              float* __restrict__ scale32) {
  __shared__ float red[8];
  for (int64_t row = blockIdx.x; row < N; row += gridDim.x) {
    const int64_t base = row * K;
    float m = 0.f;
    for (int64_t k = threadIdx.x * 8; k < K; k += 256 * 8) {
      float v[8];
      load_w8<DT>(w, base + k, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(v[j]));
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    m = red[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) m = fmaxf(m, red[i]);
    const float s = absmax_scale(m, 127.0f);
    const float inv = 1.0f / s;
    for (int64_t k = threadIdx.x * 8; k < K; k += 256 * 8) {
      float v[8];
      load_w8<DT>(w, base + k, v);
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float q = fminf(fmaxf(round_quot(v[j], s, inv), -127.f), 127.f);
        uint32_t b = static_cast<uint32_t>(static_cast<int>(q)) & 0xFFu;
        if (j < 4) lo |= b << (8 * j);
        else hi |= b << (8 * (j - 4));
      }
      *reinterpret_cast<uint2*>(codes + base + k) = make_uint2(lo, hi);
    }
    if (threadIdx.x == 0) {
      scale16[row] = __float2half_rn(s);
      if (scale32) scale32[row] = s;
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------------------- ggml g32
// Four threads per block of 32 values (8 each).  KIND 8: int8, scale = absmax/127; KIND 4: int4,
// scale = (first value of largest magnitude)/-8, codes stored as q + 8.  float32 arithmetic as qnumpy.
// Scale of one block of 32 values held 8 per thread by 4 consecutive lanes (sub = lane % 4), float32 as
// hub_gpu.qnumpy: int8 max|v| / 127; int4 the signed value of the first largest magnitude / -8.
// `quad` names the four lanes of the block (the quads of a warp may leave their loop at different steps).
template <int KIND>
__device__ __forceinline__ float g32_scale(const float (&v)[8], int sub, unsigned quad) {
  if (KIND == 8) {
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(v[j]));
#pragma unroll
    for (int o = 2; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(quad, m, o, 4));
    return __fdiv_rn(m, 127.0f);
  }
  // first index of the largest magnitude (numpy argmax), then its signed value
  float am = -1.f, mv = 0.f;
  int idx = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float a = fabsf(v[j]);
    if (a > am) { am = a; mv = v[j]; idx = sub * 8 + j; }
  }
#pragma unroll
  for (int o = 2; o >= 1; o >>= 1) {
    float oam = __shfl_xor_sync(quad, am, o, 4);
    float omv = __shfl_xor_sync(quad, mv, o, 4);
    int oidx = __shfl_xor_sync(quad, idx, o, 4);
    if (oam > am || (oam == am && oidx < idx)) { am = oam; mv = omv; idx = oidx; }
  }
  return __fdiv_rn(mv, -8.0f);
}

template <int DT, int KIND>
__global__ void __launch_bounds__(256) quant_g32_kernel(const void* __restrict__ w, int64_t nblocks,
                                                        uint32_t* __restrict__ words,
                                                        float* __restrict__ scale32) {
  const int sub = threadIdx.x & 3;
  const unsigned quad = 0xFu << (threadIdx.x & 28);
  int64_t b = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 2;
  const int64_t bstride = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 2;
  for (; b < nblocks; b += bstride) {
    float v[8];
    load_w8<DT>(w, b * 32 + sub * 8, v);
    const float sc = g32_scale<KIND>(v, sub, quad);
    const float inv = (sc != 0.f) ? __fdiv_rn(1.0f, sc) : 0.f;
    uint32_t out0 = 0, out1 = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float q = rintf(__fmul_rn(v[j], inv));
      if (KIND == 8) {
        q = fminf(fmaxf(q, -127.f), 127.f);
        uint32_t c = static_cast<uint32_t>(static_cast<int>(q)) & 0xFFu;
        if (j < 4) out0 |= c << (8 * j);
        else out1 |= c << (8 * (j - 4));
      } else {
        q = fminf(fmaxf(q, -8.f), 7.f);
        out0 |= (static_cast<uint32_t>(static_cast<int>(q) + 8) & 0xFu) << (4 * j);
      }
    }
    if (KIND == 8) {
      *reinterpret_cast<uint2*>(words + b * 8 + sub * 2) = make_uint2(out0, out1);
    } else {
      words[b * 4 + sub] = out0;
    }
    if (sub == 0) scale32[b] = sc;
  }
}

// lowbit.round_weights in one pass (apsi/lowbit.py:37-50 with hub_gpu.qnumpy): out = clip(rint(v * inv), lo,
// hi) * scale in float32, so a value that rounds to zero keeps its sign exactly as the reference's float
// arithmetic does (integer codes would lose it).
template <int DT, int KIND>
__global__ void __launch_bounds__(256) round_g32_kernel(const void* __restrict__ w, int64_t nblocks,
                                                        float* __restrict__ out) {
  const int sub = threadIdx.x & 3;
  const unsigned quad = 0xFu << (threadIdx.x & 28);
  int64_t b = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 2;
  const int64_t bstride = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 2;
  for (; b < nblocks; b += bstride) {
    float v[8];
    load_w8<DT>(w, b * 32 + sub * 8, v);
    const float sc = g32_scale<KIND>(v, sub, quad);
    const float inv = (sc != 0.f) ? __fdiv_rn(1.0f, sc) : 0.f;
    const float lo = KIND == 8 ? -127.f : -8.f, hi = KIND == 8 ? 127.f : 7.f;
    float d[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) d[j] = __fmul_rn(fminf(fmaxf(rintf(__fmul_rn(v[j], inv)), lo), hi), sc);
    float4* o = reinterpret_cast<float4*>(out + b * 32 + sub * 8);
    o[0] = make_float4(d[0], d[1], d[2], d[3]);
    o[1] = make_float4(d[4], d[5], d[6], d[7]);
  }
}

// ------------------------------------------------------------------------------------------- dequantise
// One thread per 8 consecutive values.  FMT as LB_FMT_*; OUT 0 = float32, 1 = bfloat16; SF32: the scales are
// float32 (the reference's own scale) instead of binary16.
template <int FMT, int OUT, bool SF32>
__device__ __forceinline__ float load_scale(const void* scales, int64_t i) {
  if (SF32) return __ldg(reinterpret_cast<const float*>(scales) + i);
  return __half2float(__ldg(reinterpret_cast<const __half*>(scales) + i));
}

template <int FMT, int OUT, bool SF32>
__global__ void __launch_bounds__(256) dequant_kernel(const void* __restrict__ codes, const void* __restrict__ scales,
                                                      int64_t N, int64_t K, void* __restrict__ out) {
  const int64_t n8 = N * K / 8;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < n8;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e0 = t * 8;
    const int64_t row = e0 / K;
    const int64_t col = e0 - row * K;
    float q[8];
    float s;
    if (FMT == 2) {  // int4 g128, two's complement nibbles
      uint32_t wd = __ldg(reinterpret_cast<const uint32_t*>(codes) + t);
#pragma unroll
      for (int j = 0; j < 8; ++j) q[j] = static_cast<float>(static_cast<int>(wd << (28 - 4 * j)) >> 28);
      s = load_scale<FMT, OUT, SF32>(scales, row * (K / 128) + col / 128);
    } else if (FMT == 1) {  // int8 per row
      uint2 wd = __ldg(reinterpret_cast<const uint2*>(codes) + t);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        q[j] = static_cast<float>(static_cast<int8_t>(wd.x >> (8 * j)));
        q[j + 4] = static_cast<float>(static_cast<int8_t>(wd.y >> (8 * j)));
      }
      s = load_scale<FMT, OUT, SF32>(scales, row);
    } else if (FMT == 3) {  // q8_0 g32 words
      uint2 wd = __ldg(reinterpret_cast<const uint2*>(codes) + t);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        q[j] = static_cast<float>(static_cast<int8_t>(wd.x >> (8 * j)));
        q[j + 4] = static_cast<float>(static_cast<int8_t>(wd.y >> (8 * j)));
      }
      s = __ldg(reinterpret_cast<const float*>(scales) + row * (K / 32) + col / 32);
    } else {  // q4_0 g32 words, nibble = q + 8
      uint32_t wd = __ldg(reinterpret_cast<const uint32_t*>(codes) + t);
#pragma unroll
      for (int j = 0; j < 8; ++j) q[j] = static_cast<float>(static_cast<int>((wd >> (4 * j)) & 0xFu) - 8);
      s = __ldg(reinterpret_cast<const float*>(scales) + row * (K / 32) + col / 32);
    }
    if (OUT == 0) {
      float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + e0);
      o[0] = make_float4(q[0] * s, q[1] * s, q[2] * s, q[3] * s);
      o[1] = make_float4(q[4] * s, q[5] * s, q[6] * s, q[7] * s);
    } else {
      uint32_t r[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 p = __floats2bfloat162_rn(q[2 * j] * s, q[2 * j + 1] * s);
        r[j] = *reinterpret_cast<uint32_t*>(&p);
      }
      *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + e0) = make_uint4(r[0], r[1], r[2], r[3]);
    }
  }
}

// ------------------------------------------------------------------------------------------- launchers
static int grid_for(int64_t work_threads, int sms) {
  int64_t blocks = (work_threads + 255) / 256;
  int64_t cap = static_cast<int64_t>(sms) * 16;
  return static_cast<int>(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

cudaError_t launch_quant_int4_g128(const void* w, int dt, int64_t N, int64_t K, uint8_t* packed, uint16_t* s16,
                                   float* s32, int sms, cudaStream_t st) {
  const int64_t ng = N * (K / 128);
  const int grid = grid_for(ng * 8, sms);
  if (dt == 0)
    quant_int4_g128_kernel<0><<<grid, 256, 0, st>>>(w, ng, reinterpret_cast<uint32_t*>(packed),
                                                    reinterpret_cast<__half*>(s16), s32);
  else
    quant_int4_g128_kernel<1><<<grid, 256, 0, st>>>(w, ng, reinterpret_cast<uint32_t*>(packed),
                                                    reinterpret_cast<__half*>(s16), s32);
  return cudaGetLastError();
}

cudaError_t launch_quant_int8_rows(const void* w, int dt, int64_t N, int64_t K, int8_t* codes, uint16_t* s16,
                                   float* s32, int sms, cudaStream_t st) {
  const int grid = static_cast<int>(N < static_cast<int64_t>(sms) * 8 ? N : static_cast<int64_t>(sms) * 8);
  if (dt == 0)
    quant_int8_rows_kernel<0><<<grid, 256, 0, st>>>(w, N, K, codes, reinterpret_cast<__half*>(s16), s32);
  else
    quant_int8_rows_kernel<1><<<grid, 256, 0, st>>>(w, N, K, codes, reinterpret_cast<__half*>(s16), s32);
  return cudaGetLastError();
}

cudaError_t launch_quant_g32(int kind, const void* w, int dt, int64_t N, int64_t K, uint32_t* words, float* s32,
                             int sms, cudaStream_t st) {
  const int64_t nb = N * (K / 32);
  const int grid = grid_for(nb * 4, sms);
  if (kind == 8) {
    if (dt == 0) quant_g32_kernel<0, 8><<<grid, 256, 0, st>>>(w, nb, words, s32);
    else quant_g32_kernel<1, 8><<<grid, 256, 0, st>>>(w, nb, words, s32);
  } else {
    if (dt == 0) quant_g32_kernel<0, 4><<<grid, 256, 0, st>>>(w, nb, words, s32);
    else quant_g32_kernel<1, 4><<<grid, 256, 0, st>>>(w, nb, words, s32);
  }
  return cudaGetLastError();
}

cudaError_t launch_round_g32(int kind, const void* w, int dt, int64_t N, int64_t K, float* out, int sms,
                             cudaStream_t st) {
  const int64_t nb = N * (K / 32);
  const int grid = grid_for(nb * 4, sms);
  if (kind == 8) {
    if (dt == 0) round_g32_kernel<0, 8><<<grid, 256, 0, st>>>(w, nb, out);
    else round_g32_kernel<1, 8><<<grid, 256, 0, st>>>(w, nb, out);
  } else {
    if (dt == 0) round_g32_kernel<0, 4><<<grid, 256, 0, st>>>(w, nb, out);
    else round_g32_kernel<1, 4><<<grid, 256, 0, st>>>(w, nb, out);
  }
  return cudaGetLastError();
}

cudaError_t launch_dequant(int fmt, const void* codes, const void* scales, int sf32, int64_t N, int64_t K,
                           void* out, int out_dt, int sms, cudaStream_t st) {
  const int grid = grid_for(N * K / 8, sms);
#define LB_DQ(F, S)                                                                              \
  if (fmt == F && sf32 == S) {                                                                   \
    if (out_dt == 0) dequant_kernel<F, 0, S><<<grid, 256, 0, st>>>(codes, scales, N, K, out);    \
    else dequant_kernel<F, 1, S><<<grid, 256, 0, st>>>(codes, scales, N, K, out);                \
  }
  LB_DQ(1, 0) LB_DQ(1, 1) LB_DQ(2, 0) LB_DQ(2, 1) LB_DQ(3, 1) LB_DQ(4, 1)
#undef LB_DQ
  return cudaGetLastError();
}

}  // namespace lb

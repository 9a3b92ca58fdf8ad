// Minifloat weight formats (fp8 e4m3 / e5m2, fp6 e3m2 / e2m3, fp4 e2m1): absmax scales, encoding onto the
// format grid, packing and decoding, with the arithmetic of the reference's precision.quantize / dequantize
// (apsi/precision.py:23-138, 182-274).
//
//   scale   per row (axis 0): float32(max|row| / fmt.max), 1.0 when the maximum is 0 or NaN;
//           per tensor (axis None): max|x| is reduced on the device and the scale max / fmt.max is formed in
//           float64 (the reference keeps it as a Python float).
//   encode  y = float64(x) / scale; round to nearest on the grid with ties to the even code, magnitudes above
//           fmt.max saturate, the sign bit follows signbit(y) (so -0.0 keeps it), NaN takes the format's first
//           NaN code (or the all-ones magnitude when the format has none).  The rounding is done as rint() of
//           y scaled by the ulp of its binade (the smallest normal binade for subnormals and zero): exact in
//           float64, and the same grid point as the reference's search in its sorted value table.
//   pack    8-bit formats one byte per value; fp6 four values per three bytes (little-endian 24-bit word);
//           fp4 two per byte, the even flat index in the low nibble; flat row-major order, zero padding.
//   decode  the format's value of the code, times the float32 scale (one float32 multiply).
#include <math.h>
#include "lb_common.cuh"
#include "lb_kernels.h"

namespace lb {

template <int EB, int MB, int BIAS, bool FINITE, bool NANTOP>
struct Minifloat {
  static constexpr int EBITS = EB, MBITS = MB, BIASV = BIAS, MAG_BITS = EB + MB;
  static constexpr int TOP = (1 << EB) - 1;
  // largest finite magnitude code
  static constexpr int MAX_CODE = NANTOP ? ((TOP << MB) | ((1 << MB) - 2)) : (FINITE ? ((TOP << MB) | ((1 << MB) - 1))
                                                                                     : (((TOP - 1) << MB) | ((1 << MB) - 1)));
  // first NaN code (the all-ones magnitude when the format has no NaN)
  static constexpr int NAN_CODE = NANTOP ? ((TOP << MB) | ((1 << MB) - 1)) : (FINITE ? ((1 << (EB + MB)) - 1) : ((TOP << MB) | 1));

  __host__ __device__ static double max_value() {
    const int e = MAX_CODE >> MB, m = MAX_CODE & ((1 << MB) - 1);
    return ldexp(static_cast<double>((1 << MB) + m), e - BIAS - MB);
  }

  __device__ static uint32_t encode(double y) {
    if (isnan(y)) return NAN_CODE;
    const uint32_t sign = signbit(y) ? 1u : 0u;
    const double a = fmin(fabs(y), max_value());
    int e = 1 - BIAS;
    if (a > 0.0) {
      int ex;
      frexp(a, &ex);                       // a = f * 2^ex, f in [0.5, 1)
      e = max(ex - 1, 1 - BIAS);
    }
    const double r = rint(ldexp(a, MB - e));
    const uint32_t code = (static_cast<uint32_t>(e + BIAS) << MB) + static_cast<uint32_t>(r) - (1u << MB);
    return code | (sign << (EB + MB));
  }

  __device__ static float decode(uint32_t code) {
    const uint32_t mag = code & ((1u << (EB + MB)) - 1u);
    const int e = static_cast<int>(mag >> MB), m = static_cast<int>(mag & ((1u << MB) - 1u));
    float v = (e == 0) ? ldexpf(static_cast<float>(m), 1 - BIAS - MB)
                       : ldexpf(static_cast<float>((1 << MB) + m), e - BIAS - MB);
    if (!FINITE && e == TOP) v = (m == 0) ? INFINITY : NAN;
    if (NANTOP && e == TOP && m == (1 << MB) - 1) v = NAN;
    return ((code >> (EB + MB)) & 1u) ? -v : v;
  }
};

using MfE4M3 = Minifloat<4, 3, 7, true, true>;
using MfE5M2 = Minifloat<5, 2, 15, false, false>;
using MfE3M2 = Minifloat<3, 2, 3, true, false>;
using MfE2M3 = Minifloat<2, 3, 1, true, false>;
using MfE2M1 = Minifloat<2, 1, 1, true, false>;

int minifloat_bits(int fmt) {
  switch (fmt) {
    case 5: case 6: return 8;
    case 7: case 8: return 6;
    case 9: return 4;
    default: return 0;
  }
}

int64_t minifloat_bytes(int fmt, int64_t n) {
  const int bits = minifloat_bits(fmt);
  if (bits == 8) return n;
  if (bits == 6) return ((n + 3) / 4) * 3;
  if (bits == 4) return (n + 1) / 2;
  return -1;
}

__device__ __forceinline__ float load_w(const void* w, int dt, int64_t i) {
  if (dt == 1) return __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(w)[i]) << 16);
  return reinterpret_cast<const float*>(w)[i];
}

// |x| as ordered bits: non-negative floats order like their bit patterns, and every NaN (exponent all ones,
// mantissa non-zero) is above +inf, so an unsigned maximum propagates NaN as numpy's max does
__device__ __forceinline__ uint32_t abs_bits(float v) { return __float_as_uint(v) & 0x7FFFFFFFu; }

// per row: scale32[r] = float32(max / fmt.max), or 1.0 for a zero or NaN maximum
template <class F>
__global__ void __launch_bounds__(256) mf_rowscale_kernel(const void* w, int dt, int64_t R, int64_t C,
                                                          float* scale32) {
  __shared__ uint32_t red[8];
  for (int64_t r = blockIdx.x; r < R; r += gridDim.x) {
    uint32_t m = 0;
    for (int64_t c = threadIdx.x; c < C; c += blockDim.x) m = max(m, abs_bits(load_w(w, dt, r * C + c)));
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t mm = 0;
      for (int i = 0; i < (int)(blockDim.x >> 5); ++i) mm = max(mm, red[i]);
      const float mf = __uint_as_float(mm);
      scale32[r] = (mm > 0u && !isnan(mf)) ? static_cast<float>(static_cast<double>(mf) / F::max_value()) : 1.0f;
    }
    __syncthreads();
  }
}

// per tensor: absmax bits reduced with an atomic maximum (the word starts at zero)
__global__ void __launch_bounds__(256) mf_tensormax_kernel(const void* w, int dt, int64_t n, uint32_t* absmax) {
  uint32_t m = 0;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    m = max(m, abs_bits(load_w(w, dt, i)));
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0 && m) atomicMax(absmax, m);
}

__device__ __forceinline__ double tensor_scale(const uint32_t* absmax, double fmax) {
  const uint32_t mm = *absmax;
  const float mf = __uint_as_float(mm);
  return (mm > 0u && !isnan(mf)) ? static_cast<double>(mf) / fmax : 1.0;
}

// 8 values per thread (flat index 8t .. 8t + 7): encode, pack, store the bytes that belong to them
template <class F>
__global__ void __launch_bounds__(256) mf_encode_kernel(const void* w, int dt, int64_t R, int64_t C, int per_row,
                                                        const float* scale32, const uint32_t* absmax, uint8_t* out) {
  constexpr int BITS = (F::MAG_BITS + 1 == 8) ? 8 : ((F::MAG_BITS + 1 == 6) ? 6 : 4);
  const int64_t n = R * C;
  const double ts = per_row ? 1.0 : tensor_scale(absmax, F::max_value());
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t * 8 < n;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint32_t c[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t i = t * 8 + j;
      c[j] = 0u;
      if (i < n) {
        const double s = per_row ? static_cast<double>(scale32[i / C]) : ts;
        c[j] = F::encode(static_cast<double>(load_w(w, dt, i)) / s);
      }
    }
    if (BITS == 8) {
      const int64_t base = t * 8;
      if (base + 8 <= n) {
        *reinterpret_cast<uint2*>(out + base) = make_uint2(c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24),
                                                           c[4] | (c[5] << 8) | (c[6] << 16) | (c[7] << 24));
      } else {
        for (int j = 0; j < 8 && base + j < n; ++j) out[base + j] = static_cast<uint8_t>(c[j]);
      }
    } else if (BITS == 4) {
      const int64_t base = t * 4, nb = (n + 1) / 2;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (base + j < nb) out[base + j] = static_cast<uint8_t>((c[2 * j] & 0xFu) | ((c[2 * j + 1] & 0xFu) << 4));
    } else {
      const int64_t base = t * 6, nb = ((n + 3) / 4) * 3;
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        const uint32_t word = (c[4 * g] & 63u) | ((c[4 * g + 1] & 63u) << 6) | ((c[4 * g + 2] & 63u) << 12) |
                              ((c[4 * g + 3] & 63u) << 18);
#pragma unroll
        for (int b = 0; b < 3; ++b)
          if (base + 3 * g + b < nb) out[base + 3 * g + b] = static_cast<uint8_t>(word >> (8 * b));
      }
    }
  }
}

template <class F>
__global__ void __launch_bounds__(256) mf_decode_kernel(const uint8_t* codes, int64_t R, int64_t C, int per_row,
                                                        const float* scale32, float tscale, void* out, int out_dt) {
  constexpr int BITS = (F::MAG_BITS + 1 == 8) ? 8 : ((F::MAG_BITS + 1 == 6) ? 6 : 4);
  const int64_t n = R * C;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t * 8 < n;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint32_t c[8];
    if (BITS == 8) {
#pragma unroll
      for (int j = 0; j < 8; ++j) c[j] = (t * 8 + j < n) ? codes[t * 8 + j] : 0u;
    } else if (BITS == 4) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t b = (t * 8 + 2 * j < n) ? codes[t * 4 + j] : 0u;
        c[2 * j] = b & 0xFu;
        c[2 * j + 1] = b >> 4;
      }
    } else {
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        uint32_t word = 0u;
        if (t * 8 + 4 * g < n)
          word = codes[t * 6 + 3 * g] | (codes[t * 6 + 3 * g + 1] << 8) | (codes[t * 6 + 3 * g + 2] << 16);
#pragma unroll
        for (int k = 0; k < 4; ++k) c[4 * g + k] = (word >> (6 * k)) & 63u;
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t i = t * 8 + j;
      if (i < n) {
        const float s = per_row ? scale32[i / C] : tscale;
        const float v = __fmul_rn(F::decode(c[j]), s);
        if (out_dt == 1) {
          __nv_bfloat16 h = __float2bfloat16_rn(v);
          reinterpret_cast<uint16_t*>(out)[i] = *reinterpret_cast<uint16_t*>(&h);
        } else {
          reinterpret_cast<float*>(out)[i] = v;
        }
      }
    }
  }
}

template <class F>
static cudaError_t launch_mf_quant_t(const void* w, int dt, int64_t R, int64_t C, int per_row, uint8_t* codes,
                                     float* scale32, float* absmax, int sms, cudaStream_t st) {
  const int64_t n = R * C;
  if (per_row) {
    const unsigned g = static_cast<unsigned>(R < 65535 ? R : 65535);
    mf_rowscale_kernel<F><<<g, 256, 0, st>>>(w, dt, R, C, scale32);
  } else {
    cudaError_t e = cudaMemsetAsync(absmax, 0, sizeof(float), st);
    if (e != cudaSuccess) return e;
    const int64_t want = (n + 255) / 256;
    const unsigned g = static_cast<unsigned>(want < sms * 8 ? (want > 0 ? want : 1) : sms * 8);
    mf_tensormax_kernel<<<g, 256, 0, st>>>(w, dt, n, reinterpret_cast<uint32_t*>(absmax));
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int64_t groups = (n + 7) / 8;
  const int64_t want = (groups + 255) / 256;
  const unsigned g = static_cast<unsigned>(want < sms * 16 ? (want > 0 ? want : 1) : sms * 16);
  mf_encode_kernel<F><<<g, 256, 0, st>>>(w, dt, R, C, per_row, scale32, reinterpret_cast<const uint32_t*>(absmax),
                                         codes);
  return cudaGetLastError();
}

cudaError_t launch_quant_minifloat(int fmt, const void* w, int dt, int64_t R, int64_t C, int per_row,
                                   uint8_t* codes, float* scale32, float* absmax, int sms, cudaStream_t st) {
  switch (fmt) {
    case 5: return launch_mf_quant_t<MfE4M3>(w, dt, R, C, per_row, codes, scale32, absmax, sms, st);
    case 6: return launch_mf_quant_t<MfE5M2>(w, dt, R, C, per_row, codes, scale32, absmax, sms, st);
    case 7: return launch_mf_quant_t<MfE3M2>(w, dt, R, C, per_row, codes, scale32, absmax, sms, st);
    case 8: return launch_mf_quant_t<MfE2M3>(w, dt, R, C, per_row, codes, scale32, absmax, sms, st);
    case 9: return launch_mf_quant_t<MfE2M1>(w, dt, R, C, per_row, codes, scale32, absmax, sms, st);
    default: return cudaErrorInvalidValue;
  }
}

template <class F>
static cudaError_t launch_mf_decode_t(const uint8_t* codes, int64_t R, int64_t C, int per_row, const float* scale32,
                                      float tscale, void* out, int out_dt, int sms, cudaStream_t st) {
  const int64_t groups = (R * C + 7) / 8;
  const int64_t want = (groups + 255) / 256;
  const unsigned g = static_cast<unsigned>(want < sms * 16 ? (want > 0 ? want : 1) : sms * 16);
  mf_decode_kernel<F><<<g, 256, 0, st>>>(codes, R, C, per_row, scale32, tscale, out, out_dt);
  return cudaGetLastError();
}

cudaError_t launch_dequant_minifloat(int fmt, const uint8_t* codes, int64_t R, int64_t C, int per_row,
                                     const float* scale32, float tscale, void* out, int out_dt, int sms,
                                     cudaStream_t st) {
  switch (fmt) {
    case 5: return launch_mf_decode_t<MfE4M3>(codes, R, C, per_row, scale32, tscale, out, out_dt, sms, st);
    case 6: return launch_mf_decode_t<MfE5M2>(codes, R, C, per_row, scale32, tscale, out, out_dt, sms, st);
    case 7: return launch_mf_decode_t<MfE3M2>(codes, R, C, per_row, scale32, tscale, out, out_dt, sms, st);
    case 8: return launch_mf_decode_t<MfE2M3>(codes, R, C, per_row, scale32, tscale, out, out_dt, sms, st);
    case 9: return launch_mf_decode_t<MfE2M1>(codes, R, C, per_row, scale32, tscale, out, out_dt, sms, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace lb

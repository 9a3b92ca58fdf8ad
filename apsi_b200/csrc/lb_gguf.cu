// GGUF Q8_0 / Q4_0 block codec on the device, with the float32 arithmetic of the reference's writer and reader
// (apsi/modelio.py:56-95):
//
//   Q8_0  34 bytes per 32 values: binary16 d = amax / 127, then int8 sign(y) * floor(|y| + 0.5), y = x * (1 / d)
//         (1 / d taken as 0 when d == 0)
//   Q4_0  18 bytes per 32 values: binary16 d = x[first argmax |x|] / -8, then codes min(15, trunc(x * (1 / d) + 8.5)),
//         value j in the low nibble and value j + 16 in the high nibble of byte j
//
// One warp per block.  Every float32 operation is a separately rounded IEEE operation (__fmul_rn / __fadd_rn /
// __fdiv_rn), as numpy evaluates the expressions, so the bytes match the reference for finite inputs.
#include "lb_common.cuh"
#include "lb_kernels.h"

namespace lb {

__global__ void __launch_bounds__(256) gguf_encode_kernel(int kind, const float* __restrict__ x, int64_t nblocks,
                                                          uint8_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int bytes = kind == 8 ? 34 : 18;
  for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); b < nblocks; b += warps) {
    const float v = x[b * 32 + lane];
    uint8_t* o = out + b * bytes;
    if (kind == 8) {
      float m = fabsf(v);
#pragma unroll
      for (int s = 16; s >= 1; s >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, s));
      const float d = __fdiv_rn(m, 127.0f);
      const float inv = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
      const float y = __fmul_rn(v, inv);
      const float r = floorf(__fadd_rn(fabsf(y), 0.5f));
      const int q = y > 0.f ? static_cast<int>(r) : (y < 0.f ? -static_cast<int>(r) : 0);
      o[2 + lane] = static_cast<uint8_t>(static_cast<int8_t>(q));
      if (lane == 0) *reinterpret_cast<uint16_t*>(o) = __half_as_ushort(__float2half_rn(d));   // blocks are 2-byte aligned
    } else {
      // the signed value at the first largest magnitude
      float a = fabsf(v);
      int idx = lane;
#pragma unroll
      for (int s = 16; s >= 1; s >>= 1) {
        const float a2 = __shfl_xor_sync(0xffffffffu, a, s);
        const int i2 = __shfl_xor_sync(0xffffffffu, idx, s);
        if (a2 > a || (a2 == a && i2 < idx)) { a = a2; idx = i2; }
      }
      const float mx = __shfl_sync(0xffffffffu, v, idx);
      const float d = __fdiv_rn(mx, -8.0f);
      const float inv = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
      const float t = __fadd_rn(__fmul_rn(v, inv), 8.5f);
      int q = static_cast<int>(t);                 // truncation toward zero (t >= 0.5 here)
      q = q < 15 ? q : 15;
      const int hi = __shfl_down_sync(0xffffffffu, q, 16);
      if (lane < 16) o[2 + lane] = static_cast<uint8_t>((q & 0xF) | ((hi & 0xF) << 4));
      if (lane == 0) *reinterpret_cast<uint16_t*>(o) = __half_as_ushort(__float2half_rn(d));   // blocks are 2-byte aligned
    }
  }
}

__global__ void __launch_bounds__(256) gguf_decode_kernel(int kind, const uint8_t* __restrict__ in, int64_t nblocks,
                                                          float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int bytes = kind == 8 ? 34 : 18;
  for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); b < nblocks; b += warps) {
    const uint8_t* p = in + b * bytes;
    const uint16_t hb = static_cast<uint16_t>(p[0] | (p[1] << 8));
    const float d = __half2float(__ushort_as_half(hb));
    int q;
    if (kind == 8) {
      q = static_cast<int8_t>(p[2 + lane]);
    } else {
      const uint8_t byte = p[2 + (lane & 15)];
      q = static_cast<int>(lane < 16 ? (byte & 0xF) : (byte >> 4)) - 8;
    }
    out[b * 32 + lane] = __fmul_rn(static_cast<float>(q), d);
  }
}

cudaError_t launch_gguf(int encode, int kind, const void* src, int64_t n, void* dst, int sms, cudaStream_t st) {
  const int64_t nblocks = n / 32;
  const int64_t want = (nblocks + 7) / 8;
  const unsigned g = static_cast<unsigned>(want < sms * 16 ? (want > 0 ? want : 1) : sms * 16);
  if (encode)
    gguf_encode_kernel<<<g, 256, 0, st>>>(kind, reinterpret_cast<const float*>(src), nblocks,
                                          reinterpret_cast<uint8_t*>(dst));
  else
    gguf_decode_kernel<<<g, 256, 0, st>>>(kind, reinterpret_cast<const uint8_t*>(src), nblocks,
                                          reinterpret_cast<float*>(dst));
  return cudaGetLastError();
}

}  // namespace lb

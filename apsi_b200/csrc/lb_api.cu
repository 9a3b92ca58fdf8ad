// C ABI of the library (include/apsi_lowbit.h): argument checks, device setup, dispatch.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <atomic>
#include <mutex>
#include <new>

#include "../../include/apsi_lowbit.h"
#include "lb_common.cuh"
#include "lb_kernels.h"

namespace lb {
namespace {
thread_local char t_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
  return code;
}

struct DevInfo {
  std::atomic<int> ready{0};
  int sms = 0, l2 = 0, major = 0, minor = 0;
};
DevInfo g_dev[64];
std::mutex g_init_mu;

int init_device(int dev, DevInfo** out) {
  if (dev < 0 || dev >= 64) return fail(LB_E_DEVICE, "device %d out of range", dev);
  DevInfo& d = g_dev[dev];
  if (!d.ready.load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lk(g_init_mu);
    if (!d.ready.load(std::memory_order_relaxed)) {
      cudaDeviceProp prop;
      cudaError_t e = cudaGetDeviceProperties(&prop, dev);
      if (e != cudaSuccess) return fail(LB_E_DEVICE, "cudaGetDeviceProperties(%d): %s", dev, cudaGetErrorString(e));
      if (prop.major != 10)
        return fail(LB_E_DEVICE, "device %d is compute capability %d.%d; this library is built for sm_100a only",
                    dev, prop.major, prop.minor);
      d.sms = prop.multiProcessorCount;
      d.l2 = prop.l2CacheSize;
      d.major = prop.major;
      d.minor = prop.minor;
      d.ready.store(1, std::memory_order_release);
    }
  }
  *out = &d;
  return LB_OK;
}

int current(DevInfo** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(LB_E_DEVICE, "no CUDA device: %s", cudaGetErrorString(e));
  return init_device(dev, out);
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int launched(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return fail(LB_E_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  t_err[0] = 0;
  return LB_OK;
}

int check_weight_input(const void* w, int dt, int64_t N, int64_t K, int64_t kmult, const char* who) {
  if (!w) return fail(LB_E_ARG, "%s: weight pointer is NULL", who);
  if (dt != LB_DT_F32 && dt != LB_DT_BF16) return fail(LB_E_ARG, "%s: w_dtype must be LB_DT_F32 or LB_DT_BF16", who);
  if (N <= 0 || K <= 0) return fail(LB_E_ARG, "%s: N and K must be positive (got %lld, %lld)", who, (long long)N, (long long)K);
  if (K % kmult) return fail(LB_E_ARG, "%s: K (%lld) must be a multiple of %lld", who, (long long)K, (long long)kmult);
  if (!aligned(w, 16)) return fail(LB_E_ALIGN, "%s: weight pointer must be 16-byte aligned", who);
  return LB_OK;
}
}  // namespace

// ------------------------------------------------------------------------------------------- interleave
// [G][M][Nl] -> [M][G * Nl]: source row (g, m) of Nl values is destination row m, columns [g Nl, (g + 1) Nl).
// One CTA per row at a time; 16-byte vectors when the rows allow it (HBM-bound copy).
__global__ void interleave_kernel(const uint16_t* __restrict__ src, int G, int64_t M, int64_t Nl,
                                  uint16_t* __restrict__ dst, int vec) {
  const int64_t rows = static_cast<int64_t>(G) * M;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const int64_t g = r / M, m = r - g * M;
    const uint16_t* s = src + r * Nl;
    uint16_t* d = dst + (m * G + g) * Nl;
    if (vec) {
      const uint4* s4 = reinterpret_cast<const uint4*>(s);
      uint4* d4 = reinterpret_cast<uint4*>(d);
      for (int64_t j = threadIdx.x; j < Nl / 8; j += blockDim.x) d4[j] = s4[j];
    } else {
      for (int64_t j = threadIdx.x; j < Nl; j += blockDim.x) d[j] = s[j];
    }
  }
}

cudaError_t launch_interleave(const void* src, int G, int64_t M, int64_t Nl, void* dst, int sms, cudaStream_t st) {
  const int64_t rows = static_cast<int64_t>(G) * M;
  const int vec = (Nl % 8 == 0 && reinterpret_cast<uintptr_t>(src) % 16 == 0 && reinterpret_cast<uintptr_t>(dst) % 16 == 0);
  int64_t blocks = rows < static_cast<int64_t>(sms) * 8 ? rows : static_cast<int64_t>(sms) * 8;
  interleave_kernel<<<static_cast<unsigned>(blocks > 0 ? blocks : 1), 256, 0, st>>>(
      reinterpret_cast<const uint16_t*>(src), G, M, Nl, reinterpret_cast<uint16_t*>(dst), vec);
  return cudaGetLastError();
}

}  // namespace lb

using namespace lb;

extern "C" {

int lb_version(void) { return LB_VERSION; }

const char* lb_last_error(void) { return t_err; }

int lb_init(int device) {
  DevInfo* d;
  return init_device(device, &d);
}

int lb_device_errors(void* stream, int* bits_out) {
  if (!bits_out) return fail(LB_E_ARG, "lb_device_errors: bits_out is NULL");
  DevInfo* d;
  int r = current(&d);
  if (r) return r;
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(LB_E_DEVICE, "lb_device_errors: %s", cudaGetErrorString(e));
  int v = 0, zero = 0;
  e = cudaMemcpyFromSymbol(&v, g_dev_errors, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_dev_errors, &zero, sizeof(int));
  if (e != cudaSuccess) return fail(LB_E_DEVICE, "lb_device_errors: %s", cudaGetErrorString(e));
  *bits_out = v;
  return LB_OK;
}

int lb_quant_int8_rows(const void* w, int w_dtype, int64_t N, int64_t K, int8_t* codes, uint16_t* scale16,
                       float* scale32, void* stream) {
  int r = check_weight_input(w, w_dtype, N, K, 8, "lb_quant_int8_rows");
  if (r) return r;
  if (!codes || !scale16) return fail(LB_E_ARG, "lb_quant_int8_rows: codes and scale16 are required");
  if (!aligned(codes, 8) || !aligned(scale16, 2) || (scale32 && !aligned(scale32, 4)))
    return fail(LB_E_ALIGN, "lb_quant_int8_rows: codes must be 8-byte aligned");
  DevInfo* d;
  if ((r = current(&d))) return r;
  return launched(launch_quant_int8_rows(w, w_dtype, N, K, codes, scale16, scale32, d->sms,
                                         static_cast<cudaStream_t>(stream)),
                  "quant_int8_rows");
}

int lb_quant_int4_g128(const void* w, int w_dtype, int64_t N, int64_t K, uint8_t* packed, uint16_t* scale16,
                       float* scale32, void* stream) {
  int r = check_weight_input(w, w_dtype, N, K, 128, "lb_quant_int4_g128");
  if (r) return r;
  if (!packed || !scale16) return fail(LB_E_ARG, "lb_quant_int4_g128: packed and scale16 are required");
  if (!aligned(packed, 4) || !aligned(scale16, 2) || (scale32 && !aligned(scale32, 4)))
    return fail(LB_E_ALIGN, "lb_quant_int4_g128: packed must be 4-byte aligned");
  DevInfo* d;
  if ((r = current(&d))) return r;
  return launched(launch_quant_int4_g128(w, w_dtype, N, K, packed, scale16, scale32, d->sms,
                                         static_cast<cudaStream_t>(stream)),
                  "quant_int4_g128");
}

static int quant_g32(int kind, const void* w, int w_dtype, int64_t N, int64_t K, uint32_t* words, float* scale32,
                     void* stream, const char* who) {
  int r = check_weight_input(w, w_dtype, N, K, 32, who);
  if (r) return r;
  if (!words || !scale32) return fail(LB_E_ARG, "%s: words and scale32 are required", who);
  if (!aligned(words, 8) || !aligned(scale32, 4)) return fail(LB_E_ALIGN, "%s: words must be 8-byte aligned", who);
  DevInfo* d;
  if ((r = current(&d))) return r;
  return launched(launch_quant_g32(kind, w, w_dtype, N, K, words, scale32, d->sms, static_cast<cudaStream_t>(stream)),
                  who);
}

int lb_quant_q8_0_g32(const void* w, int w_dtype, int64_t N, int64_t K, uint32_t* words, float* scale32,
                      void* stream) {
  return quant_g32(8, w, w_dtype, N, K, words, scale32, stream, "lb_quant_q8_0_g32");
}

int lb_quant_q4_0_g32(const void* w, int w_dtype, int64_t N, int64_t K, uint32_t* words, float* scale32,
                      void* stream) {
  return quant_g32(4, w, w_dtype, N, K, words, scale32, stream, "lb_quant_q4_0_g32");
}

int lb_round_g32(int fmt, const void* w, int w_dtype, int64_t N, int64_t K, float* out, void* stream) {
  if (fmt != LB_FMT_Q8_0_G32 && fmt != LB_FMT_Q4_0_G32)
    return fail(LB_E_UNSUPPORTED, "lb_round_g32: format %d is not a g32 format", fmt);
  int r = check_weight_input(w, w_dtype, N, K, 32, "lb_round_g32");
  if (r) return r;
  if (!out) return fail(LB_E_ARG, "lb_round_g32: out is required");
  if (!aligned(out, 16)) return fail(LB_E_ALIGN, "lb_round_g32: out must be 16-byte aligned");
  DevInfo* d;
  if ((r = current(&d))) return r;
  return launched(launch_round_g32(fmt == LB_FMT_Q8_0_G32 ? 8 : 4, w, w_dtype, N, K, out, d->sms,
                                   static_cast<cudaStream_t>(stream)),
                  "lb_round_g32");
}

int lb_dequant(int fmt, const void* codes, const void* scales, int scale_dtype, int64_t N, int64_t K, void* out,
               int out_dtype, void* stream) {
  if (fmt < LB_FMT_INT8_ROW || fmt > LB_FMT_Q4_0_G32) return fail(LB_E_ARG, "lb_dequant: unknown format %d", fmt);
  if (!codes || !scales || !out) return fail(LB_E_ARG, "lb_dequant: NULL pointer");
  if (out_dtype != LB_DT_F32 && out_dtype != LB_DT_BF16) return fail(LB_E_ARG, "lb_dequant: bad out_dtype");
  if (scale_dtype != LB_DT_F32 && scale_dtype != LB_DT_F16) return fail(LB_E_ARG, "lb_dequant: bad scale_dtype");
  if ((fmt == LB_FMT_Q8_0_G32 || fmt == LB_FMT_Q4_0_G32) && scale_dtype != LB_DT_F32)
    return fail(LB_E_ARG, "lb_dequant: the g32 formats have float32 scales");
  if (N <= 0 || K <= 0) return fail(LB_E_ARG, "lb_dequant: N and K must be positive");
  const int64_t kmult = fmt == LB_FMT_INT4_G128 ? 128 : (fmt == LB_FMT_INT8_ROW ? 8 : 32);
  if (K % kmult) return fail(LB_E_ARG, "lb_dequant: K (%lld) must be a multiple of %lld", (long long)K, (long long)kmult);
  if (!aligned(codes, 8) || !aligned(out, 16) || !aligned(scales, scale_dtype == LB_DT_F32 ? 4 : 2))
    return fail(LB_E_ALIGN, "lb_dequant: codes 8-byte, out 16-byte, scales element aligned");
  DevInfo* d;
  int r = current(&d);
  if (r) return r;
  return launched(launch_dequant(fmt, codes, scales, scale_dtype == LB_DT_F32 ? 1 : 0, N, K, out, out_dtype, d->sms,
                                 static_cast<cudaStream_t>(stream)),
                  "dequant");
}

static bool is_minifloat(int fmt) { return fmt >= LB_FMT_FP8_E4M3 && fmt <= LB_FMT_FP4_E2M1; }

int64_t lb_minifloat_bytes(int fmt, int64_t n) {
  if (!is_minifloat(fmt) || n < 0) return -1;
  return minifloat_bytes(fmt, n);
}

int lb_quant_minifloat(int fmt, const void* w, int w_dtype, int64_t R, int64_t C, int per_row, uint8_t* codes,
                       float* scale32, float* absmax, void* stream) {
  if (!is_minifloat(fmt)) return fail(LB_E_ARG, "lb_quant_minifloat: %d is not a minifloat format", fmt);
  if (!w || !codes) return fail(LB_E_ARG, "lb_quant_minifloat: NULL pointer");
  if (w_dtype != LB_DT_F32 && w_dtype != LB_DT_BF16)
    return fail(LB_E_ARG, "lb_quant_minifloat: w_dtype must be LB_DT_F32 or LB_DT_BF16");
  if (R <= 0 || C <= 0) return fail(LB_E_ARG, "lb_quant_minifloat: R and C must be positive");
  if (per_row ? !scale32 : !absmax)
    return fail(LB_E_ARG, "lb_quant_minifloat: per_row needs scale32[R], per tensor needs absmax[1]");
  if (!aligned(w, w_dtype == LB_DT_F32 ? 4 : 2) || !aligned(codes, 8) || (scale32 && !aligned(scale32, 4)) ||
      (absmax && !aligned(absmax, 4)))
    return fail(LB_E_ALIGN, "lb_quant_minifloat: w element-aligned, codes 8-byte, scale32 / absmax 4-byte aligned");
  DevInfo* d;
  int r = current(&d);
  if (r) return r;
  return launched(launch_quant_minifloat(fmt, w, w_dtype, R, C, per_row, codes, scale32, absmax, d->sms,
                                         static_cast<cudaStream_t>(stream)),
                  "quant_minifloat");
}

int lb_dequant_minifloat(int fmt, const uint8_t* codes, int64_t R, int64_t C, int per_row, const float* scale32,
                         float tensor_scale, void* out, int out_dtype, void* stream) {
  if (!is_minifloat(fmt)) return fail(LB_E_ARG, "lb_dequant_minifloat: %d is not a minifloat format", fmt);
  if (!codes || !out || (per_row && !scale32)) return fail(LB_E_ARG, "lb_dequant_minifloat: NULL pointer");
  if (out_dtype != LB_DT_F32 && out_dtype != LB_DT_BF16) return fail(LB_E_ARG, "lb_dequant_minifloat: bad out_dtype");
  if (R <= 0 || C <= 0) return fail(LB_E_ARG, "lb_dequant_minifloat: R and C must be positive");
  if (!aligned(out, out_dtype == LB_DT_F32 ? 4 : 2) || (scale32 && !aligned(scale32, 4)))
    return fail(LB_E_ALIGN, "lb_dequant_minifloat: out and scale32 must be element-aligned");
  DevInfo* d;
  int r = current(&d);
  if (r) return r;
  return launched(launch_dequant_minifloat(fmt, codes, R, C, per_row, scale32, tensor_scale, out, out_dtype, d->sms,
                                           static_cast<cudaStream_t>(stream)),
                  "dequant_minifloat");
}

int lb_gguf_encode(int kind, const float* x, int64_t n, uint8_t* blocks, void* stream) {
  if (kind != 8 && kind != 4) return fail(LB_E_ARG, "lb_gguf_encode: kind must be 8 (Q8_0) or 4 (Q4_0)");
  if (!x || !blocks) return fail(LB_E_ARG, "lb_gguf_encode: NULL pointer");
  if (n <= 0 || n % 32) return fail(LB_E_ARG, "lb_gguf_encode: n (%lld) must be a positive multiple of 32", (long long)n);
  if (!aligned(x, 4)) return fail(LB_E_ALIGN, "lb_gguf_encode: x must be 4-byte aligned");
  DevInfo* d;
  int r = current(&d);
  if (r) return r;
  return launched(launch_gguf(1, kind, x, n, blocks, d->sms, static_cast<cudaStream_t>(stream)), "gguf_encode");
}

int lb_gguf_decode(int kind, const uint8_t* blocks, int64_t n, float* out, void* stream) {
  if (kind != 8 && kind != 4) return fail(LB_E_ARG, "lb_gguf_decode: kind must be 8 (Q8_0) or 4 (Q4_0)");
  if (!blocks || !out) return fail(LB_E_ARG, "lb_gguf_decode: NULL pointer");
  if (n <= 0 || n % 32) return fail(LB_E_ARG, "lb_gguf_decode: n (%lld) must be a positive multiple of 32", (long long)n);
  if (!aligned(out, 4)) return fail(LB_E_ALIGN, "lb_gguf_decode: out must be 4-byte aligned");
  DevInfo* d;
  int r = current(&d);
  if (r) return r;
  return launched(launch_gguf(0, kind, blocks, n, out, d->sms, static_cast<cudaStream_t>(stream)), "gguf_decode");
}

static bool use_gemv(int64_t M) { return M <= 16; }

// formats with a fused product: int8 rows, int4 groups of 128, fp8 e4m3 / e5m2, fp6 e3m2 / e2m3 and fp4 e2m1
// rows (float32 row scales); fp6 rows need K % 16 == 0 for the decode product and K % 64 == 0 above M = 16
static bool has_product(int fmt) {
  return fmt == LB_FMT_INT8_ROW || fmt == LB_FMT_INT4_G128 || (fmt >= LB_FMT_FP8_E4M3 && fmt <= LB_FMT_FP4_E2M1);
}
static bool is_fp6(int fmt) { return fmt == LB_FMT_FP6_E3M2 || fmt == LB_FMT_FP6_E2M3; }

int lb_linear_workspace_size(int fmt, int64_t M, int64_t N, int64_t K, size_t* bytes) {
  if (!bytes) return fail(LB_E_ARG, "lb_linear_workspace_size: bytes is NULL");
  if (!has_product(fmt))
    return fail(LB_E_UNSUPPORTED, "lb_linear: format %d has no product kernel in this build", fmt);
  if (M <= 0 || N <= 0 || K <= 0) return fail(LB_E_ARG, "lb_linear_workspace_size: sizes must be positive");
  if (!use_gemv(M) && is_fp6(fmt) && K % 64)
    return fail(LB_E_UNSUPPORTED, "lb_linear: fp6 products above M = 16 need K %% 64 == 0");
  *bytes = use_gemv(M) ? 0 : gemm_workspace_bytes(M, N, K);
  return LB_OK;
}

// Argument checks and dispatch shared by lb_linear_ex and lb_linear_sharded (dst: column-sharded outputs).
static int linear_impl(int fmt, const void* x, int64_t M, int64_t K, const void* codes, const void* scales, int64_t N,
                       const void* bias, int accumulate, void* y, int64_t ldy, void* workspace, size_t ws_bytes,
                       unsigned flags, void* stream, const OutRanks* dst, const RmsPrologue* ln = nullptr) {
  if (!has_product(fmt))
    return fail(LB_E_UNSUPPORTED, "lb_linear: format %d has no product kernel in this build", fmt);
  if (flags & ~static_cast<unsigned>(LB_LINEAR_STATIC_WEIGHTS)) return fail(LB_E_ARG, "lb_linear: unknown flags");
  if (!x || !codes || !scales || !y) return fail(LB_E_ARG, "lb_linear: x, codes, scales and y are required");
  if (M <= 0 || N <= 0 || K <= 0) return fail(LB_E_ARG, "lb_linear: M, N, K must be positive");
  if (M > (1LL << 31) || N > (1LL << 31)) return fail(LB_E_ARG, "lb_linear: M and N must be below 2^31");
  const int64_t kmult = (fmt == LB_FMT_INT4_G128 || fmt == LB_FMT_FP4_E2M1) ? 128 : (is_fp6(fmt) ? 16 : 64);
  if (K % kmult) return fail(LB_E_ARG, "lb_linear: K (%lld) must be a multiple of %lld", (long long)K, (long long)kmult);
  if (!use_gemv(M) && is_fp6(fmt) && K % 64)
    return fail(LB_E_UNSUPPORTED, "lb_linear: fp6 products above M = 16 need K %% 64 == 0");
  if (ldy < N) return fail(LB_E_ARG, "lb_linear: ldy (%lld) < N (%lld)", (long long)ldy, (long long)N);
  if (!aligned(x, 16) || !aligned(codes, 16) || !aligned(scales, 16))
    return fail(LB_E_ALIGN, "lb_linear: x, codes and scales must be 16-byte aligned");
  if (!aligned(y, 2) || (bias && !aligned(bias, 2))) return fail(LB_E_ALIGN, "lb_linear: y and bias must be 2-byte aligned");
  if (use_gemv(M) && K > gemv_max_k(fmt))
    return fail(LB_E_UNSUPPORTED, "lb_linear: K (%lld) above %d is not supported for M <= 16", (long long)K,
                gemv_max_k(fmt));
  size_t need = use_gemv(M) ? 0 : gemm_workspace_bytes(M, N, K);
  if (need) {
    if (!workspace || ws_bytes < need)
      return fail(LB_E_WORKSPACE, "lb_linear: workspace of %zu bytes needed (got %zu)", need, workspace ? ws_bytes : 0);
    if (!aligned(workspace, 256)) return fail(LB_E_ALIGN, "lb_linear: workspace must be 256-byte aligned");
  }
  DevInfo* d;
  int r = current(&d);
  if (r) return r;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool pdl = (flags & LB_LINEAR_STATIC_WEIGHTS) != 0;
  if (use_gemv(M))
    return launched(launch_gemv(fmt, x, M, K, codes, scales, N, bias, accumulate, y, ldy, d->sms, pdl, st, dst, ln),
                    "gemv");
  const char* why = nullptr;
  cudaError_t e = launch_gemm(fmt, x, M, K, codes, scales, N, bias, accumulate, y, ldy, workspace, d->sms, st, &why, dst);
  if (e != cudaSuccess && why) return fail(LB_E_LAUNCH, "gemm: %s (%s)", why, cudaGetErrorString(e));
  return launched(e, "gemm");
}

int lb_linear_ex(int fmt, const void* x, int64_t M, int64_t K, const void* codes, const void* scales, int64_t N,
                 const void* bias, int accumulate, void* y, int64_t ldy, void* workspace, size_t ws_bytes,
                 unsigned flags, void* stream) {
  return linear_impl(fmt, x, M, K, codes, scales, N, bias, accumulate, y, ldy, workspace, ws_bytes, flags, stream,
                     nullptr);
}

int lb_linear(int fmt, const void* x, int64_t M, int64_t K, const void* codes, const void* scales, int64_t N,
              const void* bias, int accumulate, void* y, int64_t ldy, void* workspace, size_t ws_bytes,
              void* stream) {
  return lb_linear_ex(fmt, x, M, K, codes, scales, N, bias, accumulate, y, ldy, workspace, ws_bytes, 0u, stream);
}

// A weight prepared for repeated decode products: everything lb_linear_ex checks about the weight is checked
// once, and the tensor maps of its stream are encoded once; a call then checks x, y and the device and launches.
struct lb_weight {
  int fmt;
  const void* codes;
  const void* scales;
  int64_t N, K;
  int dev, sms;
  GemvMaps maps;
};

int lb_weight_create(int fmt, const void* codes, const void* scales, int64_t N, int64_t K, lb_weight** out) {
  if (!out) return fail(LB_E_ARG, "lb_weight_create: out is NULL");
  *out = nullptr;
  if (!has_product(fmt))
    return fail(LB_E_UNSUPPORTED, "lb_weight_create: format %d has no product kernel in this build", fmt);
  if (!codes || !scales) return fail(LB_E_ARG, "lb_weight_create: codes and scales are required");
  if (N <= 0 || K <= 0) return fail(LB_E_ARG, "lb_weight_create: N and K must be positive");
  if (N > (1LL << 31)) return fail(LB_E_ARG, "lb_weight_create: N must be below 2^31");
  const int64_t kmult = (fmt == LB_FMT_INT4_G128 || fmt == LB_FMT_FP4_E2M1) ? 128 : (is_fp6(fmt) ? 16 : 64);
  if (K % kmult) return fail(LB_E_ARG, "lb_weight_create: K (%lld) must be a multiple of %lld", (long long)K, (long long)kmult);
  if (K > gemv_max_k(fmt))
    return fail(LB_E_UNSUPPORTED, "lb_weight_create: K (%lld) above %d is not supported for M <= 16", (long long)K,
                gemv_max_k(fmt));
  if (!aligned(codes, 16) || !aligned(scales, 16))
    return fail(LB_E_ALIGN, "lb_weight_create: codes and scales must be 16-byte aligned");
  DevInfo* d;
  int r = current(&d);
  if (r) return r;
  int dev = 0;
  cudaGetDevice(&dev);
  lb_weight* w = new (std::nothrow) lb_weight;
  if (!w) return fail(LB_E_ARG, "lb_weight_create: out of host memory");
  w->fmt = fmt;
  w->codes = codes;
  w->scales = scales;
  w->N = N;
  w->K = K;
  w->dev = dev;
  w->sms = d->sms;
  prepare_gemv_maps(fmt, codes, scales, N, K, &w->maps);
  *out = w;
  return LB_OK;
}

int lb_weight_linear(const lb_weight* w, const void* x, int64_t M, void* y, int64_t ldy, unsigned flags,
                     void* stream) {
  if (!w) return fail(LB_E_ARG, "lb_weight_linear: the weight is NULL");
  if (M <= 0) return fail(LB_E_ARG, "lb_weight_linear: M must be positive");
  if (!use_gemv(M))
    return fail(LB_E_UNSUPPORTED, "lb_weight_linear: M (%lld) above 16 needs lb_linear with a workspace", (long long)M);
  if (flags & ~static_cast<unsigned>(LB_LINEAR_STATIC_WEIGHTS)) return fail(LB_E_ARG, "lb_weight_linear: unknown flags");
  if (!x || !y) return fail(LB_E_ARG, "lb_weight_linear: x and y are required");
  if (ldy < w->N) return fail(LB_E_ARG, "lb_weight_linear: ldy (%lld) < N (%lld)", (long long)ldy, (long long)w->N);
  if (!aligned(x, 16) || !aligned(y, 2)) return fail(LB_E_ALIGN, "lb_weight_linear: x must be 16-byte and y 2-byte aligned");
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != w->dev)
    return fail(LB_E_DEVICE, "lb_weight_linear: the weight was prepared on device %d, the current device is %d", w->dev,
                dev);
  return launched(launch_gemv(w->fmt, x, M, w->K, w->codes, w->scales, w->N, nullptr, 0, y, ldy, w->sms,
                              (flags & LB_LINEAR_STATIC_WEIGHTS) != 0, static_cast<cudaStream_t>(stream), nullptr,
                              nullptr, &w->maps),
                  "gemv");
}

int lb_weight_destroy(lb_weight* w) {
  delete w;
  return LB_OK;
}

static size_t rms_rows_bytes(int64_t M, int64_t K) { return (static_cast<size_t>(M) * K * 2 + 255) & ~static_cast<size_t>(255); }

int lb_linear_rms_workspace_size(int fmt, int64_t M, int64_t N, int64_t K, size_t* bytes) {
  int r = lb_linear_workspace_size(fmt, M, N, K, bytes);
  if (r) return r;
  if (!use_gemv(M)) *bytes += rms_rows_bytes(M, K);
  return LB_OK;
}

int lb_linear_rms(int fmt, const void* x, int64_t M, int64_t K, const void* ln_w, int ln_dtype, float eps, float off,
                  const void* codes, const void* scales, int64_t N, const void* bias, int accumulate, void* y,
                  int64_t ldy, void* workspace, size_t ws_bytes, unsigned flags, void* stream) {
  if (!ln_w) return fail(LB_E_ARG, "lb_linear_rms: ln_w is required");
  if (is_fp6(fmt)) return fail(LB_E_UNSUPPORTED, "lb_linear_rms: fp6 formats have no normalised product");
  if (ln_dtype != LB_DT_F32 && ln_dtype != LB_DT_BF16) return fail(LB_E_ARG, "lb_linear_rms: ln_dtype must be F32 or BF16");
  if (!aligned(ln_w, ln_dtype == LB_DT_F32 ? 4 : 2)) return fail(LB_E_ALIGN, "lb_linear_rms: ln_w must be element aligned");
  if (use_gemv(M)) {
    const RmsPrologue ln{ln_w, ln_dtype == LB_DT_F32 ? 1 : 0, eps, off};
    return linear_impl(fmt, x, M, K, codes, scales, N, bias, accumulate, y, ldy, nullptr, 0, flags, stream, nullptr,
                       &ln);
  }
  // prefill: the normalised rows go to the front of the workspace, the product's own workspace follows
  if (!x || !codes || !scales || !y) return fail(LB_E_ARG, "lb_linear: x, codes, scales and y are required");
  if (M <= 0 || N <= 0 || K <= 0) return fail(LB_E_ARG, "lb_linear: M, N, K must be positive");
  size_t need = 0;
  int r = lb_linear_rms_workspace_size(fmt, M, N, K, &need);
  if (r) return r;
  if (!workspace || ws_bytes < need)
    return fail(LB_E_WORKSPACE, "lb_linear_rms: workspace of %zu bytes needed (got %zu)", need, workspace ? ws_bytes : 0);
  if (!aligned(workspace, 256)) return fail(LB_E_ALIGN, "lb_linear_rms: workspace must be 256-byte aligned");
  r = lb_rmsnorm(x, M, K, ln_w, ln_dtype, eps, off, workspace, stream);
  if (r) return r;
  const size_t head = rms_rows_bytes(M, K);
  return linear_impl(fmt, workspace, M, K, codes, scales, N, bias, accumulate, y, ldy,
                     static_cast<char*>(workspace) + head, ws_bytes - head, flags, stream, nullptr);
}

int lb_interleave_cols(const void* src, int G, int64_t M, int64_t Nl, void* dst, void* stream) {
  if (!src || !dst) return fail(LB_E_ARG, "lb_interleave_cols: NULL pointer");
  if (G <= 0 || M <= 0 || Nl <= 0) return fail(LB_E_ARG, "lb_interleave_cols: sizes must be positive");
  DevInfo* d;
  int r = current(&d);
  if (r) return r;
  return launched(launch_interleave(src, G, M, Nl, dst, d->sms, static_cast<cudaStream_t>(stream)), "interleave");
}

}  // extern "C"

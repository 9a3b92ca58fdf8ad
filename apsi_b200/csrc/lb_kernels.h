// Internal launchers (host side) shared between the kernel files and the C ABI in lb_api.cu.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace lb {

// Where a product's outputs go.  n == 0: the caller's y.  n > 0 (column-sharded layer): every rank's full
// output y[g] ([M, ldy], the same ldy on every rank), this rank's columns starting at col0; the stores to other
// ranks' buffers go over NVLink (peer memory opened through CUDA IPC).
constexpr int kMaxRanks = 8;
struct OutRanks {
  uint16_t* y[kMaxRanks];
  int n;
  int64_t col0;
};

cudaError_t launch_quant_int4_g128(const void* w, int dt, int64_t N, int64_t K, uint8_t* packed, uint16_t* s16,
                                   float* s32, int sms, cudaStream_t st);
cudaError_t launch_quant_int8_rows(const void* w, int dt, int64_t N, int64_t K, int8_t* codes, uint16_t* s16,
                                   float* s32, int sms, cudaStream_t st);
cudaError_t launch_quant_g32(int kind, const void* w, int dt, int64_t N, int64_t K, uint32_t* words, float* s32,
                             int sms, cudaStream_t st);
cudaError_t launch_round_g32(int kind, const void* w, int dt, int64_t N, int64_t K, float* out, int sms,
                             cudaStream_t st);
cudaError_t launch_dequant(int fmt, const void* codes, const void* scales, int sf32, int64_t N, int64_t K,
                           void* out, int out_dt, int sms, cudaStream_t st);

int gemv_max_k(int fmt);
// RMSNorm prologue of a normalised projection (the rows of x are normalised before the product)
struct RmsPrologue {
  const void* w;   // [K] float32 or bf16
  int w_f32;
  float eps, off;
};

// The tensor maps of an int4 weight's stream (box mode of the decode GEMV), encoded once for a prepared weight.
// ok == 0: no maps (the launch takes the row-copy path, as when encoding fails).
struct GemvMaps {
  int ok;
  int stma;                  // the scales have a tensor map too
  CUtensorMap tw, ts;
};
void prepare_gemv_maps(int fmt, const void* codes, const void* scales, int64_t N, int64_t K, GemvMaps* m);

cudaError_t launch_gemv(int fmt, const void* x, int64_t M, int64_t K, const void* codes, const void* scales,
                        int64_t N, const void* bias, int acc, void* y, int64_t ldy, int sms, bool pdl,
                        cudaStream_t st, const OutRanks* dst = nullptr, const RmsPrologue* ln = nullptr,
                        const GemvMaps* maps = nullptr);

size_t gemm_workspace_bytes(int64_t M, int64_t N, int64_t K);
cudaError_t launch_gemm(int fmt, const void* x, int64_t M, int64_t K, const void* codes, const void* scales,
                        int64_t N, const void* bias, int acc, void* y, int64_t ldy, void* ws, int sms,
                        cudaStream_t st, const char** why, const OutRanks* dst = nullptr);

int minifloat_bits(int fmt);
int64_t minifloat_bytes(int fmt, int64_t n);
cudaError_t launch_quant_minifloat(int fmt, const void* w, int dt, int64_t R, int64_t C, int per_row,
                                   uint8_t* codes, float* scale32, float* absmax, int sms, cudaStream_t st);
cudaError_t launch_dequant_minifloat(int fmt, const uint8_t* codes, int64_t R, int64_t C, int per_row,
                                     const float* scale32, float tscale, void* out, int out_dt, int sms,
                                     cudaStream_t st);

cudaError_t launch_gguf(int encode, int kind, const void* src, int64_t n, void* dst, int sms, cudaStream_t st);

cudaError_t launch_interleave(const void* src, int G, int64_t M, int64_t Nl, void* dst, int sms, cudaStream_t st);

}  // namespace lb

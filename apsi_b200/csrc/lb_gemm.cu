// Prefill-regime product (M > 16 tokens) on the 5th-generation tensor cores (tcgen05).
//
//   D[n, m] = sum_k deq(W)[n, k] * x[m, k]      A = W tile (128 weight rows)   in shared memory (dequantised)
//                                                B = x tile (BN tokens)         in shared memory (TMA, SW128)
//                                                D = fp32 accumulators          in TENSOR MEMORY, two of them
//
// The weights arrive as 4/8-bit codes (TMA, a few KB per stage) and eight dequantising warps expand them into
// the fp16 A tile in shared memory, in the same 128-byte swizzled K-major layout the TMA gives the activation
// tile, so one `tcgen05.mma` (both operands from shared memory) consumes them.  Tensor memory then only holds
// accumulators: two of BN columns each, so four epilogue warps drain tile i while the MMAs of tile i + 1 run.
//
// Operands are fp16: codes are exact in fp16 and int4 weights are fp16(q * s16) with a single rounding
// (relative error <= 2^-11); the activations are converted once by prep_x_kernel with a per-row power-of-two
// factor so the conversion is exact (bf16 mantissas fit in fp16) and cannot overflow; the factor is undone in
// the epilogue.  int8 rows keep exact codes and apply the row scale in float32 in the epilogue.
//
// Roles (14 warps, persistent over work units):
//   warp 0        TMA producer: activation tile (BN x 64 fp16, SW128) + raw code tile (128 rows) per stage
//   warp 1        TMEM allocator and MMA issuer (one thread): 4 x tcgen05.mma K=16 per stage, commit -> mbarrier
//   warps 2..9    dequantise one row x one half of the stage's K into the A tile (st.shared + proxy fence)
//   warps 10..13  epilogue: tcgen05.ld -> scale / bias / accumulate -> bf16 -> global
// Measured and not kept for narrow token tiles ([28672, 8192] at M = 64, 121 us as built): a separate code ring
// up to 32 k-steps deep beside 4 x / A stages (131 us), and 128-byte-wide code tiles (4 k-steps of a row per
// copy, SWIZZLE_128B, 16 k-steps in flight) beside 6 x / A stages (125 us); and a TMA ring of activation + code
// tiles as deep as shared memory allows (13 / 8 / 5 k-steps for 64 / 128 / 256 tokens) beside a separate ring of
// 4 / 3 / 2 dequantised A tiles (124 us; configs[2] 196 -> 200 us).  With the dequantisation, the
// MMAs and the activation reloads all removed the same pipeline still took 66 us: the stage round trip, not
// the code stream, sets the pace there.
//
// Split K (M <= 128 and long K): a tile's k-steps are cut into `splits` equal parts computed by different CTAs;
// each writes its float32 accumulators to a workspace and splitk_reduce_kernel adds the parts in split order
// and applies the epilogue.  The split count depends on M and K only, so column shards sum the same way.
//
// All mbarrier waits are bounded (lb::mbar_wait); a timeout sets the device error word and the CTA drains.
#include <string.h>
#include "lb_common.cuh"
#include "lb_tmap.h"
#include "lb_kernels.h"

namespace lb {

namespace gemm {
constexpr int BM = 128;     // weight rows per tile = TMEM lanes
constexpr int BK = 64;      // K values per stage (128 bytes of fp16: one SW128 row)
constexpr int DQ_WARPS = 8;
constexpr int EPI_WARPS = 4;
constexpr int THREADS = (2 + DQ_WARPS + EPI_WARPS) * 32;   // TMA, MMA, dequantisers, epilogue
constexpr int A_STAGE = BM * BK * 2;                       // 16 KB of fp16 weights per stage
constexpr int SMEM_LIMIT = 227 * 1024;
constexpr int TAIL = 512;                                  // mbarriers, TMEM address, abort flag
// code bytes of a row per k-step: 4-bit 32, 6-bit 48 (four codes per three bytes), 8-bit 64
__host__ __device__ constexpr int raw_row(int fmt) { return (fmt == 2 || fmt == 9) ? 32 : ((fmt == 7 || fmt == 8) ? 48 : 64); }
__host__ __device__ constexpr int raw_bytes(int fmt) { return BM * raw_row(fmt); }
// Pipeline depth: as many stages as shared memory holds (at most 8).  Narrow token tiles (small M) carry few
// weight bytes per stage, so they need the deepest pipelines to keep enough of the weight stream in flight.
__host__ __device__ constexpr int stages(int fmt, int bn) {
  return (SMEM_LIMIT - 1024 - TAIL) / (bn * 128 + A_STAGE + raw_bytes(fmt)) > 8
             ? 8 : (SMEM_LIMIT - 1024 - TAIL) / (bn * 128 + A_STAGE + raw_bytes(fmt));
}
}  // namespace gemm

// K splits (see the file comment): M <= 128 and at least 224 k-steps, about 112 k-steps per split, at most 8;
// the k-steps of a split are even (a whole number of int4 scale groups).
// Depends on M and K only.
__host__ __device__ inline int gemm_splits(int64_t M, int64_t K) {
  if (M > 128) return 1;
  const int64_t s = (K / gemm::BK) / 112;
  return s < 2 ? 1 : (s > 8 ? 8 : static_cast<int>(s));
}

struct GemmParams {
  const __half* s16;        // int4: [N, K/128]; int8: [N]
  const uint16_t* bias;     // bf16 [N] or null
  uint16_t* y;              // bf16 [M, ldy]
  const float* tokscale;    // [M] power-of-two factors from prep_x_kernel
  int64_t M, N, K, ldy;
  int acc;
  int m_blocks, n_blocks, tiles, ksteps;
  // Work units.  Units [0, full) are whole BM x BN tiles.  When the last wave of tiles would leave most SMs
  // idle, tiles full .. tiles - 1 are each cut along the tokens into `parts` units of sbn = BN / parts tokens
  // (the MMA's N and the activation box shrink; k order and accumulation per output are unchanged).
  int units, full, parts, sbn;
  int splits, kper;         // K splits (1: none) and k-steps per split (even)
  float* part;              // splits > 1: float32 accumulators [splits][M][N]
  OutRanks dst;             // column-sharded layer: every rank's output (dst.n == 0: y)
};

// unit -> weight row block, first token, tokens, k-steps [k0, k1), split
__device__ __forceinline__ void gemm_unit(const GemmParams& p, int u, int bn, int& mb, int& tok0, int& width, int& k0,
                                          int& k1, int& split) {
  split = 0;
  if (p.splits > 1) {
    split = u % p.splits;
    u /= p.splits;
  }
  k0 = split * p.kper;
  k1 = k0 + p.kper < p.ksteps ? k0 + p.kper : p.ksteps;
  int tile, part = 0;
  if (u < p.full) {
    tile = u;
  } else {
    const int s = u - p.full;
    tile = p.full + s / p.parts;
    part = s - (s / p.parts) * p.parts;
  }
  mb = tile / p.n_blocks;
  const int nb = tile - mb * p.n_blocks;
  tok0 = nb * bn + part * p.sbn;
  width = u < p.full ? bn : p.sbn;
}

template <int FMT>
struct GemmCfg {
  static constexpr int RAW_ROW = gemm::raw_row(FMT);                  // code bytes of a row per stage
  static constexpr int RAW_STAGE = gemm::BM * RAW_ROW;
};

template <int BN>
struct GemmSmem {
  static constexpr int X_STAGE = BN * 128;
  static constexpr int TMEM_COLS = (2 * BN <= 128) ? 128 : (2 * BN <= 256 ? 256 : 512);   // two accumulators
};

__device__ __forceinline__ uint16_t f32_to_bf16_bits_g(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}

// ------------------------------------------------------------------------------------------- activations
// One warp per token row: absmax, power-of-two factor, K-permuted fp16 copy.
// PERM 0 (int4 nibble pairs): position L of each 8-block takes x[8b + {0,4,1,5,2,6,3,7}[L]].
// PERM 1 (int8 byte pairs):   position L of each 4-block takes x[4b + {0,2,1,3}[L]].
// PERM 2 (fp4 code pairs):    no permutation.
template <int PERM>
__global__ void __launch_bounds__(256) prep_x_kernel(const uint16_t* __restrict__ x, int64_t M, int64_t K,
                                                     uint16_t* __restrict__ x16, float* __restrict__ tokscale) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= M) return;
  const uint16_t* xr = x + row * K;
  float m = 0.f;
#pragma unroll 8
  for (int64_t k = lane * 8; k < K; k += 256) {
    uint4 v = ldg_nc_v4(xr + k);
    uint32_t r[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      m = fmaxf(m, fabsf(__uint_as_float(r[j] << 16)));
      m = fmaxf(m, fabsf(__uint_as_float(r[j] & 0xFFFF0000u)));
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  int e = 0;
  if (m > 0.f) {
    int ex;
    frexpf(m, &ex);           // m = f * 2^ex, f in [0.5, 1)
    e = ex - 15;              // max |x| * 2^-e in [2^14, 2^15)
    e = e < -110 ? -110 : (e > 110 ? 110 : e);
  }
  const float down = ldexpf(1.0f, -e);
  if (lane == 0) tokscale[row] = ldexpf(1.0f, e);
  uint16_t* out = x16 + row * K;
#pragma unroll 8
  for (int64_t k = lane * 8; k < K; k += 256) {
    uint4 v = ldg_nc_v4(xr + k);
    uint32_t r[4] = {v.x, v.y, v.z, v.w};
    float f[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      f[2 * j] = __uint_as_float(r[j] << 16) * down;
      f[2 * j + 1] = __uint_as_float(r[j] & 0xFFFF0000u) * down;
    }
    float g[8];
    if (PERM == 0) {
      g[0] = f[0]; g[1] = f[4]; g[2] = f[1]; g[3] = f[5]; g[4] = f[2]; g[5] = f[6]; g[6] = f[3]; g[7] = f[7];
    } else if (PERM == 2) {
#pragma unroll
      for (int j = 0; j < 8; ++j) g[j] = f[j];
    } else {
      g[0] = f[0]; g[1] = f[2]; g[2] = f[1]; g[3] = f[3]; g[4] = f[4]; g[5] = f[6]; g[6] = f[5]; g[7] = f[7];
    }
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __half2 h = __floats2half2_rn(g[2 * j], g[2 * j + 1]);
      o[j] = *reinterpret_cast<uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(out + k) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// The same conversion with one 256-thread block per row and the row held in registers (CH 16-byte chunks per
// thread, rows of up to CH * 2048 values): x is read from HBM once, not twice, and a row's loads are all in
// flight together.  The factor and every converted value are those of prep_x_kernel (the maximum does not
// depend on the order it is taken in).
template <int PERM>
__device__ __forceinline__ uint4 prep_chunk(uint4 v, float down) {
  const uint32_t r[4] = {v.x, v.y, v.z, v.w};
  float f[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = __uint_as_float(r[j] << 16) * down;
    f[2 * j + 1] = __uint_as_float(r[j] & 0xFFFF0000u) * down;
  }
  float g[8];
  if (PERM == 0) {
    g[0] = f[0]; g[1] = f[4]; g[2] = f[1]; g[3] = f[5]; g[4] = f[2]; g[5] = f[6]; g[6] = f[3]; g[7] = f[7];
  } else if (PERM == 2) {
#pragma unroll
    for (int j = 0; j < 8; ++j) g[j] = f[j];
  } else {
    g[0] = f[0]; g[1] = f[2]; g[2] = f[1]; g[3] = f[3]; g[4] = f[4]; g[5] = f[6]; g[6] = f[5]; g[7] = f[7];
  }
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __half2 h = __floats2half2_rn(g[2 * j], g[2 * j + 1]);
    o[j] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

template <int PERM, int CH>
__global__ void __launch_bounds__(256) prep_x_rows_kernel(const uint16_t* __restrict__ x, int64_t K,
                                                          uint16_t* __restrict__ x16, float* __restrict__ tokscale) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const int nch = static_cast<int>(K / 8);
  const uint16_t* xr = x + row * K;
  uint4 v[CH];
  float m = 0.f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int ch = threadIdx.x + c * 256;
    v[c] = ch < nch ? ldg_nc_v4(xr + ch * 8) : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const uint32_t r[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      m = fmaxf(m, fabsf(__uint_as_float(r[j] << 16)));
      m = fmaxf(m, fabsf(__uint_as_float(r[j] & 0xFFFF0000u)));
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) m = fmaxf(m, red[i]);
  int e = 0;
  if (m > 0.f) {
    int ex;
    frexpf(m, &ex);
    e = ex - 15;
    e = e < -110 ? -110 : (e > 110 ? 110 : e);
  }
  const float down = ldexpf(1.0f, -e);
  if (threadIdx.x == 0) tokscale[row] = ldexpf(1.0f, e);
  uint16_t* out = x16 + row * K;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int ch = threadIdx.x + c * 256;
    if (ch < nch) *reinterpret_cast<uint4*>(out + ch * 8) = prep_chunk<PERM>(v[c], down);
  }
}

template <int PERM>
static void launch_prep_x(const uint16_t* x, int64_t M, int64_t K, uint16_t* x16, float* tokscale, cudaStream_t st) {
  const int64_t chunks = (K / 8 + 255) / 256;                 // 16-byte chunks per thread
  if (chunks <= 1) prep_x_rows_kernel<PERM, 1><<<static_cast<unsigned>(M), 256, 0, st>>>(x, K, x16, tokscale);
  else if (chunks <= 2) prep_x_rows_kernel<PERM, 2><<<static_cast<unsigned>(M), 256, 0, st>>>(x, K, x16, tokscale);
  else if (chunks <= 4) prep_x_rows_kernel<PERM, 4><<<static_cast<unsigned>(M), 256, 0, st>>>(x, K, x16, tokscale);
  else prep_x_kernel<PERM><<<static_cast<unsigned>((M + 7) / 8), 256, 0, st>>>(x, M, K, x16, tokscale);
}

// ------------------------------------------------------------------------------------------- dequantisers
// int4: 16 bytes = 32 codes of one row (k = 8i + j for word i, nibble j) -> 16 fp16 pairs in logical K order
// (pair 4i + p holds physical nibbles (p, p + 4) of word i), each fp16(q * s).
__device__ __forceinline__ void deq_int4_f16(const uint4 raw, uint32_t s2, uint32_t (&o)[16]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t v = w[i];
    const uint32_t v8 = v >> 8;
    // 1024 + (q + 8) and 1024 + 16 (q + 8): offset-binary through the XOR folded into the LOP3
    const uint32_t p0 = lop3_and_xor_or(v, 0x000F000Fu, 0x64086408u);
    const uint32_t p1 = lop3_and_xor_or(v, 0x00F000F0u, 0x64806480u);
    const uint32_t p2 = lop3_and_xor_or(v8, 0x000F000Fu, 0x64086408u);
    const uint32_t p3 = lop3_and_xor_or(v8, 0x00F000F0u, 0x64806480u);
    // exact codes: p0 - 1032 ; p1 / 16 - 72
    const uint32_t q0 = h2_fma(p0, 0x3C003C00u, 0xE408E408u);
    const uint32_t q1 = h2_fma(p1, 0x2C002C00u, 0xD480D480u);
    const uint32_t q2 = h2_fma(p2, 0x3C003C00u, 0xE408E408u);
    const uint32_t q3 = h2_fma(p3, 0x2C002C00u, 0xD480D480u);
    o[4 * i + 0] = h2_mul(q0, s2);
    o[4 * i + 1] = h2_mul(q1, s2);
    o[4 * i + 2] = h2_mul(q2, s2);
    o[4 * i + 3] = h2_mul(q3, s2);
  }
}
// int8: 32 bytes of one row -> 16 fp16 pairs of exact codes; pair 2i holds bytes (0, 2), pair 2i+1 bytes
// (1, 3) of word i.
__device__ __forceinline__ void deq_int8_f16(const uint4 a, const uint4 b, uint32_t (&o)[16]) {
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t v = w[i] ^ 0x80808080u;                       // q + 128
    const uint32_t p02 = prmt(v, 0x00006464u, 0x5240u);          // (1024 + n0, 1024 + n2)
    const uint32_t p13 = prmt(v, 0x00006464u, 0x5341u);          // (1024 + n1, 1024 + n3)
    o[2 * i] = h2_fma(p02, 0x3C003C00u, 0xE480E480u);            // - 1152
    o[2 * i + 1] = h2_fma(p13, 0x3C003C00u, 0xE480E480u);
  }
}

// fp4 rows: 16 bytes = 32 codes of one row -> 16 exact fp16 pairs in natural K order (pair 4i + p holds codes
// 8i + 2p, 8i + 2p + 1), through the hardware e2m1 conversion; the row scale is applied in the epilogue.
__device__ __forceinline__ void deq_fp4_f16(const uint4 raw, uint32_t (&o)[16]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t p[4];
    deq_fp4_word(w[i], p);
    o[4 * i] = p[0]; o[4 * i + 1] = p[1]; o[4 * i + 2] = p[2]; o[4 * i + 3] = p[3];
  }
}

// fp6 rows: 24 bytes of one row (8 groups of three bytes = 32 codes; value j of a group at bits 6j .. 6j + 5 of
// its little-endian 24-bit word) -> 16 exact fp16 pairs in natural K order through the hardware conversion;
// the row scale is applied in the epilogue.
template <int FMT>
__device__ __forceinline__ void deq_fp6_f16(const uint32_t (&w)[6], uint32_t (&o)[16]) {
  const uint32_t g[8] = {w[0] & 0xFFFFFFu, (w[0] >> 24) | ((w[1] << 8) & 0xFFFF00u),
                         (w[1] >> 16) | ((w[2] << 16) & 0xFF0000u), w[2] >> 8,
                         w[3] & 0xFFFFFFu, (w[3] >> 24) | ((w[4] << 8) & 0xFFFF00u),
                         (w[4] >> 16) | ((w[5] << 16) & 0xFF0000u), w[5] >> 8};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    // the four 6-bit fields into the low bits of four bytes, then two codes per conversion
    const uint32_t u = (g[i] & 0x3Fu) | ((g[i] << 2) & 0x3F00u) | ((g[i] << 4) & 0x3F0000u) | ((g[i] << 6) & 0x3F000000u);
    uint32_t lo, hi;
    if (FMT == 7) {
      asm("{\n\t.reg .b16 a;\n\tcvt.u16.u32 a, %1;\n\tcvt.rn.f16x2.e3m2x2 %0, a;\n\t}" : "=r"(lo) : "r"(u));
      asm("{\n\t.reg .b16 a;\n\tcvt.u16.u32 a, %1;\n\tcvt.rn.f16x2.e3m2x2 %0, a;\n\t}" : "=r"(hi) : "r"(u >> 16));
    } else {
      asm("{\n\t.reg .b16 a;\n\tcvt.u16.u32 a, %1;\n\tcvt.rn.f16x2.e2m3x2 %0, a;\n\t}" : "=r"(lo) : "r"(u));
      asm("{\n\t.reg .b16 a;\n\tcvt.u16.u32 a, %1;\n\tcvt.rn.f16x2.e2m3x2 %0, a;\n\t}" : "=r"(hi) : "r"(u >> 16));
    }
    o[2 * i] = lo;
    o[2 * i + 1] = hi;
  }
}

// fp8 rows: 32 bytes of one row -> 16 fp16 pairs, exact, in the pairing of deq_int8_f16 (bytes (0, 2), (1, 3)
// of each word): e4m3 through the hardware conversion, e5m2 as the high byte of an fp16.
template <int FMT>
__device__ __forceinline__ void deq_fp8_f16(const uint4 a, const uint4 b, uint32_t (&o)[16]) {
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (FMT == 5) {
      uint32_t d0, d1;
      const uint32_t s0 = prmt(w[i], 0u, 0x0020u), s1 = prmt(w[i], 0u, 0x0031u);
      asm("{\n\t.reg .b16 a;\n\tcvt.u16.u32 a, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, a;\n\t}" : "=r"(d0) : "r"(s0));
      asm("{\n\t.reg .b16 a;\n\tcvt.u16.u32 a, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, a;\n\t}" : "=r"(d1) : "r"(s1));
      o[2 * i] = d0;
      o[2 * i + 1] = d1;
    } else {
      o[2 * i] = prmt(w[i], 0u, 0x2404u);
      o[2 * i + 1] = prmt(w[i], 0u, 0x3414u);
    }
  }
}

// ------------------------------------------------------------------------------------------- the GEMM
// A (the dequantised weights) and B (the activations) both come from shared memory in the 128-byte swizzled
// K-major layout; the fp32 accumulators live in tensor memory, two of them, so the epilogue of one tile
// overlaps the main loop of the next.
__device__ __forceinline__ void tc_mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Epilogue value of one output: fp32 accumulator * token factor * row scale + bias, then stored (accumulated into
// y, or into every rank's output for a column-sharded layer).
template <bool SH>
__device__ __forceinline__ void gemm_store(const GemmParams& p, int64_t tok, int64_t row, float v) {
  if constexpr (SH) {                       // this rank's column of every rank's output
    const uint16_t bb = f32_to_bf16_bits_g(v);
    const int64_t off = tok * p.ldy + p.dst.col0 + row;
    for (int g = 0; g < p.dst.n; ++g) p.dst.y[g][off] = bb;
  } else {
    uint16_t* yp = p.y + tok * p.ldy + row;
    if (p.acc) v += __uint_as_float(static_cast<uint32_t>(*yp) << 16);
    *yp = f32_to_bf16_bits_g(v);
  }
}

template <int FMT>
__device__ __forceinline__ float gemm_row_scale(const GemmParams& p, int64_t rowc) {
  if (FMT == 1) return __half2float(p.s16[rowc]);
  if (FMT >= 5 && FMT <= 9) return reinterpret_cast<const float*>(p.s16)[rowc];   // fp8 / fp6 / fp4: float32 row scales
  return 1.f;
}

// SH: column-sharded outputs (stores into every rank's buffer); a separate instance, so the ordinary
// epilogue carries no extra code
template <int FMT, int BN, bool SH>
__global__ void __launch_bounds__(gemm::THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                const __grid_constant__ CUtensorMap tm_xs, const GemmParams p) {
  using namespace gemm;
  using Cfg = GemmCfg<FMT>;
  using Sm = GemmSmem<BN>;
  constexpr int STAGES = stages(FMT, BN);
  // Narrow token tiles (BN <= 128, six or eight stages) with 4-bit codes: two consecutive k-steps share one set
  // of mbarriers (one wait, arrival and commit per pair of stages: half the hand-offs; their units always hold
  // an even number of k-steps).  [28672, 8192] at M = 64: 112.0 -> 103.5 us, M = 128: 124.8 -> 120.9 us.  With
  // the four stages of BN = 256 the pairs leave too little overlap (configs[2]: 195 -> 231 us), so not there.
  constexpr int GS = ((FMT == 2 || FMT == 9) && BN <= 128 && STAGES % 2 == 0) ? 2 : 1;
  extern __shared__ __align__(1024) uint8_t dyn_smem[];
  // 1024-align the carve-out (SW128 atoms)
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));
  uint8_t* xs = smem;                                          // STAGES x X_STAGE  (TMA, SW128)
  uint8_t* as = xs + STAGES * Sm::X_STAGE;                     // STAGES x A_STAGE  (dequantisers, SW128)
  uint8_t* raw = as + STAGES * A_STAGE;                        // STAGES x RAW_STAGE (TMA)
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw + STAGES * Cfg::RAW_STAGE);
  uint64_t* full_x = bars;                                     // activation tile landed
  uint64_t* full_w = bars + STAGES;                            // code tile landed
  uint64_t* a_full = bars + 2 * STAGES;                        // A tile written
  uint64_t* empty = bars + 3 * STAGES;                         // MMAs done with the slot
  uint64_t* acc_full = bars + 4 * STAGES;                      // [2]
  uint64_t* acc_empty = acc_full + 2;                          // [2]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_x[s], 1);
      mbar_init(&full_w[s], 1);
      mbar_init(&a_full[s], DQ_WARPS);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], EPI_WARPS);
    }
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_w);
    if (p.parts > 1) prefetch_tmap(&tm_xs);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, Sm::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  volatile int* abort_v = abort_flag;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t it = 0;
      for (int u = blockIdx.x; u < p.units; u += gridDim.x) {
        int mb, tok0, width, k0, k1, sp;
        gemm_unit(p, u, BN, mb, tok0, width, k0, k1, sp);
        for (int ks = k0; ks < k1; ++ks, ++it) {
          const uint32_t slot = it % STAGES, bi = slot / GS;
          if (slot % GS == 0) {
            if (it >= STAGES) mbar_wait(&empty[bi], ((it / STAGES) - 1) & 1, abort_v);
            mbar_arrive_expect_tx(&full_x[bi], static_cast<uint32_t>(GS * width) * 128u);
            mbar_arrive_expect_tx(&full_w[bi], GS * Cfg::RAW_STAGE);
          }
          tma_load_2d(xs + slot * Sm::X_STAGE, width == BN ? &tm_x : &tm_xs, ks * BK, tok0, &full_x[bi]);
          tma_load_2d(raw + slot * Cfg::RAW_STAGE, &tm_w, ks * Cfg::RAW_ROW, mb * BM, &full_w[bi]);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t it = 0, tcount = 0;
      for (int u = blockIdx.x; u < p.units; u += gridDim.x, ++tcount) {
        int mb, tok0, width, k0, k1, sp;
        gemm_unit(p, u, BN, mb, tok0, width, k0, k1, sp);
        const uint32_t idesc = idesc_f16_f32(BM, width);
        const uint32_t b = tcount & 1;
        if (tcount >= 2) mbar_wait(&acc_empty[b], ((tcount >> 1) - 1) & 1, abort_v);   // epilogue of tile - 2
        tc_fence_after();
        const uint32_t d_tmem = tmem + b * BN;
        for (int ks = k0; ks < k1; ++ks, ++it) {
          const uint32_t slot = it % STAGES, bi = slot / GS;
          if (slot % GS == 0) {
            const uint32_t ph = (it / STAGES) & 1;
            mbar_wait(&full_x[bi], ph, abort_v);
            mbar_wait(&a_full[bi], ph, abort_v);
            tc_fence_after();
          }
          const uint32_t xaddr = smem_u32(xs + slot * Sm::X_STAGE);
          const uint32_t aaddr = smem_u32(as + slot * A_STAGE);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            tc_mma_ss(d_tmem, smem_desc_sw128(aaddr + kk * 32), smem_desc_sw128(xaddr + kk * 32), idesc,
                      (ks > k0 || kk > 0) ? 1u : 0u);
          if (slot % GS == GS - 1) tc_commit(&empty[bi]);
        }
        tc_commit(&acc_full[b]);
      }
    }
  } else if (warp < 2 + DQ_WARPS) {
    // ------------------------------------------------------------------ dequantise into shared memory
    const int d = threadIdx.x - 64;         // 0..255
    const int rloc = d & (BM - 1);          // row within the tile
    const int h = d >> 7;                   // K half of each stage (32 values = 64 bytes of fp16)
    const uint32_t arow = static_cast<uint32_t>((rloc >> 3) * 1024 + (rloc & 7) * 128);
    uint32_t it = 0;
    for (int u = blockIdx.x; u < p.units; u += gridDim.x) {
      int mb, tok0, width, k0, k1, sp;
      gemm_unit(p, u, BN, mb, tok0, width, k0, k1, sp);
      const int64_t row = static_cast<int64_t>(mb) * BM + rloc;
      const int64_t rowc = row < p.N ? row : p.N - 1;
      // int4 scales of this row, one group of 128 per two stages, fetched four groups ahead through a small
      // register queue so their latency does not stall a stage (k0 is even: a split starts on a group)
      static_assert(BK * 2 == 128, "two stages per scale group");
      const int ng = static_cast<int>(p.K / 128);
      const int g0 = k0 >> 1;
      const unsigned short* srow = reinterpret_cast<const unsigned short*>(p.s16) + rowc * ng;
      unsigned short sq0 = 0, sq1 = 0, sq2 = 0, sq3 = 0;
      if (FMT == 2) {
        sq0 = __ldg(srow + g0);
        if (g0 + 1 < ng) sq1 = __ldg(srow + g0 + 1);
        if (g0 + 2 < ng) sq2 = __ldg(srow + g0 + 2);
        if (g0 + 3 < ng) sq3 = __ldg(srow + g0 + 3);
      }
      uint32_t s2 = 0;
      // unrolled by 8 k-steps (four scale groups): the queue's moves become register renames, so each scale
      // load has four groups to land ([28672, 8192] at M = 64: 116.7 -> 111.4 us, the same bits)
#pragma unroll 8
      for (int ks = k0; ks < k1; ++ks, ++it) {
        const uint32_t slot = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (FMT == 2 && (ks & 1) == 0) {
          const int gi = ks >> 1;
          s2 = static_cast<uint32_t>(sq0) * 0x00010001u;
          sq0 = sq1; sq1 = sq2; sq2 = sq3;
          if (gi + 4 < ng) sq3 = __ldg(srow + gi + 4);
        }
        const uint32_t bi = slot / GS;
        if (slot % GS == 0) {
          mbar_wait(&full_w[bi], ph, abort_v);
          if (it >= STAGES) mbar_wait(&empty[bi], ((it / STAGES) - 1) & 1, abort_v);   // MMA done with A
        }
        uint32_t o[16];
        const uint32_t rbase = smem_u32(raw + slot * Cfg::RAW_STAGE) + rloc * Cfg::RAW_ROW;
        if (FMT == 2 || FMT == 9) {
          // SWIZZLE_32B: 16-byte chunk index ^= bit 7 of the offset (row >> 2)
          const uint4 r = lds_v4(rbase + 16 * (h ^ ((rloc >> 2) & 1)));
          if (FMT == 2) deq_int4_f16(r, s2, o);
          else deq_fp4_f16(r, o);
        } else if (FMT == 7 || FMT == 8) {
          // unswizzled 48-byte rows: this half's 24 bytes as three 8-byte words
          uint32_t w[6];
#pragma unroll
          for (int j = 0; j < 3; ++j) {
            uint32_t a, b;
            asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(a), "=r"(b) : "r"(rbase + 24 * h + 8 * j));
            w[2 * j] = a;
            w[2 * j + 1] = b;
          }
          deq_fp6_f16<FMT>(w, o);
        } else {
          // SWIZZLE_64B: chunk index (0..3) ^= bits 7..8 of the offset (row >> 1)
          const int sw = (rloc >> 1) & 3;
          const uint4 a = lds_v4(rbase + 16 * ((2 * h) ^ sw));
          const uint4 b = lds_v4(rbase + 16 * ((2 * h + 1) ^ sw));
          if (FMT == 1) deq_int8_f16(a, b, o);
          else deq_fp8_f16<FMT>(a, b, o);
        }
        // row rloc, 16-byte chunks 4h .. 4h+3 of its 128-byte K row, 128-byte swizzle: chunk ^= row % 8
        const uint32_t abase = smem_u32(as + slot * A_STAGE) + arow;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t c = static_cast<uint32_t>((4 * h + j) ^ (rloc & 7));
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(abase + c * 16), "r"(o[4 * j]),
                       "r"(o[4 * j + 1]), "r"(o[4 * j + 2]), "r"(o[4 * j + 3])
                       : "memory");
        }
        if (slot % GS == GS - 1) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // visible to the tensor cores
          __syncwarp();
          if (lane == 0) mbar_arrive(&a_full[bi]);
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue: TMEM -> bf16 outputs
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    const int rloc = q * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    uint32_t tcount = 0;
    for (int u = blockIdx.x; u < p.units; u += gridDim.x, ++tcount) {
      int mb, tok0, width, k0, k1, sp;
      gemm_unit(p, u, BN, mb, tok0, width, k0, k1, sp);
      const int64_t row = static_cast<int64_t>(mb) * BM + rloc;
      const int64_t rowc = row < p.N ? row : p.N - 1;
      const uint32_t b = tcount & 1;
      mbar_wait(&acc_full[b], (tcount >> 1) & 1, abort_v);
      tc_fence_after();
      const float rs = gemm_row_scale<FMT>(p, rowc);
      const float bias = p.bias ? __uint_as_float(static_cast<uint32_t>(p.bias[rowc]) << 16) : 0.f;
      const bool row_ok = row < p.N;
      if (p.splits > 1) {                   // this split's float32 accumulators; the reduction does the rest
        float* dst = p.part + static_cast<int64_t>(sp) * p.M * p.N + row;
#pragma unroll 1
        for (int c0 = 0; c0 < width; c0 += 16) {
          uint32_t dv[16];
          tmem_ld_x16(tmem + lane_addr + b * BN + c0, dv);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int64_t tok = static_cast<int64_t>(tok0) + c0 + j;
            if (row_ok && tok < p.M) dst[tok * p.N] = __uint_as_float(dv[j]);
          }
        }
      } else {
#pragma unroll 1
        for (int c0 = 0; c0 < width; c0 += 16) {
          uint32_t dv[16];
          tmem_ld_x16(tmem + lane_addr + b * BN + c0, dv);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int64_t tok = static_cast<int64_t>(tok0) + c0 + j;
            if (row_ok && tok < p.M)
              gemm_store<SH>(p, tok, row, __uint_as_float(dv[j]) * (p.tokscale[tok] * rs) + bias);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Sm::TMEM_COLS);
  }
}

// The K splits of a tile added in split order, then the epilogue of gemm_kernel: one thread per output.
template <int FMT, bool SH>
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const GemmParams p) {
  const int64_t total = p.M * p.N;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t tok = i / p.N, row = i - tok * p.N;
    float v = p.part[i];
    for (int s = 1; s < p.splits; ++s) v += p.part[s * total + i];
    const float rs = gemm_row_scale<FMT>(p, row);
    const float bias = p.bias ? __uint_as_float(static_cast<uint32_t>(p.bias[row]) << 16) : 0.f;
    gemm_store<SH>(p, tok, row, v * (p.tokscale[tok] * rs) + bias);
  }
}

// ------------------------------------------------------------------------------------------- host side
static int gemm_bn_for(int64_t M) { return M <= 64 ? 64 : (M <= 128 ? 128 : 256); }

size_t gemm_smem_bytes(int fmt, int bn) {
  return 1024 + static_cast<size_t>(gemm::stages(fmt, bn)) * (bn * 128 + gemm::A_STAGE + gemm::raw_bytes(fmt)) +
         gemm::TAIL;
}

// Workspace layout: fp16 activations [M, K] | per-token factors [M] | (K splits) float32 accumulators
// [splits][M][N], each part 256-byte aligned.
static size_t ws_front_bytes(int64_t M, int64_t K) {
  size_t x16 = static_cast<size_t>(M * K) * 2;
  x16 = (x16 + 255) & ~static_cast<size_t>(255);
  return x16 + ((static_cast<size_t>(M) * sizeof(float) + 255) & ~static_cast<size_t>(255));
}

size_t gemm_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  const int splits = gemm_splits(M, K);
  const size_t part = splits > 1 ? static_cast<size_t>(splits) * M * N * sizeof(float) : 0;
  return ws_front_bytes(M, K) + part + 256;
}

template <int FMT, int BN, bool SH>
static cudaError_t launch_gemm_t(const CUtensorMap& tx, const CUtensorMap& tw, const CUtensorMap& txs,
                                 const GemmParams& p, int sms, cudaStream_t st) {
  const size_t smem = gemm_smem_bytes(FMT, BN);
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel<FMT, BN, SH>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  const int grid = p.units < sms ? p.units : sms;
  gemm_kernel<FMT, BN, SH><<<grid, gemm::THREADS, smem, st>>>(tx, tw, txs, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || p.splits == 1) return e;
  const int64_t total = p.M * p.N;
  int64_t blocks = (total + 255) / 256;
  if (blocks > static_cast<int64_t>(sms) * 8) blocks = static_cast<int64_t>(sms) * 8;
  splitk_reduce_kernel<FMT, SH><<<static_cast<unsigned>(blocks), 256, 0, st>>>(p);
  return cudaGetLastError();
}

// the instance for a format: token tile, sharded outputs
template <int FMT>
static cudaError_t launch_gemm_f(int bn, bool sh, const CUtensorMap& tx, const CUtensorMap& tw,
                                 const CUtensorMap& txs, const GemmParams& p, int sms, cudaStream_t st) {
  if (bn == 64) return sh ? launch_gemm_t<FMT, 64, true>(tx, tw, txs, p, sms, st)
                          : launch_gemm_t<FMT, 64, false>(tx, tw, txs, p, sms, st);
  if (bn == 128) return sh ? launch_gemm_t<FMT, 128, true>(tx, tw, txs, p, sms, st)
                           : launch_gemm_t<FMT, 128, false>(tx, tw, txs, p, sms, st);
  return sh ? launch_gemm_t<FMT, 256, true>(tx, tw, txs, p, sms, st)
            : launch_gemm_t<FMT, 256, false>(tx, tw, txs, p, sms, st);
}

cudaError_t launch_gemm(int fmt, const void* x, int64_t M, int64_t K, const void* codes, const void* scales,
                        int64_t N, const void* bias, int acc, void* y, int64_t ldy, void* ws, int sms,
                        cudaStream_t st, const char** why, const OutRanks* dst) {
  PFN_encodeTiled enc = get_encode();
  if (!enc) {
    *why = "cuTensorMapEncodeTiled is not available from the driver";
    return cudaErrorNotSupported;
  }
  // workspace: permuted fp16 activations + per-token factors (+ K-split accumulators)
  size_t x16b = static_cast<size_t>(M * K) * 2;
  x16b = (x16b + 255) & ~static_cast<size_t>(255);
  uint16_t* x16 = reinterpret_cast<uint16_t*>(ws);
  float* tokscale = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + x16b);
  float* part = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + ws_front_bytes(M, K));
  {
    const uint16_t* xb = reinterpret_cast<const uint16_t*>(x);
    if (fmt == 2) launch_prep_x<0>(xb, M, K, x16, tokscale, st);
    else if (fmt == 9 || fmt == 7 || fmt == 8) launch_prep_x<2>(xb, M, K, x16, tokscale, st);   // natural K order
    else launch_prep_x<1>(xb, M, K, x16, tokscale, st);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  const int BN = gemm_bn_for(M);
  CUtensorMap tx, tw, txs;
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(K * 2)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(gemm::BK), static_cast<cuuint32_t>(BN)};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, x16, dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      *why = "cuTensorMapEncodeTiled failed for the activation tensor";
      return cudaErrorInvalidValue;
    }
  }
  {
    const bool nib = (fmt == 2 || fmt == 9);          // 4-bit codes
    const bool six = (fmt == 7 || fmt == 8);          // 6-bit codes, four per three bytes
    const int64_t row_bytes = nib ? K / 2 : (six ? K / 4 * 3 : K);
    const cuuint32_t raw_row = static_cast<cuuint32_t>(gemm::raw_row(fmt));
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(N)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
    cuuint32_t box[2] = {raw_row, static_cast<cuuint32_t>(gemm::BM)};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(codes), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE,
                     nib ? CU_TENSOR_MAP_SWIZZLE_32B : (six ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_64B),
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      *why = "cuTensorMapEncodeTiled failed for the weight codes";
      return cudaErrorInvalidValue;
    }
  }
  GemmParams p;
  p.s16 = reinterpret_cast<const __half*>(scales);
  p.bias = reinterpret_cast<const uint16_t*>(bias);
  p.y = reinterpret_cast<uint16_t*>(y);
  p.tokscale = tokscale;
  p.M = M; p.N = N; p.K = K; p.ldy = ldy;
  p.acc = acc;
  p.m_blocks = static_cast<int>((N + gemm::BM - 1) / gemm::BM);
  p.n_blocks = static_cast<int>((M + BN - 1) / BN);
  p.tiles = p.m_blocks * p.n_blocks;
  p.ksteps = static_cast<int>(K / gemm::BK);
  // a last wave under half full: cut its tiles along the tokens so every SM ends at about the same time
  p.units = p.tiles;
  p.full = p.tiles;
  p.parts = 1;
  p.sbn = BN;
  p.splits = gemm_splits(M, K);
  p.kper = p.ksteps;
  p.part = part;
  if (p.splits > 1) {                 // equal, even k-step counts; no split left empty
    p.kper = (p.ksteps + p.splits - 1) / p.splits;
    p.kper += p.kper & 1;
    p.splits = (p.ksteps + p.kper - 1) / p.kper;
  }
  if (p.splits > 1) {
    p.units = p.tiles * p.splits;
  } else {
    const int rem = p.tiles % sms;
    if (BN >= 128 && p.tiles > sms && rem > 0 && rem * 2 <= sms) {
      int parts = BN / 64;
      while (parts > 1 && rem * parts > sms) parts >>= 1;
      if (parts > 1) {
        p.full = p.tiles - rem;
        p.parts = parts;
        p.sbn = BN / parts;
        p.units = p.full + rem * parts;
      }
    }
  }
  memcpy(&txs, &tx, sizeof(tx));
  if (p.parts > 1) {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(K * 2)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(gemm::BK), static_cast<cuuint32_t>(p.sbn)};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(&txs, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, x16, dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      *why = "cuTensorMapEncodeTiled failed for the activation tensor (last-wave box)";
      return cudaErrorInvalidValue;
    }
  }
  p.dst = dst ? *dst : OutRanks{};
  switch (fmt) {
    case 2: return launch_gemm_f<2>(BN, p.dst.n != 0, tx, tw, txs, p, sms, st);
    case 9: return launch_gemm_f<9>(BN, p.dst.n != 0, tx, tw, txs, p, sms, st);
    case 5: return launch_gemm_f<5>(BN, p.dst.n != 0, tx, tw, txs, p, sms, st);
    case 6: return launch_gemm_f<6>(BN, p.dst.n != 0, tx, tw, txs, p, sms, st);
    case 7: return launch_gemm_f<7>(BN, p.dst.n != 0, tx, tw, txs, p, sms, st);
    case 8: return launch_gemm_f<8>(BN, p.dst.n != 0, tx, tw, txs, p, sms, st);
    default: return launch_gemm_f<1>(BN, p.dst.n != 0, tx, tw, txs, p, sms, st);
  }
}

}  // namespace lb

// Decode-regime product (M <= 16 tokens): y[M, N] = x[M, K] . deq(W)[N, K]^T.
//
// The weight stream is the cost: every byte of codes is read once from HBM.  One CTA owns a block of 16
// output rows and one K split.  A producer warp streams the block's rows through a 4-stage shared-memory
// ring with TMA bulk copies (cp.async.bulk, completion on mbarriers); eight consumer warps each take one
// 64-byte unit per row per stage (int4: 128 values = one scale group; int8: 64 values).
//
// Dequantisation happens in registers and keeps the integer codes EXACT: a LOP3 places each code (offset by
// 8 through an XOR folded into the same LOP3) in the mantissa of a bfloat16 with exponent 2^7, one packed
// subtraction removes the offset.  The exact codes and the bfloat16 activations go through m16n8k16 tensor-
// core products with float32 accumulation; the float scale of each 128-value group is applied to the
// group's float32 partial sum (int8: the row scale to the final sum).  So the only rounding besides float32
// accumulation is the final bfloat16 store.  K positions inside a thread's 32 values are permuted to match
// the nibble pairs the LOP3 produces; the activations are permuted identically with PRMT.
//
// Sums are deterministic and depend only on K: per warp in stage order, then warps 0..7, then K splits
// 0..n-1 of fixed size (the CTAs of one row block form a thread-block cluster and the split partials are
// added in rank order through distributed shared memory), so a column-sharded layer gives bit-identical
// outputs to the unsharded one, and the kernel needs no global scratch memory.
#include "lb_common.cuh"
#include "lb_kernels.h"

namespace lb {

namespace gemv {
constexpr int RB = 16;                 // rows per CTA (one m16 tile)
constexpr int UNIT = 64;               // bytes of one row per warp per stage
constexpr int WARPS = 8;               // consumer warps
constexpr int STAGE_ROW = UNIT * WARPS;         // 512 bytes of a row per stage
constexpr int ROW_STRIDE = STAGE_ROW + 64;      // padded so rows g and g+8 fall in different banks
constexpr int STAGES = 4;
constexpr int STAGE_BYTES = RB * ROW_STRIDE;
}  // namespace gemv

struct GemvParams {
  const uint16_t* x;      // bf16 [M, K]
  const uint8_t* w;       // codes
  const __half* s16;      // scales
  const uint16_t* bias;   // bf16 [N] or null
  uint16_t* y;            // bf16 [M, ldy]
  int64_t N, K, ldy;
  int M, acc, nsplit, units_per_split, total_units;
};

// bf16 pair (136 + q_lo, 136 + q_hi) from the nibbles at bits 0-3 and 16-19 of v, then the exact codes.
__device__ __forceinline__ uint32_t deq4_pair(uint32_t v) {
  return bf2_sub(lop3_and_xor_or(v, 0x000F000Fu, 0x43084308u), 0x43084308u);
}
// Exact signed bytes 0 and 2 of v as a bf16 pair: low nibble unsigned, high nibble signed, q = 16*hi + lo.
__device__ __forceinline__ uint32_t deq8_pair(uint32_t v) {
  const uint32_t lo = lop3_and_or(v, 0x000F000Fu, 0x43004300u);           // 128 + lo
  const uint32_t hi = lop3_and_xor_or(v >> 4, 0x000F000Fu, 0x43084308u);  // 136 + hi
  const uint32_t t = bf2_sub(hi, 0x43084308u);                             // hi
  const uint32_t u = bf2_fma(t, 0x41804180u, lo);                          // 16 hi + 128 + lo, in [0, 255]
  return bf2_sub(u, 0x43004300u);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}

template <int FMT>
__device__ __forceinline__ void finish_output(const GemvParams& p, int64_t row0, int orow, int otok, float sum) {
  const int64_t n = row0 + orow;
  if (otok >= p.M || n >= p.N) return;
  if (FMT == 1) sum *= __half2float(p.s16[n]);
  if (p.bias) sum += bf16_bits_to_f32(p.bias[n]);
  uint16_t* yp = p.y + static_cast<int64_t>(otok) * p.ldy + n;
  if (p.acc) sum += bf16_bits_to_f32(*yp);
  *yp = f32_to_bf16_bits(sum);
}

template <int FMT, int MT>
__global__ void __launch_bounds__(288) gemv_kernel(const GemvParams p) {
  using namespace gemv;
  __shared__ __align__(128) uint8_t ring[STAGES * STAGE_BYTES];
  __shared__ __align__(16) float red[WARPS * 32 * 4 * MT];
  __shared__ __align__(16) float csum[256];
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * RB;
  const int split = blockIdx.y;
  const int unit_begin = split * p.units_per_split;
  const int unit_end = min(unit_begin + p.units_per_split, p.total_units);
  const int nstages = (unit_end - unit_begin + WARPS - 1) / WARPS;
  const int64_t row_bytes = (FMT == 2) ? p.K / 2 : p.K;
  const int rows_valid = static_cast<int>((p.N - row0) < RB ? (p.N - row0) : RB);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], WARPS);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  float final_sum = 0.f;
  if (warp == WARPS) {
    // ------------------------------------------------------------------ producer (TMA bulk copies)
    for (int st = 0; st < nstages; ++st) {
      const int slot = st % STAGES;
      if (st >= STAGES) mbar_wait(&empty_bar[slot], ((st / STAGES) - 1) & 1, &abort_flag);
      const int u0 = unit_begin + st * WARPS;
      const int su = min(unit_end - u0, WARPS);
      const uint32_t bytes_row = static_cast<uint32_t>(su * UNIT);
      if (lane == 0) mbar_arrive_expect_tx(&full_bar[slot], bytes_row * rows_valid);
      __syncwarp();
      if (lane < rows_valid) {
        const uint8_t* src = p.w + (row0 + lane) * row_bytes + static_cast<int64_t>(u0) * UNIT;
        bulk_g2s(ring + slot * STAGE_BYTES + lane * ROW_STRIDE, src, bytes_row, &full_bar[slot]);
      }
    }
  } else {
    // ------------------------------------------------------------------ consumers
    const int g = lane >> 2;     // row (and token) within the m16n8 tile
    const int c = lane & 3;      // which 32 (int4) / 16 (int8) values of the unit
    const int64_t rg = row0 + g < p.N ? row0 + g : p.N - 1;
    const int64_t rg8 = row0 + g + 8 < p.N ? row0 + g + 8 : p.N - 1;
    float tot[MT][4];
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
      for (int i = 0; i < 4; ++i) tot[t][i] = 0.f;

    for (int st = 0; st < nstages; ++st) {
      const int slot = st % STAGES;
      const int unit = unit_begin + st * WARPS + warp;
      const bool active = unit < unit_end;
      // activations of this unit (L2-resident), issued before the wait so they overlap it
      constexpr int XW = (FMT == 2) ? 16 : 8;  // 32-bit words of x per thread per token tile
      uint32_t X[MT][XW];
      float sg = 0.f, sg8 = 0.f;
#pragma unroll
      for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int v = 0; v < XW; ++v) X[t][v] = 0u;
      if (active) {
        const int64_t kbase = (FMT == 2) ? static_cast<int64_t>(unit) * 128 + 32 * c
                                         : static_cast<int64_t>(unit) * 64 + 16 * c;
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const int tok = t * 8 + g;
          if (tok < p.M) {
            const uint16_t* xp = p.x + static_cast<int64_t>(tok) * p.K + kbase;
#pragma unroll
            for (int v = 0; v < XW / 4; ++v) {
              const uint4 q = ldg_nc_v4(xp + 8 * v);
              X[t][4 * v] = q.x; X[t][4 * v + 1] = q.y; X[t][4 * v + 2] = q.z; X[t][4 * v + 3] = q.w;
            }
          }
        }
        if (FMT == 2) {
          const int64_t ng = p.K / 128;
          sg = __half2float(p.s16[rg * ng + unit]);
          sg8 = __half2float(p.s16[rg8 * ng + unit]);
        }
      }
      mbar_wait(&full_bar[slot], (st / STAGES) & 1, &abort_flag);
      uint32_t Wg[4] = {0u, 0u, 0u, 0u}, Wg8[4] = {0u, 0u, 0u, 0u};
      if (active) {
        const uint32_t base = smem_u32(ring + slot * STAGE_BYTES) + warp * UNIT + c * 16;
        const uint4 a = lds_v4(base + g * ROW_STRIDE);
        const uint4 b = lds_v4(base + (g + 8) * ROW_STRIDE);
        Wg[0] = a.x; Wg[1] = a.y; Wg[2] = a.z; Wg[3] = a.w;
        Wg8[0] = b.x; Wg8[1] = b.y; Wg8[2] = b.z; Wg8[3] = b.w;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[slot]);
      if (!active) continue;

      if (FMT == 2) {
        float cg[MT][4];
#pragma unroll
        for (int t = 0; t < MT; ++t)
#pragma unroll
          for (int i = 0; i < 4; ++i) cg[t][i] = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int i = j >> 1;
          const int sh = 8 * (j & 1);
          uint32_t a[4];
          a[0] = deq4_pair(Wg[i] >> sh);         // row g,   logical k 2c, 2c+1  <- nibbles sh/4, sh/4+4
          a[1] = deq4_pair(Wg8[i] >> sh);        // row g+8
          a[2] = deq4_pair(Wg[i] >> (sh + 4));   // row g,   logical k 2c+8, 2c+9 <- nibbles sh/4+1, sh/4+5
          a[3] = deq4_pair(Wg8[i] >> (sh + 4));  // row g+8
          const int xp = 4 * i + (j & 1);
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            uint32_t b[2];
            b[0] = prmt(X[t][xp], X[t][xp + 2], 0x5410u);
            b[1] = prmt(X[t][xp], X[t][xp + 2], 0x7632u);
            mma_bf16_16816(cg[t], a, b, cg[t]);
          }
        }
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          tot[t][0] = fmaf(cg[t][0], sg, tot[t][0]);
          tot[t][1] = fmaf(cg[t][1], sg, tot[t][1]);
          tot[t][2] = fmaf(cg[t][2], sg8, tot[t][2]);
          tot[t][3] = fmaf(cg[t][3], sg8, tot[t][3]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t a[4];
          a[0] = deq8_pair(Wg[j]);          // row g,   bytes 0, 2 of word j
          a[1] = deq8_pair(Wg8[j]);
          a[2] = deq8_pair(Wg[j] >> 8);     // row g,   bytes 1, 3
          a[3] = deq8_pair(Wg8[j] >> 8);
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            uint32_t b[2];
            b[0] = prmt(X[t][2 * j], X[t][2 * j + 1], 0x5410u);
            b[1] = prmt(X[t][2 * j], X[t][2 * j + 1], 0x7632u);
            mma_bf16_16816(tot[t], a, b, tot[t]);
          }
        }
      }
    }

    // ---------------------------------------------------------------- reduce the 8 warps in fixed order
    {
      float* r = red + (warp * 32 + lane) * 4 * MT;
#pragma unroll
      for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int i = 0; i < 4; ++i) r[4 * t + i] = tot[t][i];
    }
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const int tid = threadIdx.x;       // 0..255: output (row tid % 16, token tid / 16)
    const int orow = tid & 15;
    const int otok = tid >> 4;
    if (otok < p.M) {
      const int tt = otok >> 3, tk = otok & 7;
      const int src_lane = (orow & 7) * 4 + (tk >> 1);
      const int reg = tt * 4 + (orow >> 3) * 2 + (tk & 1);
#pragma unroll
      for (int w = 0; w < WARPS; ++w) final_sum += red[(w * 32 + src_lane) * 4 * MT + reg];
    }
    csum[tid] = final_sum;
  }

  if (p.nsplit > 1) {
    // ------------------------------------------------------------------ reduce the K splits of the cluster
    // The CTAs of one row block form a cluster (rank = split).  Rank 0 reads every rank's partials through
    // distributed shared memory in rank order; the second cluster barrier keeps the other CTAs (and their
    // shared memory) alive until it has.
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (split == 0 && threadIdx.x < 256) {
      float sum = 0.f;
      const uint32_t local = smem_u32(&csum[threadIdx.x]);
      for (int r = 0; r < p.nsplit; ++r) {
        uint32_t remote;
        float v;
        asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(r));
        asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
        sum += v;
      }
      finish_output<FMT>(p, row0, threadIdx.x & 15, threadIdx.x >> 4, sum);
    }
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  } else if (threadIdx.x < 256) {
    finish_output<FMT>(p, row0, threadIdx.x & 15, threadIdx.x >> 4, final_sum);
  }
}

// ------------------------------------------------------------------------------------------- launcher
// K split size is fixed (64 units = 4096 bytes of a row), so results never depend on N or on sharding.
constexpr int kUnitsPerSplit = 64;
constexpr int kMaxSplits = 8;  // portable cluster size

int gemv_max_k(int fmt) { return kMaxSplits * kUnitsPerSplit * gemv::UNIT * (fmt == 2 ? 2 : 1); }

template <int FMT, int MT>
static cudaError_t launch_gemv_t(const GemvParams& p, int64_t nblk, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(nblk), static_cast<unsigned>(p.nsplit), 1);
  cfg.blockDim = dim3(288, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = static_cast<unsigned>(p.nsplit);
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = p.nsplit > 1 ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_kernel<FMT, MT>, p);
}

cudaError_t launch_gemv(int fmt, const void* x, int64_t M, int64_t K, const void* codes, const void* scales,
                        int64_t N, const void* bias, int acc, void* y, int64_t ldy, cudaStream_t st) {
  GemvParams p;
  p.x = reinterpret_cast<const uint16_t*>(x);
  p.w = reinterpret_cast<const uint8_t*>(codes);
  p.s16 = reinterpret_cast<const __half*>(scales);
  p.bias = reinterpret_cast<const uint16_t*>(bias);
  p.y = reinterpret_cast<uint16_t*>(y);
  p.N = N; p.K = K; p.ldy = ldy;
  p.M = static_cast<int>(M);
  p.acc = acc;
  const int64_t row_bytes = (fmt == 2) ? K / 2 : K;
  p.total_units = static_cast<int>(row_bytes / gemv::UNIT);
  p.units_per_split = kUnitsPerSplit;
  p.nsplit = (p.total_units + kUnitsPerSplit - 1) / kUnitsPerSplit;
  const int64_t nblk = (N + gemv::RB - 1) / gemv::RB;
  if (fmt == 2) return M <= 8 ? launch_gemv_t<2, 1>(p, nblk, st) : launch_gemv_t<2, 2>(p, nblk, st);
  return M <= 8 ? launch_gemv_t<1, 1>(p, nblk, st) : launch_gemv_t<1, 2>(p, nblk, st);
}

}  // namespace lb

// Decode-regime product (M <= 16 tokens): y[M, N] = x[M, K] . deq(W)[N, K]^T.
//
// The weight stream is the cost: every byte of codes is read once from HBM.  Work is cut in row blocks of
// 16 output rows.  A producer warp streams a CTA's row blocks through a deep shared-memory ring with TMA
// bulk copies (cp.async.bulk, completion on mbarriers), one copy per row per stage; eight consumer warps
// each take two 64-byte units per row per stage (int4: 128 values = one scale group; int8: 64 values).
//
// Activations are converted once per CTA into shared memory as fp16, already in the order of the tensor-
// core B fragments, with a power-of-two factor per (token, K range) so the bf16 -> fp16 conversion is exact.
// Codes are dequantised in registers and kept EXACT: one LOP3 places a code (offset by 8 through an XOR
// folded into the same LOP3) in the mantissa of 1024 in fp16, one packed FMA removes the offset.  The exact
// codes and activations go through m16n8k16 tensor-core products with float32 accumulation; the fp16 scale
// of each 128-value group multiplies the group's float32 partial (int8: the row scale multiplies the final
// sum).  The only rounding besides float32 accumulation is the final bfloat16 store.
//
// Sums have a fixed structure that depends only on K: the codes of a row are cut in K ranges of 2 KB
// (32 units); within a range each warp adds its units in order, the eight warps are added in order, and the
// ranges are added in order.  Large-N calls run persistent CTAs (one per SM) that walk whole row blocks;
// small-N calls give each K range its own CTA in a thread-block cluster and add the ranges in rank order
// through distributed shared memory.  Both produce identical bits, so a column-sharded layer matches the
// unsharded one exactly.  No global scratch memory is used.
#include "lb_common.cuh"
#include "lb_kernels.h"

namespace lb {

namespace gemv {
constexpr int RB = 16;                          // rows per row block (one m16 tile)
constexpr int UNIT = 64;                        // bytes of one row per unit
constexpr int WARPS = 8;                        // consumer warps
constexpr int STAGE_UNITS = 16;                 // units per stage (two per warp)
constexpr int STAGE_ROW = UNIT * STAGE_UNITS;   // 1024 bytes of a row per stage
constexpr int ROW_STRIDE = STAGE_ROW + 64;      // rows g and g+8 in different banks
constexpr int STAGE_BYTES = RB * ROW_STRIDE;    // 17408
constexpr int RANGE_UNITS = 32;                 // units per K range (2 KB of codes per row)
constexpr int MAX_RANGES = 32;
constexpr int MAX_CLUSTER = 8;
constexpr int SMEM_LIMIT = 227 * 1024;
constexpr int MIN_SLOTS = 3, MAX_SLOTS = 12;
}  // namespace gemv

struct GemvParams {
  const uint16_t* x;      // bf16 [M, K]
  const uint8_t* w;       // codes
  const __half* s16;      // scales
  const uint16_t* bias;   // bf16 [N] or null
  uint16_t* y;            // bf16 [M, ldy]
  int64_t N, K, ldy;
  int M, acc;
  int total_units;        // units per row
  int nblocks;            // row blocks
  int nranges;            // K ranges per row
  int slots;              // ring slots
  int xs_units;           // units of x staged (cluster: one range; persistent: all)
  int cluster;            // 1: grid (nblocks, nranges), one range per CTA
};

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}

// m16n8k16 fp16 tensor-core product, fp32 accumulate: d += a * b.
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// int4: one word (8 codes, two's complement nibbles) -> four fp16 pairs of exact codes:
// P0 = (n0, n4), P1 = (n1, n5), P2 = (n2, n6), P3 = (n3, n7).
__device__ __forceinline__ void deq4_word(uint32_t w, uint32_t (&P)[4]) {
  const uint32_t w8 = w >> 8;
  P[0] = h2_fma(lop3_and_xor_or(w, 0x000F000Fu, 0x64086408u), 0x3C003C00u, 0xE408E408u);   // (1032+q) - 1032
  P[1] = h2_fma(lop3_and_xor_or(w, 0x00F000F0u, 0x64806480u), 0x2C002C00u, 0xD480D480u);   // (1024+16(q+8))/16 - 72
  P[2] = h2_fma(lop3_and_xor_or(w8, 0x000F000Fu, 0x64086408u), 0x3C003C00u, 0xE408E408u);
  P[3] = h2_fma(lop3_and_xor_or(w8, 0x00F000F0u, 0x64806480u), 0x2C002C00u, 0xD480D480u);
}
// int8: one word (4 codes) -> two fp16 pairs of exact codes: (b0, b2), (b1, b3).
__device__ __forceinline__ void deq8_word(uint32_t w, uint32_t& q02, uint32_t& q13) {
  const uint32_t v = w ^ 0x80808080u;                                        // q + 128
  q02 = h2_fma(prmt(v, 0x00006464u, 0x5240u), 0x3C003C00u, 0xE480E480u);     // (1024 + n) - 1152
  q13 = h2_fma(prmt(v, 0x00006464u, 0x5341u), 0x3C003C00u, 0xE480E480u);
}

// Shared-memory carve-up, in bytes from the (1024-aligned) base.
struct GemvSmem {
  int ring, xs, xsc, red, csum, bars, total;
  int token_stride;   // bytes of one token's staged activations
};

__host__ __device__ inline GemvSmem gemv_smem(int fmt, int M, int xs_units, int slots) {
  using namespace gemv;
  GemvSmem s;
  const int xu = (fmt == 2) ? 256 : 128;     // staged bytes of x per unit per token
  s.token_stride = xs_units * xu + 64;
  s.ring = 0;
  s.xs = slots * STAGE_BYTES;
  s.xsc = s.xs + ((M * s.token_stride + 127) & ~127);
  s.red = s.xsc + 2 * 16 * MAX_RANGES * 4;
  s.csum = s.red + 2 * WARPS * 32 * 8 * 4;
  s.bars = s.csum + 256 * 4;
  s.total = s.bars + 2 * MAX_SLOTS * 8 + 64;
  return s;
}

template <int FMT, int MT>
__global__ void __launch_bounds__(288, 1) gemv_kernel(const GemvParams p) {
  using namespace gemv;
  extern __shared__ __align__(1024) uint8_t dyn_smem[];
  const GemvSmem L = gemv_smem(FMT, p.M, p.xs_units, p.slots);
  uint8_t* ring = dyn_smem + L.ring;
  uint8_t* xs = dyn_smem + L.xs;
  float* xsc = reinterpret_cast<float*>(dyn_smem + L.xsc);     // [16 tokens][MAX_RANGES] 2^e factors
  int* xmax = reinterpret_cast<int*>(xsc + 16 * MAX_RANGES);   // [16 tokens][MAX_RANGES] absmax bits
  float* red = reinterpret_cast<float*>(dyn_smem + L.red);     // [2][WARPS][32][8]
  float* csum = reinterpret_cast<float*>(dyn_smem + L.csum);   // [256]
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(dyn_smem + L.bars);
  uint64_t* empty_bar = full_bar + MAX_SLOTS;
  int* abort_flag = reinterpret_cast<int*>(empty_bar + MAX_SLOTS);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t row_bytes = (FMT == 2) ? p.K / 2 : p.K;
  // this CTA's work: row blocks b0, b0 + bstep, ...; units [u_begin, u_end) of each row
  int b0, bstep, u_begin, u_end;
  if (p.cluster) {
    b0 = blockIdx.x; bstep = p.nblocks;
    u_begin = blockIdx.y * RANGE_UNITS;
    u_end = min(u_begin + RANGE_UNITS, p.total_units);
  } else {
    b0 = blockIdx.x; bstep = gridDim.x;
    u_begin = 0; u_end = p.total_units;
  }
  const int nst = (u_end - u_begin + STAGE_UNITS - 1) / STAGE_UNITS;   // stages per row block
  const int slots = p.slots;

  if (threadIdx.x == 0) {
    for (int s = 0; s < slots; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], WARPS);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  volatile int* abort_v = abort_flag;

  if (warp == WARPS) {
    // ------------------------------------------------------------------ producer: TMA bulk copies
    uint32_t it = 0;
    for (int b = b0; b < p.nblocks; b += bstep) {
      const int64_t row0 = static_cast<int64_t>(b) * RB;
      const int rows_valid = static_cast<int>((p.N - row0 < RB ? p.N - row0 : RB));
      for (int st = 0; st < nst; ++st, ++it) {
        const uint32_t slot = it % slots;
        if (it >= static_cast<uint32_t>(slots)) mbar_wait(&empty_bar[slot], ((it / slots) - 1) & 1, abort_v);
        const int u0 = u_begin + st * STAGE_UNITS;
        const uint32_t bytes_row = static_cast<uint32_t>(min(u_end - u0, STAGE_UNITS) * UNIT);
        if (lane == 0) mbar_arrive_expect_tx(&full_bar[slot], bytes_row * rows_valid);
        __syncwarp();
        if (lane < rows_valid)
          bulk_g2s(ring + slot * STAGE_BYTES + lane * ROW_STRIDE,
                   p.w + (row0 + lane) * row_bytes + static_cast<int64_t>(u0) * UNIT, bytes_row, &full_bar[slot]);
      }
    }
  } else {
    // ------------------------------------------------------------------ consumers
    const int tid = threadIdx.x;            // 0..255
    constexpr int XU = (FMT == 2) ? 256 : 128;
    constexpr int XCH = XU / 64;            // 16-byte chunks of x per thread per unit
    // -- stage the activations: per (token, range) power-of-two factor, fp16, fragment order.  All 256
    //    consumer threads walk the staged slice in 16-byte chunks twice: absmax per (token, range), convert.
    {
      constexpr int KPU = (FMT == 2) ? 128 : 64;          // K values per unit
      constexpr int CPR = RANGE_UNITS * KPU / 8;          // 16-byte chunks per range
      const int r_first = u_begin / RANGE_UNITS;
      const int64_t kx0 = static_cast<int64_t>(u_begin) * KPU;
      const int cpt = (u_end - u_begin) * KPU / 8;        // chunks per token
      const int nchunks = p.M * cpt;
      for (int i = tid; i < 16 * MAX_RANGES; i += 256) xmax[i] = 0;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      for (int q = tid; q < nchunks; q += 256) {
        const int t = q / cpt, j = q - t * cpt;
        const uint4 v = ldg_nc_v4(p.x + static_cast<int64_t>(t) * p.K + kx0 + j * 8);
        const uint32_t rr[4] = {v.x, v.y, v.z, v.w};
        float m = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e)
          m = fmaxf(m, fmaxf(fabsf(__uint_as_float(rr[e] << 16)), fabsf(__uint_as_float(rr[e] & 0xFFFF0000u))));
        // non-negative floats order like their bit patterns
        atomicMax(&xmax[t * MAX_RANGES + r_first + j / CPR], static_cast<int>(__float_as_uint(m)));
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");
      for (int q = tid; q < nchunks; q += 256) {
        const int t = q / cpt, j = q - t * cpt;
        const int r = r_first + j / CPR;
        const float m = __uint_as_float(static_cast<uint32_t>(xmax[t * MAX_RANGES + r]));
        int e = 0;
        if (m > 0.f) {
          int ex;
          frexpf(m, &ex);
          e = min(max(ex - 15, -110), 110);               // max |x| * 2^-e in [2^14, 2^15)
        }
        if ((j % CPR) == 0) xsc[t * MAX_RANGES + r] = ldexpf(1.0f, e);
        const float down = ldexpf(1.0f, -e);
        const uint4 v = ldg_nc_v4(p.x + static_cast<int64_t>(t) * p.K + kx0 + j * 8);
        const uint32_t rr[4] = {v.x, v.y, v.z, v.w};
        float f[8];
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2) {
          f[2 * e2] = __uint_as_float(rr[e2] << 16) * down;
          f[2 * e2 + 1] = __uint_as_float(rr[e2] & 0xFFFF0000u) * down;
        }
        float g8[8];
        if (FMT == 2) {   // nibble pairs (0,4) (1,5) (2,6) (3,7)
          g8[0] = f[0]; g8[1] = f[4]; g8[2] = f[1]; g8[3] = f[5]; g8[4] = f[2]; g8[5] = f[6]; g8[6] = f[3]; g8[7] = f[7];
        } else {          // byte pairs (0,2) (1,3) of each word
          g8[0] = f[0]; g8[1] = f[2]; g8[2] = f[1]; g8[3] = f[3]; g8[4] = f[4]; g8[5] = f[6]; g8[6] = f[5]; g8[7] = f[7];
        }
        uint32_t o[4];
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2) {
          __half2 h = __floats2half2_rn(g8[2 * e2], g8[2 * e2 + 1]);
          o[e2] = *reinterpret_cast<uint32_t*>(&h);
        }
        // 8-block j -> (unit, thread c, chunk v) of the B-fragment order
        int u, cc, vv;
        if (FMT == 2) { u = j >> 4; cc = (j >> 2) & 3; vv = j & 3; }
        else { u = j >> 3; cc = (j >> 1) & 3; vv = j & 1; }
        *reinterpret_cast<uint4*>(xs + t * L.token_stride + u * XU + vv * 64 + cc * 16) =
            make_uint4(o[0], o[1], o[2], o[3]);
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");
    }

    const int g = lane >> 2;      // row and token within the m16n8 tile
    const int c = lane & 3;
    const uint32_t xs_base = smem_u32(xs);
    float out_sum = 0.f;          // thread's output (row tid % 16, token tid / 16), summed over ranges
    float acc[MT][4];
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[t][i] = 0.f;
    uint32_t it = 0;
    int rbuf = 0;
    for (int b = b0; b < p.nblocks; b += bstep) {
      const int64_t row0 = static_cast<int64_t>(b) * RB;
      const int64_t rg = (row0 + g < p.N ? row0 + g : p.N - 1);
      const int64_t rg8 = (row0 + g + 8 < p.N ? row0 + g + 8 : p.N - 1);
      for (int st = 0; st < nst; ++st, ++it) {
        const uint32_t slot = it % slots;
        const int u0 = u_begin + st * STAGE_UNITS;
        // the two units of this warp: u0 + warp, u0 + warp + 8
        const int ua = u0 + warp, ub = u0 + warp + 8;
        float s0a = 0.f, s8a = 0.f, s0b = 0.f, s8b = 0.f;
        if (FMT == 2) {
          const int64_t ng = p.K / 128;
          if (ua < u_end) { s0a = __half2float(p.s16[rg * ng + ua]); s8a = __half2float(p.s16[rg8 * ng + ua]); }
          if (ub < u_end) { s0b = __half2float(p.s16[rg * ng + ub]); s8b = __half2float(p.s16[rg8 * ng + ub]); }
        }
        mbar_wait(&full_bar[slot], (it / slots) & 1, abort_v);
        uint4 wa0 = make_uint4(0, 0, 0, 0), wa8 = wa0, wb0 = wa0, wb8 = wa0;
        {
          const uint32_t base = smem_u32(ring + slot * STAGE_BYTES) + c * 16;
          if (ua < u_end) {
            wa0 = lds_v4(base + g * ROW_STRIDE + warp * UNIT);
            wa8 = lds_v4(base + (g + 8) * ROW_STRIDE + warp * UNIT);
          }
          if (ub < u_end) {
            wb0 = lds_v4(base + g * ROW_STRIDE + (warp + 8) * UNIT);
            wb8 = lds_v4(base + (g + 8) * ROW_STRIDE + (warp + 8) * UNIT);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[slot]);

#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int u = half ? ub : ua;
          if (u >= u_end) continue;
          const uint4 w0 = half ? wb0 : wa0;
          const uint4 w8 = half ? wb8 : wa8;
          const uint32_t W0[4] = {w0.x, w0.y, w0.z, w0.w};
          const uint32_t W8[4] = {w8.x, w8.y, w8.z, w8.w};
          // B fragments: chunk v of thread c for token tile t
          uint32_t B[MT][4 * XCH];
          const uint32_t xoff = xs_base + (u - u_begin) * XU + c * 16;
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            const int tok = t * 8 + g;
            if (tok < p.M) {
#pragma unroll
              for (int v = 0; v < XCH; ++v) {
                const uint4 q = lds_v4(xoff + tok * L.token_stride + v * 64);
                B[t][4 * v] = q.x; B[t][4 * v + 1] = q.y; B[t][4 * v + 2] = q.z; B[t][4 * v + 3] = q.w;
              }
            } else {
#pragma unroll
              for (int v = 0; v < 4 * XCH; ++v) B[t][v] = 0u;
            }
          }
          if (FMT == 2) {
            float cg[MT][4];
#pragma unroll
            for (int t = 0; t < MT; ++t)
#pragma unroll
              for (int i = 0; i < 4; ++i) cg[t][i] = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t P0[4], P8[4];
              deq4_word(W0[i], P0);
              deq4_word(W8[i], P8);
              const uint32_t aj0[4] = {P0[0], P8[0], P0[1], P8[1]};   // MMA 2i:   nibbles (0,4) | (1,5)
              const uint32_t aj1[4] = {P0[2], P8[2], P0[3], P8[3]};   // MMA 2i+1: nibbles (2,6) | (3,7)
#pragma unroll
              for (int t = 0; t < MT; ++t) {
                mma_f16_16816(cg[t], aj0, B[t][4 * i + 0], B[t][4 * i + 1]);
                mma_f16_16816(cg[t], aj1, B[t][4 * i + 2], B[t][4 * i + 3]);
              }
            }
            const float sa = half ? s0b : s0a, sb = half ? s8b : s8a;
#pragma unroll
            for (int t = 0; t < MT; ++t) {
              acc[t][0] = fmaf(cg[t][0], sa, acc[t][0]);
              acc[t][1] = fmaf(cg[t][1], sa, acc[t][1]);
              acc[t][2] = fmaf(cg[t][2], sb, acc[t][2]);
              acc[t][3] = fmaf(cg[t][3], sb, acc[t][3]);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t a[4];
              deq8_word(W0[i], a[0], a[2]);
              deq8_word(W8[i], a[1], a[3]);
#pragma unroll
              for (int t = 0; t < MT; ++t) mma_f16_16816(acc[t], a, B[t][2 * i], B[t][2 * i + 1]);
            }
          }
        }

        // ------------------------------------------------------------ end of a K range: add the warps
        const int done = u0 + STAGE_UNITS - u_begin;
        if ((done % RANGE_UNITS) == 0 || st == nst - 1) {
          const int range = u0 / RANGE_UNITS;
          float* r = red + ((rbuf * WARPS + warp) * 32 + lane) * 8;
#pragma unroll
          for (int t = 0; t < MT; ++t)
#pragma unroll
            for (int i = 0; i < 4; ++i) { r[4 * t + i] = acc[t][i]; acc[t][i] = 0.f; }
          asm volatile("bar.sync 1, 256;" ::: "memory");
          const int orow = tid & 15, otok = tid >> 4;
          if (otok < p.M) {
            const int tt = otok >> 3, tk = otok & 7;
            const int src_lane = (orow & 7) * 4 + (tk >> 1);
            const int reg = tt * 4 + (orow >> 3) * 2 + (tk & 1);
            float rs = 0.f;
#pragma unroll
            for (int w = 0; w < WARPS; ++w) rs += red[((rbuf * WARPS + w) * 32 + src_lane) * 8 + reg];
            out_sum += rs * xsc[otok * MAX_RANGES + range];
          }
          rbuf ^= 1;
        }
      }
      // ---------------------------------------------------------------- end of a row block
      if (!p.cluster) {
        const int orow = tid & 15, otok = tid >> 4;
        const int64_t n = row0 + orow;
        if (otok < p.M && n < p.N) {
          float v = out_sum;
          if (FMT == 1) v *= __half2float(p.s16[n]);
          if (p.bias) v += bf16_bits_to_f32(p.bias[n]);
          uint16_t* yp = p.y + static_cast<int64_t>(otok) * p.ldy + n;
          if (p.acc) v += bf16_bits_to_f32(*yp);
          *yp = f32_to_bf16_bits(v);
        }
        out_sum = 0.f;
      } else {
        csum[tid] = out_sum;
      }
    }
  }

  if (p.cluster) {
    // ------------------------------------------------------------------ add the K ranges of the cluster
    // Rank r of the cluster holds range r of row block blockIdx.x.  Rank 0 reads the other ranks' partials
    // through distributed shared memory in rank order; the second barrier keeps every CTA (and its shared
    // memory) alive until rank 0 has read it.
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (blockIdx.y == 0 && threadIdx.x < 256) {
      const int orow = threadIdx.x & 15, otok = threadIdx.x >> 4;
      const int64_t n = static_cast<int64_t>(blockIdx.x) * RB + orow;
      float v = 0.f;
      const uint32_t local = smem_u32(&csum[threadIdx.x]);
      for (int r = 0; r < p.nranges; ++r) {
        uint32_t remote;
        float part;
        asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(r));
        asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(part) : "r"(remote) : "memory");
        v += part;
      }
      if (otok < p.M && n < p.N) {
        if (FMT == 1) v *= __half2float(p.s16[n]);
        if (p.bias) v += bf16_bits_to_f32(p.bias[n]);
        uint16_t* yp = p.y + static_cast<int64_t>(otok) * p.ldy + n;
        if (p.acc) v += bf16_bits_to_f32(*yp);
        *yp = f32_to_bf16_bits(v);
      }
    }
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  }
}

// ------------------------------------------------------------------------------------------- launcher
int gemv_max_k(int fmt) {
  // the cluster path takes at most MAX_CLUSTER K ranges; the persistent path needs all of x in shared memory
  return gemv::MAX_CLUSTER * gemv::RANGE_UNITS * gemv::UNIT * (fmt == 2 ? 2 : 1);
}

template <int FMT, int MT>
static cudaError_t launch_gemv_t(GemvParams p, int sms, cudaStream_t st) {
  using namespace gemv;
  // persistent when there are enough row blocks and all of x fits beside a ring of MIN_SLOTS stages
  const GemvSmem full = gemv_smem(FMT, p.M, p.total_units, MIN_SLOTS);
  const bool persistent = p.nblocks >= sms && full.total <= SMEM_LIMIT - 1024 && p.nranges <= MAX_RANGES;
  if (!persistent && p.nranges > MAX_CLUSTER) return cudaErrorInvalidValue;
  p.cluster = persistent ? 0 : 1;
  p.xs_units = persistent ? p.total_units : min(p.total_units, RANGE_UNITS);
  const GemvSmem base = gemv_smem(FMT, p.M, p.xs_units, 0);
  int slots = (SMEM_LIMIT - 1024 - base.total) / STAGE_BYTES;
  slots = max(MIN_SLOTS, min(MAX_SLOTS, slots));
  p.slots = slots;
  const size_t smem = static_cast<size_t>(gemv_smem(FMT, p.M, p.xs_units, slots).total);
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(gemv_kernel<FMT, MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         SMEM_LIMIT);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  if (persistent) {
    cfg.gridDim = dim3(static_cast<unsigned>(min(p.nblocks, sms)), 1, 1);
    cfg.numAttrs = 0;
  } else {
    cfg.gridDim = dim3(static_cast<unsigned>(p.nblocks), static_cast<unsigned>(p.nranges), 1);
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = static_cast<unsigned>(p.nranges);
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = p.nranges > 1 ? 1 : 0;
  }
  cfg.blockDim = dim3(288, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  return cudaLaunchKernelEx(&cfg, gemv_kernel<FMT, MT>, p);
}

cudaError_t launch_gemv(int fmt, const void* x, int64_t M, int64_t K, const void* codes, const void* scales,
                        int64_t N, const void* bias, int acc, void* y, int64_t ldy, int sms, cudaStream_t st) {
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
  p.nblocks = static_cast<int>((N + gemv::RB - 1) / gemv::RB);
  p.nranges = (p.total_units + gemv::RANGE_UNITS - 1) / gemv::RANGE_UNITS;
  p.slots = gemv::MIN_SLOTS;
  p.xs_units = 0;
  p.cluster = 0;
  if (fmt == 2) return M <= 8 ? launch_gemv_t<2, 1>(p, sms, st) : launch_gemv_t<2, 2>(p, sms, st);
  return M <= 8 ? launch_gemv_t<1, 1>(p, sms, st) : launch_gemv_t<1, 2>(p, sms, st);
}

}  // namespace lb

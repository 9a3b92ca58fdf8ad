// Decode-regime product (M <= 16 tokens): y[M, N] = x[M, K] . deq(W)[N, K]^T.
//
// The weight stream is the cost: every byte of codes is read once from HBM.  Work is cut in row blocks of
// 16 output rows.  A CTA streams its row blocks through a shared-memory ring with TMA bulk copies
// (cp.async.bulk, completion on mbarriers): one 2 KB copy per row per stage (smaller copies do not reach full
// HBM bandwidth), plus one copy of the row block's fp16 scales.  Sixteen warps each take two 64-byte units per
// row per stage (int4: 128 values = one scale group; int8: 64 values).  Every stage ends in a CTA barrier (it
// is one K range, whose warp partials are added there), so thread 0 refills the slot just drained right after
// that barrier: no producer warp and no empty-slot barriers.
//
// Activations are converted once per CTA into shared memory as fp16, already in the order of the tensor-
// core B fragments, with a power-of-two factor per (token, K range) so the bf16 -> fp16 conversion is exact.
// Codes are dequantised in registers with one LOP3 per pair: the code, made offset-binary by an XOR folded
// into the LOP3, lands in the mantissa of 1024 in fp16 (int4 nibbles at bits 4-7 land as 1024 + 16 n), which
// is exact.  The offsets are not removed per code: each unit's tensor-core sums are split in two classes of
// K positions (even / odd nibbles), the odd class is scaled by 1/16, and one float per (token, unit),
// 1032 * sum(x even) + 72 * sum(x odd) (int8: 1152 * sum(x)), computed once while staging x, is subtracted.
// Products accumulate in float32 (m16n8k16 mma.sync); the fp16 scale of each 128-value group multiplies the
// unit's float32 partial (int8: the row scale multiplies the final sum).
//
// Sums have a fixed structure that depends only on K: the codes of a row are cut in K ranges of 2 KB
// (32 units, one stage); within a range each warp adds its two units in order, the sixteen warps are added
// in order, and the ranges are added in order.  Large-N calls run persistent CTAs (one per SM) that walk whole
// row blocks; small-N calls give each K range its own CTA in a thread-block cluster and add the ranges in
// rank order through distributed shared memory.  Both produce identical bits, so a column-sharded layer
// matches the unsharded one exactly.  No global scratch memory is used.
//
// With programmatic dependent launch (static weights), the producer streams weights before the previous
// kernel on the stream has finished; only the activations and the output wait for it (griddepcontrol.wait).
#include "lb_common.cuh"
#include "lb_kernels.h"

namespace lb {

namespace gemv {
constexpr int RB = 16;                          // rows per row block (one m16 tile)
constexpr int UNIT = 64;                        // bytes of one row per unit
constexpr int WARPS = 16;                       // all warps compute; thread 0 also issues the copies
constexpr int CONSUMERS = WARPS * 32;
constexpr int THREADS = CONSUMERS;
constexpr int STAGE_UNITS = 32;                 // units per stage (two per warp) = one K range
constexpr int STAGE_ROW = UNIT * STAGE_UNITS;   // 2048 bytes of a row per stage
constexpr int ROW_STRIDE = STAGE_ROW + 64;      // rows g and g+8 in different banks
constexpr int STAGE_BYTES = RB * ROW_STRIDE;    // 33792
constexpr int RANGE_UNITS = STAGE_UNITS;        // units per K range (2 KB of codes per row)
constexpr int MAX_RANGES = 32;
constexpr int MAX_CLUSTER = 8;
constexpr int SMEM_LIMIT = 227 * 1024;
constexpr int MIN_SLOTS = 2, MAX_SLOTS = 6;
constexpr int SCALE_SLOTS = 2;
constexpr int MAX_SCALE_SLOT = 8192;            // 16 rows x 256 groups (K <= 32768)
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
  int scale_slot;         // bytes of one scale-ring slot (persistent int4 path), 0 = scales by plain loads
};

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}
__device__ __forceinline__ float half_bits_to_f32(uint32_t h) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
}

// m16n8k16 fp16 tensor-core product, fp32 accumulate: d += a * b.
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// int4: one word (8 codes, two's complement nibbles) -> four fp16 pairs with n = q + 8:
// P0 = 1024 + (n0, n4), P1 = 1024 + 16 (n1, n5), P2 = 1024 + (n2, n6), P3 = 1024 + 16 (n3, n7).
__device__ __forceinline__ void deq4_word(uint32_t w, uint32_t (&P)[4]) {
  const uint32_t w8 = w >> 8;
  P[0] = lop3_and_xor_or(w, 0x000F000Fu, 0x64086408u);
  P[1] = lop3_and_xor_or(w, 0x00F000F0u, 0x64806480u);
  P[2] = lop3_and_xor_or(w8, 0x000F000Fu, 0x64086408u);
  P[3] = lop3_and_xor_or(w8, 0x00F000F0u, 0x64806480u);
}
// int8: one word (4 codes) -> two fp16 pairs 1024 + (n0, n2), 1024 + (n1, n3) with n = q + 128.
__device__ __forceinline__ void deq8_word(uint32_t w, uint32_t& q02, uint32_t& q13) {
  const uint32_t v = w ^ 0x80808080u;
  q02 = prmt(v, 0x00006464u, 0x5240u);
  q13 = prmt(v, 0x00006464u, 0x5341u);
}

// Shared-memory carve-up, in bytes from the base of dynamic shared memory.
struct GemvSmem {
  int ring, xs, corr, xsc, red, zeros, csum, scl, bars, total;
  int token_stride;   // bytes of one token's staged activations
};

__host__ __device__ inline int gemv_scale_slot_bytes(int fmt, int64_t K) {
  return fmt == 2 ? static_cast<int>(((16 * (K / 128) * 2) + 15) & ~15) : 0;
}

__host__ __device__ inline GemvSmem gemv_smem(int fmt, int M, int MT, int xs_units, int slots, int scale_slot) {
  using namespace gemv;
  GemvSmem s;
  const int xu = (fmt == 2) ? 256 : 128;     // staged bytes of x per unit per token
  s.token_stride = xs_units * xu + 64;
  s.ring = 0;
  s.xs = slots * STAGE_BYTES;                                  // multiple of 128
  s.corr = s.xs + ((M * s.token_stride + 127) & ~127);
  s.xsc = s.corr + ((M * xs_units * 4 + 127) & ~127);
  s.red = s.xsc + 2 * 16 * MAX_RANGES * 4;                     // xsc + xmax
  s.zeros = s.red + (MT == 1 ? 2 : 1) * WARPS * 32 * 4 * MT * 4;   // warp partials (double-buffered for MT 1)
  s.csum = s.zeros + 256;                                      // 256 zero bytes (absent tokens)
  s.scl = s.csum + 256 * 4;
  s.bars = s.scl + SCALE_SLOTS * scale_slot;
  s.total = s.bars + (MAX_SLOTS + SCALE_SLOTS) * 8 + 64;
  return s;
}

// XREG: every row is one K range, so each warp's two units (and their B fragments) are fixed for the kernel.
template <int FMT, int MT, bool XREG>
__global__ void __launch_bounds__(gemv::THREADS, 1) gemv_kernel(const GemvParams p) {
  using namespace gemv;
  extern __shared__ __align__(1024) uint8_t dyn_smem[];
  const GemvSmem L = gemv_smem(FMT, p.M, MT, p.xs_units, p.slots, p.scale_slot);
  uint8_t* ring = dyn_smem + L.ring;
  uint8_t* xs = dyn_smem + L.xs;
  float* corr = reinterpret_cast<float*>(dyn_smem + L.corr);   // [M][xs_units] offset corrections
  float* xsc = reinterpret_cast<float*>(dyn_smem + L.xsc);     // [16 tokens][MAX_RANGES] 2^e factors
  int* xmax = reinterpret_cast<int*>(xsc + 16 * MAX_RANGES);   // [16 tokens][MAX_RANGES] absmax bits
  float* red = reinterpret_cast<float*>(dyn_smem + L.red);     // [2][WARPS][32][4 * MT]
  float* csum = reinterpret_cast<float*>(dyn_smem + L.csum);   // [256]
  uint8_t* scl = dyn_smem + L.scl;                             // [SCALE_SLOTS][16][K/128] binary16
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(dyn_smem + L.bars);
  uint64_t* sfull_bar = full_bar + MAX_SLOTS;
  int* abort_flag = reinterpret_cast<int*>(sfull_bar + SCALE_SLOTS);

  pdl_launch_dependents();
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
  const int nst = (u_end - u_begin + STAGE_UNITS - 1) / STAGE_UNITS;   // stages (= ranges) per row block
  const int slots = p.slots;

  const int nmine = (p.nblocks - b0 + bstep - 1) / bstep;               // row blocks of this CTA
  const int nstages = nmine * nst;
  // issue stage `it` of this CTA (row block b0 + (it / nst) * bstep, K stage it % nst) into its ring slot;
  // called by all lanes of warp 0: lane 0 registers the byte count, lanes 0..15 copy one row each
  auto issue_stage = [&](int it) {
    const int k = it / nst, st = it - k * nst;
    const int64_t row0 = static_cast<int64_t>(b0 + k * bstep) * RB;
    const int rows_valid = static_cast<int>(p.N - row0 < RB ? p.N - row0 : RB);
    const int u0 = u_begin + st * STAGE_UNITS;
    const uint32_t bytes_row = static_cast<uint32_t>(min(u_end - u0, STAGE_UNITS) * UNIT);
    const int slot = it % slots;
    if (lane == 0) mbar_arrive_expect_tx(&full_bar[slot], bytes_row * rows_valid);
    __syncwarp();
    if (lane < rows_valid)
      bulk_g2s(ring + slot * STAGE_BYTES + lane * ROW_STRIDE,
               p.w + (row0 + lane) * row_bytes + static_cast<int64_t>(u0) * UNIT, bytes_row, &full_bar[slot]);
  };
  // issue the scales of the k-th row block of this CTA into scale slot k % SCALE_SLOTS; a partial last block
  // is read with plain loads instead
  auto issue_scales = [&](int k) {
    const int64_t row0 = static_cast<int64_t>(b0 + k * bstep) * RB;
    const int slot = k % SCALE_SLOTS;
    if (p.N - row0 >= RB) {
      const uint32_t bytes = static_cast<uint32_t>(RB * (p.K / 128) * 2);
      mbar_arrive_expect_tx(&sfull_bar[slot], bytes);
      bulk_g2s(scl + slot * p.scale_slot, p.s16 + row0 * (p.K / 128), bytes, &sfull_bar[slot]);
    } else {
      mbar_arrive(&sfull_bar[slot]);
    }
  };

  if (warp == 0) {
    if (lane == 0) {
      for (int s = 0; s < slots; ++s) mbar_init(&full_bar[s], 1);
      for (int s = 0; s < SCALE_SLOTS; ++s) mbar_init(&sfull_bar[s], 1);
      *abort_flag = 0;
      fence_barrier_init();
      // the weights do not depend on earlier kernels: start streaming before waiting for them
      if (p.scale_slot)
        for (int k = 0; k < min(nmine, SCALE_SLOTS); ++k) issue_scales(k);
    }
    __syncwarp();
    for (int it = 0; it < min(nstages, slots); ++it) issue_stage(it);
  }
  __syncthreads();
  volatile int* abort_v = abort_flag;

  {
    // ------------------------------------------------------------------ consumers
    const int tid = threadIdx.x;            // 0..CONSUMERS-1
    constexpr int XU = (FMT == 2) ? 256 : 128;
    constexpr int XCH = XU / 64;            // 16-byte chunks of x per thread per unit
    pdl_wait();                             // the activations (and the output) come from earlier kernels
    // -- stage the activations: per (token, range) power-of-two factor, fp16, fragment order.  All consumer
    //    threads walk the staged slice in 16-byte chunks twice: absmax per (token, range), then convert.
    {
      constexpr int KPU = (FMT == 2) ? 128 : 64;          // K values per unit
      constexpr int CPR = RANGE_UNITS * KPU / 8;          // 16-byte chunks per range
      const int r_first = u_begin / RANGE_UNITS;
      const int64_t kx0 = static_cast<int64_t>(u_begin) * KPU;
      const int cpt = (u_end - u_begin) * KPU / 8;        // chunks per token
      for (int i = tid; i < 16 * MAX_RANGES; i += CONSUMERS) xmax[i] = 0;
      for (int i = tid; i < 64; i += CONSUMERS) reinterpret_cast<uint32_t*>(dyn_smem + L.zeros)[i] = 0u;
      asm volatile("bar.sync 1, %0;" ::"n"(CONSUMERS) : "memory");
      for (int t = 0; t < p.M; ++t)
      for (int j = tid; j < cpt; j += CONSUMERS) {
        const uint4 v = ldg_nc_v4(p.x + static_cast<int64_t>(t) * p.K + kx0 + j * 8);
        const uint32_t rr[4] = {v.x, v.y, v.z, v.w};
        float m = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e)
          m = fmaxf(m, fmaxf(fabsf(__uint_as_float(rr[e] << 16)), fabsf(__uint_as_float(rr[e] & 0xFFFF0000u))));
        // non-negative floats order like their bit patterns
        atomicMax(&xmax[t * MAX_RANGES + r_first + j / CPR], static_cast<int>(__float_as_uint(m)));
      }
      asm volatile("bar.sync 1, %0;" ::"n"(CONSUMERS) : "memory");
      for (int t = 0; t < p.M; ++t)
      for (int j = tid; j < cpt; j += CONSUMERS) {
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
        if (FMT == 2) {   // even class (0,4) (2,6), then odd class (1,5) (3,7)
          g8[0] = f[0]; g8[1] = f[4]; g8[2] = f[2]; g8[3] = f[6]; g8[4] = f[1]; g8[5] = f[5]; g8[6] = f[3]; g8[7] = f[7];
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
      asm volatile("bar.sync 1, %0;" ::"n"(CONSUMERS) : "memory");
      // offset corrections, one thread per (token, unit), summed in a fixed order from the staged fp16 values:
      // int4: 1032 * sum(even k) + 72 * sum(odd k); int8: 1152 * sum(k)
      const int units = u_end - u_begin;
      for (int q = tid; q < p.M * units; q += CONSUMERS) {
        const int t = q / units, u = q - t * units;
        const uint8_t* src = xs + t * L.token_stride + u * XU;
        float se = 0.f, so = 0.f;
        for (int ch = 0; ch < XU / 16; ++ch) {
          const uint4 v = *reinterpret_cast<const uint4*>(src + ch * 16);
          const __half2* h = reinterpret_cast<const __half2*>(&v);
          const float2 a = __half22float2(h[0]), b = __half22float2(h[1]);
          const float2 c2 = __half22float2(h[2]), d = __half22float2(h[3]);
          if (FMT == 2) {
            se += (a.x + a.y) + (b.x + b.y);
            so += (c2.x + c2.y) + (d.x + d.y);
          } else {
            se += ((a.x + a.y) + (b.x + b.y)) + ((c2.x + c2.y) + (d.x + d.y));
          }
        }
        corr[t * units + u] = (FMT == 2) ? fmaf(1032.f, se, 72.f * so) : 1152.f * se;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(CONSUMERS) : "memory");
    }

    const int g = lane >> 2;      // row and token within the m16n8 tile
    const int c = lane & 3;
    // B fragments: token rows of x; absent tokens (tok >= M) read zeros from the other 64-byte half of the
    // bank window, so the loads need no branch and cause no conflicts
    uint32_t xrow[MT];
    bool tok_ok[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      tok_ok[t] = t * 8 + g < p.M;
      xrow[t] = smem_u32(xs) + (t * 8 + g) * L.token_stride + c * 16;
    }
    const uint32_t zbase = smem_u32(dyn_smem + L.zeros);
    const uint32_t ring_base = smem_u32(ring) + c * 16;
    const int units_staged = u_end - u_begin;
    // the C fragment of this thread holds tokens 2c and 2c+1 of each token tile
    auto corr_of = [&](int t, int u, int j) -> float {
      const int tok = t * 8 + 2 * c + j;
      return tok < p.M ? corr[tok * units_staged + (u - u_begin)] : 0.f;
    };
    auto load_b = [&](int u, uint32_t (&B)[MT][4 * XCH]) {
      const uint32_t uoff = static_cast<uint32_t>(u - u_begin) * XU;
#pragma unroll
      for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int v = 0; v < XCH; ++v) {
          const uint4 q = lds_v4(tok_ok[t] ? xrow[t] + uoff + v * 64 : zbase + ((v * 64 + 64) & 127));
          B[t][4 * v] = q.x; B[t][4 * v + 1] = q.y; B[t][4 * v + 2] = q.z; B[t][4 * v + 3] = q.w;
        }
    };
    // rows of one K range (K <= 2 KB of codes per row): each warp's two units are the same for every row
    // block, so their B fragments and corrections stay in registers
    uint32_t Bk[2][MT][4 * XCH];
    float Ck[2][MT][2];
    if constexpr (XREG) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int uu = u_begin + warp + h * WARPS;
        if (uu < u_end) {
          load_b(uu, Bk[h]);
#pragma unroll
          for (int t = 0; t < MT; ++t) { Ck[h][t][0] = corr_of(t, uu, 0); Ck[h][t][1] = corr_of(t, uu, 1); }
        }
      }
    }
    float out_sum = 0.f;          // thread's output (row tid % 16, token tid / 16), summed over ranges
    uint32_t slot = 0, phase = 0;
    uint32_t sslot = 0, sphase = 0;
    int rbuf = 0, it = 0, kb = 0;
    const int64_t ng = p.K / 128;
    for (int b = b0; b < p.nblocks; b += bstep) {
      const int64_t row0 = static_cast<int64_t>(b) * RB;
      const bool full_block = p.N - row0 >= RB;
      const int64_t rg = row0 + g < p.N ? row0 + g : p.N - 1;
      const int64_t rg8 = row0 + g + 8 < p.N ? row0 + g + 8 : p.N - 1;
      bool smem_scales = false;
      uint32_t sbase = 0;
      if (FMT == 2 && p.scale_slot) {
        mbar_wait(&sfull_bar[sslot], sphase, abort_v);
        smem_scales = full_block;
        sbase = smem_u32(scl + sslot * p.scale_slot) + static_cast<uint32_t>(g * ng * 2);
      }
      for (int st = 0; st < nst; ++st) {
        const int u0 = u_begin + st * STAGE_UNITS;
        const int ua = u0 + warp, ub = u0 + warp + WARPS;   // this warp's two units
        float sc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};           // [unit][row g / g+8]
        if (FMT == 2) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int uu = h ? ub : ua;
            if (uu < u_end) {
              if (smem_scales) {
                sc[h][0] = half_bits_to_f32(lds_u16(sbase + uu * 2));
                sc[h][1] = half_bits_to_f32(lds_u16(sbase + static_cast<uint32_t>((8 * ng + uu) * 2)));
              } else {
                sc[h][0] = __half2float(p.s16[rg * ng + uu]);
                sc[h][1] = __half2float(p.s16[rg8 * ng + uu]);
              }
            }
          }
        } else {
          sc[0][0] = sc[0][1] = sc[1][0] = sc[1][1] = 1.f;     // int8: the row scale comes at the end
        }
        mbar_wait(&full_bar[slot], phase, abort_v);
        uint4 wr[2][2];
        const uint32_t sbuf = ring_base + slot * STAGE_BYTES;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int uu = h ? ub : ua;
          if (uu < u_end) {
            const uint32_t a = sbuf + (uu - u0) * UNIT;
            wr[h][0] = lds_v4(a + g * ROW_STRIDE);
            wr[h][1] = lds_v4(a + (g + 8) * ROW_STRIDE);
          } else {
            wr[h][0] = make_uint4(0, 0, 0, 0);
            wr[h][1] = wr[h][0];
          }
        }
        if (++slot == static_cast<uint32_t>(slots)) { slot = 0; phase ^= 1; }

        float acc[MT][4];
#pragma unroll
        for (int t = 0; t < MT; ++t)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[t][i] = 0.f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int uu = h ? ub : ua;
          if (uu >= u_end) continue;
          const uint32_t W0[4] = {wr[h][0].x, wr[h][0].y, wr[h][0].z, wr[h][0].w};
          const uint32_t W8[4] = {wr[h][1].x, wr[h][1].y, wr[h][1].z, wr[h][1].w};
          uint32_t Bl[MT][4 * XCH];
          float Cl[MT][2];
          if constexpr (XREG) {
#pragma unroll
            for (int t = 0; t < MT; ++t) {
#pragma unroll
              for (int v = 0; v < 4 * XCH; ++v) Bl[t][v] = Bk[h][t][v];
              Cl[t][0] = Ck[h][t][0];
              Cl[t][1] = Ck[h][t][1];
            }
          } else {
            load_b(uu, Bl);
#pragma unroll
            for (int t = 0; t < MT; ++t) { Cl[t][0] = corr_of(t, uu, 0); Cl[t][1] = corr_of(t, uu, 1); }
          }
          const uint32_t (&B)[MT][4 * XCH] = Bl;
          const float (&Cc)[MT][2] = Cl;
          float c0[MT][4], c1[MT][4];       // two classes of K positions = two independent MMA chains
#pragma unroll
          for (int t = 0; t < MT; ++t)
#pragma unroll
            for (int i = 0; i < 4; ++i) { c0[t][i] = 0.f; c1[t][i] = 0.f; }
          if (FMT == 2) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t P0[4], P8[4];
              deq4_word(W0[i], P0);
              deq4_word(W8[i], P8);
              const uint32_t ae[4] = {P0[0], P8[0], P0[2], P8[2]};   // even nibbles: (0,4) | (2,6)
              const uint32_t ao[4] = {P0[1], P8[1], P0[3], P8[3]};   // odd nibbles:  (1,5) | (3,7), x16
#pragma unroll
              for (int t = 0; t < MT; ++t) {
                mma_f16_16816(c0[t], ae, B[t][4 * i + 0], B[t][4 * i + 1]);
                mma_f16_16816(c1[t], ao, B[t][4 * i + 2], B[t][4 * i + 3]);
              }
            }
          } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t a[4];
              deq8_word(W0[i], a[0], a[2]);
              deq8_word(W8[i], a[1], a[3]);
#pragma unroll
              for (int t = 0; t < MT; ++t) {
                if (i & 1) mma_f16_16816(c1[t], a, B[t][2 * i], B[t][2 * i + 1]);
                else mma_f16_16816(c0[t], a, B[t][2 * i], B[t][2 * i + 1]);
              }
            }
          }
          // unit sum = class0 + class1 / 16 (int8: + class1) - correction, times the group scale
          const float k1 = (FMT == 2) ? 0.0625f : 1.0f;
#pragma unroll
          for (int t = 0; t < MT; ++t) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float v = fmaf(c1[t][i], k1, c0[t][i]) - Cc[t][i & 1];
              acc[t][i] = fmaf(v, sc[h][i >> 1], acc[t][i]);
            }
          }
        }

        // ------------------------------------------------------------ end of the K range: add the warps
        {
          const int range = u0 / RANGE_UNITS;
          float* r = red + ((rbuf * WARPS + warp) * 32 + lane) * (4 * MT);
#pragma unroll
          for (int t = 0; t < MT; ++t)
#pragma unroll
            for (int i = 0; i < 4; ++i) r[4 * t + i] = acc[t][i];
          asm volatile("bar.sync 1, %0;" ::"n"(CONSUMERS) : "memory");
          // every warp has read this stage's slot: refill it with the stage `slots` ahead
          if (warp == 0 && it + slots < nstages) issue_stage(it + slots);
          ++it;
          const int orow = tid & 15, otok = tid >> 4;
          if (tid < 256 && otok < p.M) {
            const int tt = otok >> 3, tk = otok & 7;
            const int src_lane = (orow & 7) * 4 + (tk >> 1);
            const int reg = tt * 4 + (orow >> 3) * 2 + (tk & 1);
            float rs = 0.f;
#pragma unroll
            for (int w = 0; w < WARPS; ++w) rs += red[((rbuf * WARPS + w) * 32 + src_lane) * (4 * MT) + reg];
            out_sum += rs * xsc[otok * MAX_RANGES + range];
          }
          if constexpr (MT == 1) rbuf ^= 1;                     // two buffers: the next write is safe
          else asm volatile("bar.sync 1, %0;" ::"n"(CONSUMERS) : "memory");   // one buffer: wait for the reads
        }
      }
      // ---------------------------------------------------------------- end of a row block
      if (FMT == 2 && p.scale_slot) {
        // the last range barrier of this block passed, so no warp reads its scale slot any more
        if (tid == 0 && kb + SCALE_SLOTS < nmine) issue_scales(kb + SCALE_SLOTS);
        if (++sslot == SCALE_SLOTS) { sslot = 0; sphase ^= 1; }
      }
      ++kb;
      if (!p.cluster) {
        const int orow = tid & 15, otok = tid >> 4;
        const int64_t n = row0 + orow;
        if (tid < 256 && otok < p.M && n < p.N) {
          float v = out_sum;
          if (FMT == 1) v *= __half2float(p.s16[n]);
          if (p.bias) v += bf16_bits_to_f32(p.bias[n]);
          uint16_t* yp = p.y + static_cast<int64_t>(otok) * p.ldy + n;
          if (p.acc) v += bf16_bits_to_f32(*yp);
          *yp = f32_to_bf16_bits(v);
        }
        out_sum = 0.f;
      } else if (tid < 256) {
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
    if (blockIdx.y == 0 && threadIdx.x < 256) {  // consumers 0..255 own the 16 x 16 outputs
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

template <int FMT, int MT, bool XREG>
static cudaError_t launch_kernel_t(const GemvParams& p, const cudaLaunchConfig_t& cfg) {
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(gemv_kernel<FMT, MT, XREG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         gemv::SMEM_LIMIT);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  return cudaLaunchKernelEx(&cfg, gemv_kernel<FMT, MT, XREG>, p);
}

template <int FMT, int MT>
static cudaError_t launch_gemv_t(GemvParams p, int sms, bool pdl, cudaStream_t st) {
  using namespace gemv;
  // persistent when there are enough row blocks and all of x fits beside a ring of MIN_SLOTS stages
  const int sslot = gemv_scale_slot_bytes(FMT, p.K);
  const GemvSmem full = gemv_smem(FMT, p.M, MT, p.total_units, MIN_SLOTS, sslot);
  const bool persistent = p.nblocks >= sms && full.total <= SMEM_LIMIT && p.nranges <= MAX_RANGES &&
                          sslot <= MAX_SCALE_SLOT;
  if (!persistent && p.nranges > MAX_CLUSTER) return cudaErrorInvalidValue;
  p.cluster = persistent ? 0 : 1;
  p.xs_units = persistent ? p.total_units : min(p.total_units, RANGE_UNITS);
  p.scale_slot = persistent ? sslot : 0;
  const GemvSmem base = gemv_smem(FMT, p.M, MT, p.xs_units, 0, p.scale_slot);
  int slots = (SMEM_LIMIT - base.total) / STAGE_BYTES;
  slots = max(MIN_SLOTS, min(MAX_SLOTS, slots));
  p.slots = slots;
  const size_t smem = static_cast<size_t>(gemv_smem(FMT, p.M, MT, p.xs_units, slots, p.scale_slot).total);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (persistent) {
    cfg.gridDim = dim3(static_cast<unsigned>(min(p.nblocks, sms)), 1, 1);
  } else {
    cfg.gridDim = dim3(static_cast<unsigned>(p.nblocks), static_cast<unsigned>(p.nranges), 1);
    if (p.nranges > 1) {
      attr[na].id = cudaLaunchAttributeClusterDimension;
      attr[na].val.clusterDim.x = 1;
      attr[na].val.clusterDim.y = static_cast<unsigned>(p.nranges);
      attr[na].val.clusterDim.z = 1;
      ++na;
    }
  }
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  // one K range per CTA (cluster path, or persistent rows of at most one range): with one token tile the
  // fragments stay in registers
  if constexpr (MT == 1) {
    if (p.cluster || p.total_units <= RANGE_UNITS) return launch_kernel_t<FMT, MT, true>(p, cfg);
  }
  return launch_kernel_t<FMT, MT, false>(p, cfg);
}

cudaError_t launch_gemv(int fmt, const void* x, int64_t M, int64_t K, const void* codes, const void* scales,
                        int64_t N, const void* bias, int acc, void* y, int64_t ldy, int sms, bool pdl,
                        cudaStream_t st) {
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
  p.scale_slot = 0;
  if (fmt == 2) return M <= 8 ? launch_gemv_t<2, 1>(p, sms, pdl, st) : launch_gemv_t<2, 2>(p, sms, pdl, st);
  return M <= 8 ? launch_gemv_t<1, 1>(p, sms, pdl, st) : launch_gemv_t<1, 2>(p, sms, pdl, st);
}

}  // namespace lb

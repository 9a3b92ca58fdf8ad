// Decode-regime product (M <= 16 tokens): y[M, N] = x[M, K] . deq(W)[N, K]^T.
//
// The weight stream is the cost: every byte of codes is read once from HBM.  Work items are (row block, K
// range): 16 output rows (one m16 tensor-core tile) x 2 KB of codes per row (32 units of 64 bytes; int4: a
// unit is 128 values = one scale group; int8: 64 values).
//
// Roles per CTA: one producer warp streams the CTA's items, in order, through a shared-memory ring with TMA
// bulk copies (cp.async.bulk, one 2 KB copy per row -- smaller copies do not reach full HBM bandwidth -- with
// an evict-first L2 policy, as the weights are read once) and full / empty mbarriers per slot.  The consumer
// warps form G groups of four; item q belongs to group q % G, so G items are multiplied at once.  Each group
// owns every G-th slot of the ring (the ring holds a multiple of G slots), so a slot is always filled for, and
// read by, one group in item order and a parity wait can never see a phase that belongs to another item.  A
// warp copies all of its codes of an item into registers and releases the slot before multiplying.  Within an
// item, warp w of the group takes units w, w + 4, ... (eight units), in order; the four warp partials are
// added in warp order after one group barrier.
//
// int4 runs on the bf16 tensor path: a code q becomes the bf16 value 136 + q (= 128 + (q + 8), 8 significant
// bits, exact) with one LOP3 per pair -- the XOR that makes the nibble offset-binary is folded into it -- and
// the activations are used as they are, bf16 in the B-fragment order, so every product is exact in the fp32
// accumulation.  The offset is not removed per code: one float per (token, unit), 136 * sum(x), computed while
// staging x, starts the accumulation negated.  int8 runs on the fp16 path: codes 1024 + (q + 128) are exact in
// fp16, the activations are converted once per CTA to fp16 with a power-of-two factor per (token, K range) so
// the conversion is exact, and 1152 * sum(x) is the offset correction.  Products accumulate in float32
// (m16n8k16 mma.sync, two independent chains per unit); the fp16 scale of each 128-value group multiplies the
// unit's float32 partial (int8: the row scale multiplies the final sum).
//
// Fixed summation structure: the partial of an item is always formed by the same four-warp split, and the
// partials of a row's K ranges are added in range order.  The K ranges of a row block may be spread over the
// R CTAs of a thread-block cluster (rank j takes ranges j, j + R, ...); each CTA keeps its item partials in
// shared memory and, after one cluster barrier, the partials are added in range order through distributed
// shared memory.  R and the grid only decide who computes a partial, not how, so every launch shape -- and a
// column-sharded layer -- gives identical bits.  No global scratch memory is used.
//
// With programmatic dependent launch (static weights), the producer streams weights before the previous
// kernel on the stream has finished; only the activations and the output wait for it (griddepcontrol.wait).
//
// Box mode (template flag BOX): instead of one bulk copy per row, the producer fetches a whole item with ONE tensor copy of a
// 3-D box (64 bytes of a unit x 16 rows x 32 units) over the codes in their stored [N, K/2] layout, which lands
// in shared memory unit-major ([unit][row][64 B]: conflict-free 16-byte reads, no padding), plus, when the
// scale rows are 16-byte multiples (K % 1024 == 0), the item's 16 x 32 fp16 scales as a 2-D box.  Rows past N
// and units past the row are zero-filled by the copy and never read.  The arithmetic and its order are the same
// in both modes, so both give the same bits.
#include "lb_common.cuh"
#include "lb_kernels.h"
#include "lb_tmap.h"

namespace lb {

namespace gemv {
constexpr int RB = 16;                          // rows per row block (one m16 tile)
constexpr int UNIT = 64;                        // bytes of one row per unit
constexpr int RANGE_UNITS = 32;                 // units per K range (2 KB of codes per row)
constexpr int ROW_STRIDE = UNIT * RANGE_UNITS + 64;   // rows g and g+8 in different banks
constexpr int STAGE_BYTES = RB * ROW_STRIDE;    // 33792
constexpr int GW = 4;                           // warps per group
constexpr int UPW = RANGE_UNITS / GW;           // units per warp per item
constexpr int MAX_RANGES = 32;
constexpr int MAX_CLUSTER = 8;
constexpr int SMEM_LIMIT = 227 * 1024;
constexpr int HALF_SM_SMEM = 113 * 1024;        // two CTAs per SM
constexpr int MAX_SLOTS = 8;
constexpr int BOX_CODES = RB * RANGE_UNITS * UNIT;   // 32768: box mode, [unit][row][64 B]
constexpr int BOX_SCALES = RB * RANGE_UNITS * 2;     // 1024: box mode, fp16 [row][unit]
static_assert(BOX_CODES + BOX_SCALES <= STAGE_BYTES, "box mode item must fit a ring slot");
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
  int nr;                 // K ranges per row
  int R;                  // CTAs per cluster; rank j takes ranges j, j + R, ...
  int C;                  // clusters; cluster c takes row blocks c, c + C, ...
  int slots;              // ring slots
  int max_items;          // item partials per CTA (shared-memory table), 0 = outputs written directly
  OutRanks dst;           // column-sharded layer: every rank's output (dst.n == 0: y)
  const void* ln;         // RMSNorm weights [K] (float32 or bf16) of the norm prologue, or null
  int ln_f32, ln_vec;     // weights are float32; weights are 16-byte aligned
  float ln_eps, ln_off;
  int scale_tma;          // box mode: the item's scales come with it (tensor map `ts`)
  int pre;                // integer path: weight copies issued before the activations' loads are (all queued)
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
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// m16n8k16 bf16 tensor-core product, fp32 accumulate: d += a * b.
__device__ __forceinline__ void mma_bf16_16816_acc(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// int4 in bf16: one word (8 codes) -> four bf16 pairs 128 + n with n = q + 8 (exact: 8 significant bits):
// P0 = (n0, n4), P1 = (n1, n5), P2 = (n2, n6), P3 = (n3, n7).
__device__ __forceinline__ void deq4_word_bf16(uint32_t w, uint32_t (&P)[4]) {
  P[0] = lop3_and_xor_or(w, 0x000F000Fu, 0x43084308u);
  P[1] = lop3_and_xor_or(w >> 4, 0x000F000Fu, 0x43084308u);
  P[2] = lop3_and_xor_or(w >> 8, 0x000F000Fu, 0x43084308u);
  P[3] = lop3_and_xor_or(w >> 12, 0x000F000Fu, 0x43084308u);
}

// int8: one word (4 codes) -> two fp16 pairs 1024 + (n0, n2), 1024 + (n1, n3) with n = q + 128.
__device__ __forceinline__ void deq8_word(uint32_t w, uint32_t& q02, uint32_t& q13) {
  const uint32_t v = w ^ 0x80808080u;
  q02 = prmt(v, 0x00006464u, 0x5240u);
  q13 = prmt(v, 0x00006464u, 0x5341u);
}

// fp8 rows: one word (4 codes) -> the fp16 pairs (code 0, code 2), (code 1, code 3), exact.  e4m3 through the
// hardware conversion, e5m2 as the high byte of an fp16 (the two formats share exponent width and bias).
__device__ __forceinline__ uint32_t cvt_e4m3x2_f16x2(uint32_t lo16) {
  uint32_t d;
  asm("{\n\t.reg .b16 a;\n\tcvt.u16.u32 a, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, a;\n\t}" : "=r"(d) : "r"(lo16));
  return d;
}
template <int FMT>
__device__ __forceinline__ void deq_fp8_word(uint32_t w, uint32_t& q02, uint32_t& q13) {
  if (FMT == 5) {
    q02 = cvt_e4m3x2_f16x2(prmt(w, 0u, 0x0020u));
    q13 = cvt_e4m3x2_f16x2(prmt(w, 0u, 0x0031u));
  } else {
    q02 = prmt(w, 0u, 0x2404u);
    q13 = prmt(w, 0u, 0x3414u);
  }
}

// One unit (16 rows x 64 bytes of codes) against the B fragments of MT token tiles: acc += scale * (sum of
// exact code products).  `nc` holds minus the offset correction of the thread's two tokens per tile.
template <int FMT, int MT>
__device__ __forceinline__ void unit_mma(const uint4& w0, const uint4& w8, const uint32_t (&B)[MT][(FMT == 2 || FMT == 9) ? 16 : 8],
                                         const float (&nc)[MT][2], float s0, float s8, float (&acc)[MT][4]) {
  const uint32_t W0[4] = {w0.x, w0.y, w0.z, w0.w};
  const uint32_t W8[4] = {w8.x, w8.y, w8.z, w8.w};
  float c0[MT][4], c1[MT][4];       // two classes of K positions = two independent MMA chains
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    c0[t][0] = nc[t][0]; c0[t][1] = nc[t][1]; c0[t][2] = nc[t][0]; c0[t][3] = nc[t][1];
    c1[t][0] = c1[t][1] = c1[t][2] = c1[t][3] = 0.f;
  }
  if (FMT == 2) {
    // bf16 codes 136 + q against the bf16 activations: exact products, two independent chains
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t P0[4], P8[4];
      deq4_word_bf16(W0[i], P0);
      deq4_word_bf16(W8[i], P8);
      const uint32_t ae[4] = {P0[0], P8[0], P0[2], P8[2]};   // nibbles (0,4) | (2,6)
      const uint32_t ao[4] = {P0[1], P8[1], P0[3], P8[3]};   // nibbles (1,5) | (3,7)
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        mma_bf16_16816_acc(c0[t], ae, B[t][4 * i + 0], B[t][4 * i + 1]);
        mma_bf16_16816_acc(c1[t], ao, B[t][4 * i + 2], B[t][4 * i + 3]);
      }
    }
  } else if (FMT == 9) {
    // fp4: natural code pairs against the activations staged in natural order (fp16, 2^-e per range)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t P0[4], P8[4];
      deq_fp4_word(W0[i], P0);
      deq_fp4_word(W8[i], P8);
      const uint32_t a0[4] = {P0[0], P8[0], P0[1], P8[1]};   // codes (0,1) | (2,3)
      const uint32_t a1[4] = {P0[2], P8[2], P0[3], P8[3]};   // codes (4,5) | (6,7)
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        mma_f16_16816(c0[t], a0, B[t][4 * i + 0], B[t][4 * i + 1]);
        mma_f16_16816(c1[t], a1, B[t][4 * i + 2], B[t][4 * i + 3]);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t a[4];
      if (FMT == 1) {
        deq8_word(W0[i], a[0], a[2]);
        deq8_word(W8[i], a[1], a[3]);
      } else {
        deq_fp8_word<FMT>(W0[i], a[0], a[2]);
        deq_fp8_word<FMT>(W8[i], a[1], a[3]);
      }
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        if (i & 1) mma_f16_16816(c1[t], a, B[t][2 * i], B[t][2 * i + 1]);
        else mma_f16_16816(c0[t], a, B[t][2 * i], B[t][2 * i + 1]);
      }
    }
  }
  const float k1 = 1.0f;
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    acc[t][0] = fmaf(fmaf(c1[t][0], k1, c0[t][0]), s0, acc[t][0]);
    acc[t][1] = fmaf(fmaf(c1[t][1], k1, c0[t][1]), s0, acc[t][1]);
    acc[t][2] = fmaf(fmaf(c1[t][2], k1, c0[t][2]), s8, acc[t][2]);
    acc[t][3] = fmaf(fmaf(c1[t][3], k1, c0[t][3]), s8, acc[t][3]);
  }
}

// m16n8k32 product of unsigned 8-bit A and signed 8-bit B, int32 accumulate: d += a * b.
__device__ __forceinline__ void mma_u8s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// (a ^ b) & c
__device__ __forceinline__ uint32_t lop3_xor_and(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x28;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// int4 unit on the integer tensor path: codes as unsigned bytes q + 8 (one LOP3 per four), activations as two
// signed 8-bit digits of a 2^e-scaled int16 (hi in column 2t, lo in column 2t + 1 of the n8 tile), exact int32
// products; `nc` starts the accumulation at -8 * sum(digits) (the offset correction), `f` is 2^e of the thread's
// token.  Output: acc[T][0] (row g) and acc[T][1] (row g + 8) for token 4T + c.
template <int NT>
__device__ __forceinline__ void unit_i8(const uint4& w0, const uint4& w8, const uint32_t (&B)[NT][8],
                                        const int (&nc)[NT][2], const float (&f)[NT], float s0, float s8,
                                        float (&acc)[NT][2]) {
  const uint32_t W0[4] = {w0.x, w0.y, w0.z, w0.w};
  const uint32_t W8[4] = {w8.x, w8.y, w8.z, w8.w};
  uint32_t A[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    A[i][0] = lop3_xor_and(W0[i], 0x88888888u, 0x0F0F0F0Fu);          // row g, even positions
    A[i][1] = lop3_xor_and(W8[i], 0x88888888u, 0x0F0F0F0Fu);          // row g + 8
    A[i][2] = lop3_xor_and(W0[i] >> 4, 0x08080808u, 0x0F0F0F0Fu);     // row g, odd positions
    A[i][3] = lop3_xor_and(W8[i] >> 4, 0x08080808u, 0x0F0F0F0Fu);
  }
#pragma unroll
  for (int T = 0; T < NT; ++T) {
    int da[4] = {-nc[T][0], -nc[T][1], -nc[T][0], -nc[T][1]};
    int db[4] = {0, 0, 0, 0};
    mma_u8s8(da, A[0], B[T][0], B[T][1]);
    mma_u8s8(db, A[1], B[T][2], B[T][3]);
    mma_u8s8(da, A[2], B[T][4], B[T][5]);
    mma_u8s8(db, A[3], B[T][6], B[T][7]);
    const int v0 = (da[0] + db[0]) * 256 + (da[1] + db[1]);
    const int v8 = (da[2] + db[2]) * 256 + (da[3] + db[3]);
    acc[T][0] = fmaf(static_cast<float>(v0), s0 * f[T], acc[T][0]);
    acc[T][1] = fmaf(static_cast<float>(v8), s8 * f[T], acc[T][1]);
  }
}

// The same unit with fewer instructions: the codes of the even positions become bytes q + 8 and those of the
// odd positions bytes 16 (q + 8), each with ONE LOP3 and no shift, so the MMAs are regrouped by position
// class -- ae takes the even positions of two words at a time, ao the odd ones (scaled by 16) -- against the
// same staged B fragments.  ae + ao / 16 is the exact integer unit_i8 forms, and v = 256 hi + lo is formed from
// 16 v (exact, |16 v| < 2^31) with one arithmetic shift, so `acc` gets the same bits.  `sf` is s * 2^e of the
// unit (0 for a unit past the row: its finite garbage then adds exactly nothing).
__device__ __forceinline__ void unit_i8_lean(const uint4& w0, const uint4& w8, const uint4& b0, const uint4& b1,
                                             int nc0, int nc1, float sf0, float sf8, float& acc0, float& acc8) {
  const uint32_t W0[4] = {w0.x ^ 0x88888888u, w0.y ^ 0x88888888u, w0.z ^ 0x88888888u, w0.w ^ 0x88888888u};
  const uint32_t W8[4] = {w8.x ^ 0x88888888u, w8.y ^ 0x88888888u, w8.z ^ 0x88888888u, w8.w ^ 0x88888888u};
  int ae[4] = {-nc0, -nc1, -nc0, -nc1};
  int ao[4] = {0, 0, 0, 0};
  {
    const uint32_t e[4] = {W0[0] & 0x0F0F0F0Fu, W8[0] & 0x0F0F0F0Fu, W0[1] & 0x0F0F0F0Fu, W8[1] & 0x0F0F0F0Fu};
    const uint32_t o[4] = {W0[0] & 0xF0F0F0F0u, W8[0] & 0xF0F0F0F0u, W0[1] & 0xF0F0F0F0u, W8[1] & 0xF0F0F0F0u};
    mma_u8s8(ae, e, b0.x, b0.z);
    mma_u8s8(ao, o, b0.y, b0.w);
  }
  {
    const uint32_t e[4] = {W0[2] & 0x0F0F0F0Fu, W8[2] & 0x0F0F0F0Fu, W0[3] & 0x0F0F0F0Fu, W8[3] & 0x0F0F0F0Fu};
    const uint32_t o[4] = {W0[2] & 0xF0F0F0F0u, W8[2] & 0xF0F0F0F0u, W0[3] & 0xF0F0F0F0u, W8[3] & 0xF0F0F0F0u};
    mma_u8s8(ae, e, b1.x, b1.z);
    mma_u8s8(ao, o, b1.y, b1.w);
  }
  const int v0 = ((ae[0] * 16 + ao[0]) * 256 + (ae[1] * 16 + ao[1])) >> 4;
  const int v8 = ((ae[2] * 16 + ao[2]) * 256 + (ae[3] * 16 + ao[3])) >> 4;
  acc0 = fmaf(static_cast<float>(v0), sf0, acc0);
  acc8 = fmaf(static_cast<float>(v8), sf8, acc8);
}

// Shared-memory carve-up, in bytes from the base of dynamic shared memory.
struct GemvSmem {
  int ring, xs, corr, xsc, gred, ptab, zeros, bars, lnf, total;
  int token_stride;   // bytes of one token's staged activations
};

// xs_units: units of x this CTA stages (its ranges x 32); items: entries of the partial table
__host__ __device__ inline GemvSmem gemv_smem(int fmt, int M, int MT, int G, int xs_units, int slots, int items) {
  using namespace gemv;
  GemvSmem s;
  const int xu = (fmt == 2 || fmt == 20 || fmt == 9) ? 256 : 128;     // staged bytes of x per unit per token
  s.token_stride = xs_units * xu + 64;
  s.ring = 0;
  s.xs = slots * STAGE_BYTES;                                  // multiple of 128
  s.corr = s.xs + ((M * s.token_stride + 127) & ~127);
  s.xsc = s.corr + ((M * xs_units * (fmt == 20 ? 12 : 4) + 127) & ~127);   // int core: int2 + 2^e; else float
  s.gred = s.xsc + (fmt == 20 ? 0 : 2 * 16 * MAX_RANGES * 4);  // xsc + xmax (unused on the integer path)
  s.ptab = s.gred + G * 2 * GW * 32 * (fmt == 20 ? 2 : 4) * MT * 4;   // double-buffered group partials
  s.zeros = s.ptab + ((items * 16 * M * 4 + 127) & ~127);
  s.bars = s.zeros + 256;                                      // 256 zero bytes (absent tokens)
  s.lnf = s.bars + 2 * MAX_SLOTS * 8 + 32;                    // [16] RMSNorm factors per token
  s.total = s.lnf + 64;
  return s;
}

__host__ __device__ inline int ranges_of_rank(int nr, int R, int j) { return j < nr ? (nr - j + R - 1) / R : 0; }

__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Epilogue of one output: int8 row scale, bias, accumulate, bf16 store.
template <int FMT>
__device__ __forceinline__ void store_out(const GemvParams& p, int64_t n, int tok, float v) {
  if (FMT == 1) v *= __half2float(p.s16[n]);
  if (FMT >= 5 && FMT <= 9) v *= reinterpret_cast<const float*>(p.s16)[n];   // minifloat rows: float32 scales
  if (p.bias) v += bf16_bits_to_f32(p.bias[n]);
  if (p.dst.n) {                            // this rank's column of every rank's output
    const uint16_t b = f32_to_bf16_bits(v);
    const int64_t off = static_cast<int64_t>(tok) * p.ldy + p.dst.col0 + n;
#pragma unroll
    for (int g = 0; g < kMaxRanks; ++g)     // constant indices: no dynamic indexing of the parameters
      if (g < p.dst.n) p.dst.y[g][off] = b;
    return;
  }
  uint16_t* yp = p.y + static_cast<int64_t>(tok) * p.ldy + n;
  if (p.acc) v += bf16_bits_to_f32(*yp);
  *yp = f32_to_bf16_bits(v);
}

template <int FMT, int MT, int G, int MINB, bool BOX, bool LR = false>
__global__ void __launch_bounds__((G * gemv::GW + 1) * 32, MINB)
    gemv_kernel(const GemvParams p, const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap ts) {
  using namespace gemv;
  constexpr int NCW = G * GW;                  // consumer warps
  constexpr int CT = NCW * 32;                 // consumer threads
  constexpr bool I4 = (FMT == 2 || FMT == 20);   // int4 codes (20: on the integer tensor path)
  constexpr bool NIB = I4 || FMT == 9;           // 4-bit codes: 128 values per 64-byte unit
  constexpr int XU = NIB ? 256 : 128;           // staged bytes of x per unit per token
  constexpr int XCH = XU / 64;                 // 16-byte chunks of x per thread per unit
  constexpr int KPU = NIB ? 128 : 64;           // K values per unit
  constexpr int CPU = KPU / 8;                 // 16-byte chunks of x per unit
  constexpr int CPR = RANGE_UNITS * CPU;       // 16-byte chunks of x per range
  constexpr int PW = (FMT == 20) ? 2 : 4;      // partial floats per lane per token tile
  extern __shared__ __align__(1024) uint8_t dyn_smem[];

  const int R = p.R;
  const int rank = R > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int cid = blockIdx.x / R;
  const int nloc = ranges_of_rank(p.nr, R, rank);              // K ranges of this CTA
  const int nmine = cid < p.nblocks ? (p.nblocks - cid + p.C - 1) / p.C : 0;   // row blocks of the cluster
  const int nq = nmine * nloc;                                 // items of this CTA
  // the layout is the same in every CTA of a cluster (the partial tables are read remotely at one offset)
  const GemvSmem L = gemv_smem(FMT, p.M, MT, G, ranges_of_rank(p.nr, R, 0) * RANGE_UNITS, p.slots, p.max_items);
  uint8_t* ring = dyn_smem + L.ring;
  uint8_t* xs = dyn_smem + L.xs;
  float* corr = reinterpret_cast<float*>(dyn_smem + L.corr);   // [M][nloc * 32] offset corrections
  float* xsc = reinterpret_cast<float*>(dyn_smem + L.xsc);     // [16 tokens][MAX_RANGES] 2^e factors
  int* xmax = reinterpret_cast<int*>(xsc + 16 * MAX_RANGES);   // [16 tokens][MAX_RANGES] absmax bits
  float* gred = reinterpret_cast<float*>(dyn_smem + L.gred);   // [G][2][GW][32][4 * MT] warp partials
  float* ptab = reinterpret_cast<float*>(dyn_smem + L.ptab);   // [items][16 * M] item partials
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(dyn_smem + L.bars);
  uint64_t* empty_bar = full_bar + MAX_SLOTS;
  volatile int* abort_v = reinterpret_cast<int*>(empty_bar + MAX_SLOTS);
  uint64_t* x_bar = empty_bar + MAX_SLOTS + 2;                 // every consumer warp has issued its x loads
  const int units_staged = nloc * RANGE_UNITS;
  const int slots = p.slots;   // a multiple of G: group g owns slots g, g + G, ...
  // Item q belongs to group q % G and uses that group's slots in turn, so every slot is used by one group, in
  // item order, and a waiter is never more than one phase of a slot's mbarriers ahead (parity waits are exact).
  auto ring_slot = [](int q, int S) { return (q % G) + G * ((q / G) % (S / G)); };
  const bool direct = p.max_items == 0;                        // one range per row, one CTA per cluster

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t row_bytes = NIB ? p.K / 2 : p.K;

  if (threadIdx.x == 0) {
    for (int s = 0; s < slots; ++s) { mbar_init(&full_bar[s], 1); mbar_init(&empty_bar[s], GW); }
    mbar_init(x_bar, NCW);
    *abort_v = 0;
    fence_barrier_init();
  }
  if (FMT != 20)
    for (int i = threadIdx.x; i < 16 * MAX_RANGES; i += blockDim.x) xmax[i] = 0;
  for (int i = threadIdx.x; i < 64; i += blockDim.x) reinterpret_cast<uint32_t*>(dyn_smem + L.zeros)[i] = 0u;
  __syncthreads();
  pdl_launch_dependents();

  if (warp == NCW) {
    // ------------------------------------------------------------------ producer warp
    // lane 0 registers the byte count, lanes 0..15 copy one row each; the weights do not depend on earlier
    // kernels, so streaming starts before griddepcontrol.wait
    const uint64_t wpol = l2_policy_evict_first();   // the weights are read once
    if (BOX && lane == 0) {
      prefetch_tmap(&tw);
      if (p.scale_tma) prefetch_tmap(&ts);
    }
    for (int q = 0; q < nq && !*abort_v; ++q) {
      // the integer path's activations are loaded after griddepcontrol.wait; copies issued before those
      // loads would be served first, so past the first `pre` items the stream waits until they are queued
      if (FMT == 20 && q == p.pre) mbar_wait(x_bar, 0, abort_v);
      const int k = q / nloc, i = q - k * nloc;
      const int64_t row0 = static_cast<int64_t>(cid + k * p.C) * RB;
      const int rows_valid = static_cast<int>(p.N - row0 < RB ? p.N - row0 : RB);
      const int u0 = (rank + i * R) * RANGE_UNITS;
      const uint32_t bytes_row = static_cast<uint32_t>(min(p.total_units - u0, RANGE_UNITS) * UNIT);
      const int slot = ring_slot(q, slots);
      if (q >= slots) mbar_wait(&empty_bar[slot], ((q / slots) - 1) & 1, abort_v);
      if (BOX) {                            // one box per item: codes [unit][row][64 B] (+ scales [row][unit])
        if (lane == 0) {
          uint8_t* dst = ring + slot * STAGE_BYTES;
          mbar_arrive_expect_tx(&full_bar[slot], BOX_CODES + (p.scale_tma ? BOX_SCALES : 0));
          tma_load_3d_hint(dst, &tw, 0, static_cast<int>(row0), u0, &full_bar[slot], wpol);
          if (p.scale_tma) tma_load_2d(dst + BOX_CODES, &ts, u0, static_cast<int>(row0), &full_bar[slot]);
        }
        __syncwarp();
        continue;
      }
      if (lane == 0) mbar_arrive_expect_tx(&full_bar[slot], bytes_row * rows_valid);
      __syncwarp();
      if (lane < rows_valid)
        bulk_g2s_hint(ring + slot * STAGE_BYTES + lane * ROW_STRIDE,
                      p.w + (row0 + lane) * row_bytes + static_cast<int64_t>(u0) * UNIT, bytes_row, &full_bar[slot],
                      wpol);
    }
  } else {
    // ------------------------------------------------------------------ consumers
    pdl_wait();                             // the activations (and the output) come from earlier kernels
    const int ctid = threadIdx.x;
    float* lnf = reinterpret_cast<float*>(dyn_smem + L.lnf);
    if (p.ln) {
      // norm prologue: one warp per token reduces the whole row (every K range) in the order of lb_rmsnorm
      for (int t = warp; t < p.M; t += NCW) {
        const float f = rms_row_factor_warp(p.x + static_cast<int64_t>(t) * p.K, p.K, p.ln_eps, true);
        if (lane == 0) lnf[t] = f;
      }
      named_sync(1, CT);
    }
    // Stage the activations of this CTA's ranges: per (token, range) power-of-two factor, fp16, B-fragment
    // order, and the offset correction per (token, unit).  Pass 1 loads XB chunks per thread at a time, parks
    // each raw chunk in its final slot and takes the absmax per (token, range); pass 2 converts the chunks in
    // place.  Chunk q is handled by consumer thread q % CT in both passes; the chunks of one unit sit in CPU
    // consecutive lanes and their class sums are added with a fixed shuffle tree.
    {
      constexpr int XB = MT == 1 ? 4 : 8;        // chunks per thread in flight
      const int cpt = nloc * CPR;                              // chunks per token (multiple of 32)
      const int nch = p.M * cpt;
      // chunk q -> (token, local range, chunk within range); invalid past the end of the row
      auto locate = [&](int q, int& t, int& il, int& jj, int& r) {
        t = q / cpt;
        const int j = q - t * cpt;
        il = j / CPR;
        jj = j - il * CPR;
        r = rank + il * R;
        return q < nch && r * RANGE_UNITS + jj / CPU < p.total_units;
      };
      auto slot_of = [&](int t, int il, int jj) -> uint8_t* {
        int u, cc, vv;
        if (NIB) { u = jj >> 4; cc = (jj >> 2) & 3; vv = jj & 3; }
        else { u = jj >> 3; cc = (jj >> 1) & 3; vv = jj & 1; }
        return xs + t * L.token_stride + (il * RANGE_UNITS + u) * XU + vv * 64 + cc * 16;
      };
      if (FMT == 2) {
        // int4: the bf16 activations are used as they are (the bf16 products are exact), permuted into the
        // B-fragment order; one pass, the offset correction 136 * sum(x) per (token, unit)
        for (int base = 0; base < nch; base += CT * XB) {
          uint4 v[XB];
          RmsW wv[XB];
#pragma unroll
          for (int b = 0; b < XB; ++b) {
            int t, il, jj, r;
            v[b] = make_uint4(0u, 0u, 0u, 0u);
            if (locate(base + b * CT + ctid, t, il, jj, r)) {
              const int64_t k0 = static_cast<int64_t>(r) * RANGE_UNITS * KPU + jj * 8;
              v[b] = ldg_nc_v4(p.x + static_cast<int64_t>(t) * p.K + k0);
              if (p.ln) wv[b] = rms_load_w(p.ln, p.ln_f32 != 0, k0, p.K, p.ln_vec != 0);
            }
          }
          if (p.ln) {                            // norm prologue: bf16((x * fac) * (w + off)), as lb_rmsnorm
#pragma unroll
            for (int b = 0; b < XB; ++b) {
              int t, il, jj, r;
              if (locate(base + b * CT + ctid, t, il, jj, r)) v[b] = rms_apply_chunk(v[b], lnf[t], wv[b], p.ln_f32 != 0, p.ln_off);
            }
          }
#pragma unroll
          for (int b = 0; b < XB; ++b) {
            const int q = base + b * CT + ctid;
            int t, il, jj, r;
            const bool ok = locate(q, t, il, jj, r);
            float sum = 0.f;
            if (ok) {
              // (x0,x4) (x2,x6) (x1,x5) (x3,x7), matching the code pairs of deq4_word_bf16
              const uint32_t o0 = prmt(v[b].x, v[b].z, 0x5410u), o1 = prmt(v[b].y, v[b].w, 0x5410u);
              const uint32_t o2 = prmt(v[b].x, v[b].z, 0x7632u), o3 = prmt(v[b].y, v[b].w, 0x7632u);
              *reinterpret_cast<uint4*>(slot_of(t, il, jj)) = make_uint4(o0, o1, o2, o3);
              auto lo = [](uint32_t u) { return __uint_as_float(u << 16); };
              auto hi = [](uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); };
              sum = ((lo(o0) + hi(o0)) + (lo(o1) + hi(o1))) + ((lo(o2) + hi(o2)) + (lo(o3) + hi(o3)));
              if (jj == 0) xsc[t * MAX_RANGES + r] = 1.0f;
            }
#pragma unroll
            for (int o2 = CPU / 2; o2 >= 1; o2 >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o2);
            if (ok && (jj % CPU) == 0) corr[t * units_staged + il * RANGE_UNITS + jj / CPU] = 136.f * sum;
          }
        }
        named_sync(1, CT);
      } else if (FMT == 20) {
        // int4 on the integer path: per (token, unit) e with max|x| * 2^-e in [2^13, 2^14), x16 = rint(x * 2^-e), split into signed
        // bytes hi = (x16 + 128) >> 8 and lo = x16 - 256 hi, written in the B-fragment order of the m16n8k32
        // tiles (column 2t: hi, 2t + 1: lo of token t); the offset correction 8 * sum(digit) per (token, unit).
        // One half-warp per (token, unit): lane j of the half takes the unit's 16-byte chunk j, so the unit's
        // absmax and digit sums are 4-step shuffle trees inside the half.  A warp issues the loads of its pairs
        // of SB passes before any arithmetic, and a pass with no pair for the warp is skipped (this path runs
        // for M <= 2, where a CTA stages at most 2 x 32 units per K range).
        int* corr_i = reinterpret_cast<int*>(corr);                       // [M][units][2]
        float* fac = corr + 2 * p.M * units_staged;                       // [M][units] 2^e
        constexpr int PPI = 2 * NCW;                                      // pairs per pass: two per warp
        constexpr int SB = 2;                                             // passes with loads in flight together
        const int npair = p.M * units_staged;
        const int j = lane & 15;
        if (2 * warp >= npair && lane == 0) mbar_arrive(x_bar);        // no pair for this warp
        for (int base = 2 * warp; base < npair; base += PPI * SB) {      // warp-uniform
          uint4 v[SB];
          RmsW wv[SB];
          int tv[SB], ilv[SB], jjv[SB];
          bool okv[SB];
#pragma unroll
          for (int b = 0; b < SB; ++b) {
            const int pi = base + b * PPI + (lane >> 4);
            int t = 0, uloc = pi;
            while (uloc >= units_staged) { uloc -= units_staged; ++t; }
            const int il = uloc / RANGE_UNITS, u = uloc % RANGE_UNITS;
            const int r = rank + il * R;
            tv[b] = t; ilv[b] = il; jjv[b] = u * CPU + j;
            okv[b] = pi < npair && r * RANGE_UNITS + u < p.total_units;
            v[b] = make_uint4(0u, 0u, 0u, 0u);
            if (okv[b]) {
              const int64_t k0 = static_cast<int64_t>(r) * RANGE_UNITS * KPU + jjv[b] * 8;
              v[b] = ldg_nc_v4(p.x + static_cast<int64_t>(t) * p.K + k0);
              if (p.ln) wv[b] = rms_load_w(p.ln, p.ln_f32 != 0, k0, p.K, p.ln_vec != 0);
            }
          }
          if (base == 2 * warp) {                // this warp's first loads are issued
            __syncwarp();
            if (lane == 0) mbar_arrive(x_bar);
          }
          if (p.ln) {                            // norm prologue: bf16((x * fac) * (w + off)), as lb_rmsnorm
#pragma unroll
            for (int b = 0; b < SB; ++b)
              if (okv[b]) v[b] = rms_apply_chunk(v[b], lnf[tv[b]], wv[b], p.ln_f32 != 0, p.ln_off);
          }
#pragma unroll
          for (int b = 0; b < SB; ++b) {
            if (base + b * PPI >= npair) break;                           // warp-uniform
            const int t = tv[b], il = ilv[b], jj = jjv[b];
            const bool ok = okv[b];
            const uint32_t rr[4] = {v[b].x, v[b].y, v[b].z, v[b].w};
            float xf[8];
#pragma unroll
            for (int e2 = 0; e2 < 4; ++e2) {
              xf[2 * e2] = __uint_as_float(rr[e2] << 16);
              xf[2 * e2 + 1] = __uint_as_float(rr[e2] & 0xFFFF0000u);
            }
            float m = 0.f;
#pragma unroll
            for (int e2 = 0; e2 < 8; ++e2) m = fmaxf(m, fabsf(xf[e2]));
#pragma unroll
            for (int o2 = CPU / 2; o2 >= 1; o2 >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o2));
            int e = 0;
            if (m > 0.f) {
              int ex;
              frexpf(m, &ex);
              e = min(max(ex - 14, -126), 114);
            }
            const float down = __int_as_float((127 - e) << 23);            // 2^-e, exact
            int hd[8], ld[8], sh = 0, sl = 0;
#pragma unroll
            for (int e2 = 0; e2 < 8; ++e2) {
              const int x16 = __float2int_rn(xf[e2] * down);
              hd[e2] = (x16 + 128) >> 8;
              ld[e2] = x16 - (hd[e2] << 8);
              sh += hd[e2];
              sl += ld[e2];
            }
            auto pack4 = [](int a, int b2, int c2, int d) {
              return prmt(prmt(static_cast<uint32_t>(a), static_cast<uint32_t>(b2), 0x0040u),
                          prmt(static_cast<uint32_t>(c2), static_cast<uint32_t>(d), 0x0040u), 0x5410u);
            };
            if (ok) {
              const int uloc = il * RANGE_UNITS + (jj >> 4);
              const int jc = jj & 15, cq = jc >> 2, i = jc & 3;
              const int T = t >> 2, tt = t & 3;
              const int ncols = min(8, 2 * p.M - 8 * T);
              uint8_t* base_p = xs + T * units_staged * 1024 + uloc * (ncols * 128) + (i >> 1) * (ncols * 64) +
                                cq * 16 + (i & 1) * 8;
              *reinterpret_cast<uint2*>(base_p + (2 * tt) * 64) =
                  make_uint2(pack4(hd[0], hd[2], hd[4], hd[6]), pack4(hd[1], hd[3], hd[5], hd[7]));
              *reinterpret_cast<uint2*>(base_p + (2 * tt + 1) * 64) =
                  make_uint2(pack4(ld[0], ld[2], ld[4], ld[6]), pack4(ld[1], ld[3], ld[5], ld[7]));
            }
            // both digit sums in one word: |sum hi| < 2^13 and |sum lo| < 2^15 over a unit, so
            // 65536 sh + sl adds without overflow and its low half is sum lo as a signed 16-bit value
            int both = sh * 65536 + sl;
#pragma unroll
            for (int o2 = CPU / 2; o2 >= 1; o2 >>= 1) both += __shfl_xor_sync(0xffffffffu, both, o2);
            if (ok && (jj & 15) == 0) {
              const int uloc = il * RANGE_UNITS + (jj >> 4);
              const int slo = static_cast<int16_t>(both & 0xFFFF);
              const int shi = (both - slo) / 65536;
              corr_i[(t * units_staged + uloc) * 2] = 8 * shi;
              corr_i[(t * units_staged + uloc) * 2 + 1] = 8 * slo;
              fac[t * units_staged + uloc] = __int_as_float((127 + e) << 23);   // 2^e
            }
          }
        }
        named_sync(1, CT);
      } else {
      for (int base = 0; base < nch; base += CT * XB) {        // pass 1
          uint4 v[XB];
          RmsW wv[XB];
  #pragma unroll
          for (int b = 0; b < XB; ++b) {
            int t, il, jj, r;
            v[b] = make_uint4(0u, 0u, 0u, 0u);
            if (locate(base + b * CT + ctid, t, il, jj, r)) {
              const int64_t k0 = static_cast<int64_t>(r) * RANGE_UNITS * KPU + jj * 8;
              v[b] = ldg_nc_v4(p.x + static_cast<int64_t>(t) * p.K + k0);
              if (p.ln) wv[b] = rms_load_w(p.ln, p.ln_f32 != 0, k0, p.K, p.ln_vec != 0);
            }
          }
          if (p.ln) {                            // norm prologue: bf16((x * fac) * (w + off)), as lb_rmsnorm
#pragma unroll
            for (int b = 0; b < XB; ++b) {
              int t, il, jj, r;
              if (locate(base + b * CT + ctid, t, il, jj, r)) v[b] = rms_apply_chunk(v[b], lnf[t], wv[b], p.ln_f32 != 0, p.ln_off);
            }
          }
  #pragma unroll
          for (int b = 0; b < XB; ++b) {
            const int q = base + b * CT + ctid;
            int t, il, jj, r;
            const bool ok = locate(q, t, il, jj, r);
            if (ok) *reinterpret_cast<uint4*>(slot_of(t, il, jj)) = v[b];
            const uint32_t rr[4] = {v[b].x, v[b].y, v[b].z, v[b].w};
            float m = 0.f;
  #pragma unroll
            for (int e = 0; e < 4; ++e)
              m = fmaxf(m, fmaxf(fabsf(__uint_as_float(rr[e] << 16)), fabsf(__uint_as_float(rr[e] & 0xFFFF0000u))));
            // a warp's 32 chunks lie in one (token, range)
  #pragma unroll
            for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane == 0 && ok && m > 0.f)   // non-negative floats order like their bit patterns
              atomicMax(&xmax[t * MAX_RANGES + r], static_cast<int>(__float_as_uint(m)));
          }
        }
        named_sync(1, CT);
        for (int q = ctid; q < ((nch + 31) & ~31); q += CT) {   // pass 2
          float se = 0.f, so = 0.f;
          int t, il, jj, r;
          const bool valid = locate(q, t, il, jj, r);
          if (valid) {
            const float m = __uint_as_float(static_cast<uint32_t>(xmax[t * MAX_RANGES + r]));
            int e = 0;
            if (m > 0.f) {
              int ex;
              frexpf(m, &ex);
              e = min(max(ex - 15, -110), 110);               // max |x| * 2^-e in [2^14, 2^15)
            }
            if (jj == 0) xsc[t * MAX_RANGES + r] = ldexpf(1.0f, e);
            const float down = ldexpf(1.0f, -e);
            uint4* dst = reinterpret_cast<uint4*>(slot_of(t, il, jj));
            const uint4 v = *dst;
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
            } else if (FMT == 9) {   // fp4: natural order (the code pairs of deq_fp4_word)
#pragma unroll
              for (int e2 = 0; e2 < 8; ++e2) g8[e2] = f[e2];
            } else {          // byte pairs (0,2) (1,3) of each word
              g8[0] = f[0]; g8[1] = f[2]; g8[2] = f[1]; g8[3] = f[3]; g8[4] = f[4]; g8[5] = f[6]; g8[6] = f[5]; g8[7] = f[7];
            }
            uint32_t o[4];
  #pragma unroll
            for (int e2 = 0; e2 < 4; ++e2) {
              __half2 h = __floats2half2_rn(g8[2 * e2], g8[2 * e2 + 1]);
              o[e2] = *reinterpret_cast<uint32_t*>(&h);
            }
            // the values are exact in fp16, so the class sums use the converted values
            se = (g8[0] + g8[1]) + (g8[2] + g8[3]);
            so = (g8[4] + g8[5]) + (g8[6] + g8[7]);
            if (FMT == 1) { se += so; so = 0.f; }
            *dst = make_uint4(o[0], o[1], o[2], o[3]);
          }
          // class sums of a unit: its CPU consecutive lanes, fixed shuffle tree
  #pragma unroll
          for (int o2 = CPU / 2; o2 >= 1; o2 >>= 1) {
            se += __shfl_xor_sync(0xffffffffu, se, o2);
            so += __shfl_xor_sync(0xffffffffu, so, o2);
          }
          if (valid && (jj % CPU) == 0)
            corr[t * units_staged + il * RANGE_UNITS + jj / CPU] =
                (FMT == 2) ? fmaf(1032.f, se, 72.f * so) : (FMT == 1 ? 1152.f * se : 0.f);   // fp8: no offset
        }
        named_sync(1, CT);
      }
      }

    // ------------------------------------------------------------------ stream, dequantise, multiply
    const int grp = warp / GW;    // group
    const int gw = warp % GW;     // warp within the group
    const int g = lane >> 2;      // row and token within the m16n8 tile
    const int c = lane & 3;
    uint32_t xrow[MT];
    bool tok_ok[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      tok_ok[t] = t * 8 + g < p.M;
      xrow[t] = smem_u32(xs) + (t * 8 + g) * L.token_stride + c * 16;
    }
    const uint32_t zbase = smem_u32(dyn_smem + L.zeros);
    const uint32_t ring_base = smem_u32(ring) + c * 16;
    const int64_t ng = p.K / 128;
    for (int q = grp, n_it = 0; q < nq; q += G, ++n_it) {
      const int k = q / nloc, il = q - k * nloc;
      const int r = rank + il * R;
      const int64_t row0 = static_cast<int64_t>(cid + k * p.C) * RB;
      const int u0 = r * RANGE_UNITS;
      const int uend = min(u0 + RANGE_UNITS, p.total_units);
      const int64_t rg = row0 + g < p.N ? row0 + g : p.N - 1;
      const int64_t rg8 = row0 + g + 8 < p.N ? row0 + g + 8 : p.N - 1;
      // scales first (their latency overlaps the wait for the codes); in box mode with scale boxes they
      // arrive with the codes
      const bool sc_in_slot = BOX && p.scale_tma;
      float sc[UPW][2];
#pragma unroll
      for (int h = 0; h < UPW; ++h) {
        sc[h][0] = sc[h][1] = 1.f;
        const int uu = u0 + gw + h * GW;
        if (I4 && uu < uend && !sc_in_slot) {
          sc[h][0] = __half2float(__ldg(p.s16 + rg * ng + uu));
          sc[h][1] = __half2float(__ldg(p.s16 + rg8 * ng + uu));
        }
      }
      const int slot = ring_slot(q, slots);
      mbar_wait(&full_bar[slot], (q / slots) & 1, abort_v);
      const uint32_t sbuf = ring_base + slot * STAGE_BYTES;
      // all of this warp's codes of the item go to registers, then the slot is released at once (LR: the codes
      // are read from the slot unit by unit and the slot is released after the multiply)
      constexpr bool HOLD = BOX && LR && FMT == 20;
      uint4 wr[HOLD ? 1 : UPW][2];
      const uint32_t code_base = sbuf + g * UNIT;          // box mode: unit j's row g at j * 1024 + g * 64
      if constexpr (HOLD) {
        const uint32_t sscale = smem_u32(ring) + slot * STAGE_BYTES + BOX_CODES;
#pragma unroll
        for (int h = 0; h < UPW; ++h) {
          const int j = gw + h * GW;
          if (sc_in_slot && u0 + j < uend) {
            __half_raw h0, h8;
            h0.x = static_cast<unsigned short>(lds_u16(sscale + (g * RANGE_UNITS + j) * 2));
            h8.x = static_cast<unsigned short>(lds_u16(sscale + ((g + 8) * RANGE_UNITS + j) * 2));
            sc[h][0] = __half2float(__half(h0));
            sc[h][1] = __half2float(__half(h8));
          }
        }
      } else if constexpr (BOX) {
        // [unit][row][64 B]: unit j's row g at j * 1024 + g * 64 (ring_base already adds c * 16)
        const uint32_t sb = sbuf;
        const uint32_t sscale = smem_u32(ring) + slot * STAGE_BYTES + BOX_CODES;
#pragma unroll
        for (int h = 0; h < UPW; ++h) {
          const int j = gw + h * GW;
          const uint32_t a = sb + j * (RB * UNIT) + g * UNIT;
          wr[h][0] = lds_v4(a);
          wr[h][1] = lds_v4(a + 8 * UNIT);
          if (I4 && sc_in_slot && u0 + j < uend) {
            __half_raw h0, h8;
            h0.x = static_cast<unsigned short>(lds_u16(sscale + (g * RANGE_UNITS + j) * 2));
            h8.x = static_cast<unsigned short>(lds_u16(sscale + ((g + 8) * RANGE_UNITS + j) * 2));
            sc[h][0] = __half2float(__half(h0));
            sc[h][1] = __half2float(__half(h8));
          }
        }
      } else {
#pragma unroll
      for (int h = 0; h < UPW; ++h) {
        const int uu = u0 + gw + h * GW;
        if (uu < uend) {
          const uint32_t a = sbuf + (uu - u0) * UNIT;
          wr[h][0] = lds_v4(a + g * ROW_STRIDE);
          wr[h][1] = lds_v4(a + (g + 8) * ROW_STRIDE);
        } else {
          wr[h][0] = make_uint4(0, 0, 0, 0);
          wr[h][1] = wr[h][0];
        }
      }
      }
      if (!HOLD) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[slot]);
      }
      float acc[MT][PW];
#pragma unroll
      for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int j = 0; j < PW; ++j) acc[t][j] = 0.f;
      if constexpr (FMT == 20) {
        // one 4-token tile (M <= 2 here: columns 2 tok, 2 tok + 1 are the hi / lo digits of token tok = c)
        const int* corr_i = reinterpret_cast<const int*>(corr);
        const float* fac = corr + 2 * p.M * units_staged;
        const int ncols = 2 * p.M;
        const int tok = c < p.M ? c : 0;                  // lanes of absent tokens compute unused columns
        const int uloc0 = il * RANGE_UNITS + gw;          // unit h of this warp: uloc0 + h * GW
        const uint8_t* xb = xs + uloc0 * (ncols * 128) + (g < ncols ? g : 0) * 64 + c * 16;
        const int ci = tok * units_staged + uloc0;
        float a0 = 0.f, a8 = 0.f;
#pragma unroll
        for (int h = 0; h < UPW; ++h) {
          const bool ok = u0 + gw + h * GW < uend;
          const uint8_t* bp = xb + h * GW * (ncols * 128);
          const uint4 b0 = *reinterpret_cast<const uint4*>(bp);
          const uint4 b1 = *reinterpret_cast<const uint4*>(bp + ncols * 64);
          const int2 cv = *reinterpret_cast<const int2*>(corr_i + (ci + h * GW) * 2);
          const float f = fac[ci + h * GW];
          const float sf0 = ok ? sc[h][0] * f : 0.f;
          const float sf8 = ok ? sc[h][1] * f : 0.f;
          if constexpr (HOLD) {
            const uint32_t a = code_base + (gw + h * GW) * (RB * UNIT);
            unit_i8_lean(lds_v4(a), lds_v4(a + 8 * UNIT), b0, b1, cv.x, cv.y, sf0, sf8, a0, a8);
          } else {
            unit_i8_lean(wr[h][0], wr[h][1], b0, b1, cv.x, cv.y, sf0, sf8, a0, a8);
          }
        }
        if constexpr (HOLD) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty_bar[slot]);
        }
        acc[0][0] = a0;
        acc[0][1] = a8;
      } else {
#pragma unroll
      for (int h = 0; h < UPW; ++h) {
        const int uu = u0 + gw + h * GW;
        if (uu >= uend) continue;
        uint32_t Bl[MT][4 * XCH];
        float Nl[MT][2];
        const uint32_t uloc = static_cast<uint32_t>(il * RANGE_UNITS + (uu - u0));
#pragma unroll
        for (int t = 0; t < MT; ++t) {
#pragma unroll
          for (int v = 0; v < XCH; ++v) {
            const uint4 qv = lds_v4(tok_ok[t] ? xrow[t] + uloc * XU + v * 64 : zbase + ((v * 64 + 64) & 127));
            Bl[t][4 * v] = qv.x; Bl[t][4 * v + 1] = qv.y; Bl[t][4 * v + 2] = qv.z; Bl[t][4 * v + 3] = qv.w;
          }
#pragma unroll
          for (int j2 = 0; j2 < 2; ++j2) {
            const int tok = t * 8 + 2 * c + j2;
            Nl[t][j2] = tok < p.M ? -corr[tok * units_staged + uloc] : 0.f;
          }
        }
        float a4[MT][4];
#pragma unroll
        for (int t = 0; t < MT; ++t) { a4[t][0] = acc[t][0]; a4[t][1] = acc[t][1]; a4[t][2] = acc[t][2]; a4[t][3] = acc[t][3]; }
        unit_mma<FMT, MT>(wr[h][0], wr[h][1], Bl, Nl, sc[h][0], sc[h][1], a4);
#pragma unroll
        for (int t = 0; t < MT; ++t) { acc[t][0] = a4[t][0]; acc[t][1] = a4[t][1]; acc[t][2] = a4[t][2]; acc[t][3] = a4[t][3]; }
      }
      }

      // -------------------------------------------------------------- the item's partial: four warps
      const int buf = n_it & 1;
      {
        float* dst = gred + (((grp * 2 + buf) * GW + gw) * 32 + lane) * (PW * MT);
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          if constexpr (PW == 4)
            *reinterpret_cast<float4*>(dst + 4 * t) = make_float4(acc[t][0], acc[t][1], acc[t][2], acc[t][3]);
          else
            *reinterpret_cast<float2*>(dst + 2 * t) = make_float2(acc[t][0], acc[t][1]);
        }
      }
      named_sync(2 + grp, GW * 32);
      if (gw == (n_it % GW)) {
        const float* src = gred + ((grp * 2 + buf) * GW) * 32 * (PW * MT);
        for (int o = lane; o < 16 * p.M; o += 32) {
          const int orow = o & 15, otok = o >> 4;
          int src_lane, reg;
          if constexpr (FMT == 20) {          // 4-token tiles: token 4T + c in lane (row & 7) * 4 + c
            src_lane = (orow & 7) * 4 + (otok & 3);
            reg = (otok >> 2) * 2 + (orow >> 3);
          } else {                           // 8-token tiles: tokens 2c, 2c + 1 in lane (row & 7) * 4 + c
            const int tt = otok >> 3, tk = otok & 7;
            src_lane = (orow & 7) * 4 + (tk >> 1);
            reg = tt * 4 + (orow >> 3) * 2 + (tk & 1);
          }
          float v = 0.f;
#pragma unroll
          for (int w = 0; w < GW; ++w) v += src[(w * 32 + src_lane) * (PW * MT) + reg];
          if constexpr (FMT != 20) v *= xsc[otok * MAX_RANGES + r];
          if (direct) {
            const int64_t n = row0 + orow;
            if (n < p.N) store_out<FMT>(p, n, otok, v);
          } else {
            ptab[q * 16 * p.M + o] = v;
          }
        }
      }
    }
  }

  if (!direct) {
    // ------------------------------------------------------------------ add the K ranges in order
    // Item (k, il) of cluster rank j holds range j + il * R of row block k.  Rank j adds the ranges of row
    // blocks k = j, j + R, ... in range order, reading the other ranks' tables through distributed shared
    // memory (its own table when R = 1); the second barrier keeps every CTA alive until all reads are done.
    if (R > 1) asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    else __syncthreads();
    const int per_block = 16 * p.M;
    for (int e = threadIdx.x; e < ((nmine + R - 1 - rank) / R) * per_block; e += blockDim.x) {
      const int k = rank + (e / per_block) * R, o = e % per_block;
      const int orow = o & 15, otok = o >> 4;
      float v = 0.f;
      for (int rr = 0; rr < p.nr; ++rr) {
        const int owner = rr % R, il = rr / R;
        const int idx = (k * ranges_of_rank(p.nr, R, owner) + il) * per_block + o;
        float part;
        if (R > 1) {
          uint32_t remote;
          asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(&ptab[idx])), "r"(owner));
          asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(part) : "r"(remote) : "memory");
        } else {
          part = ptab[idx];
        }
        v = (rr == 0) ? part : v + part;
      }
      const int64_t n = static_cast<int64_t>(cid + k * p.C) * RB + orow;
      if (n < p.N) store_out<FMT>(p, n, otok, v);
    }
    if (R > 1) asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  }
}

// ------------------------------------------------------------------------------------------- fp6 rows
// fp6 e3m2 (FMT 7) / e2m3 (FMT 8) rows, M <= 16: four codes per three bytes (value j of a group at bits
// 6j .. 6j + 5 of its little-endian 24-bit word) do not fit the 64-byte units of gemv_kernel, so this product
// runs on the CUDA cores.  One warp per row at a time; lane l takes the 12-byte chunks l, l + 32, ... of the
// row (16 values each), turns each pair of codes into an exact fp16 pair with the hardware conversion and
// accumulates value * x in float32 per token in chunk order; the lanes are added by the xor butterfly (a fixed
// order, so every launch and every column shard gives the same bits); the epilogue is gemv_kernel's.
template <int FMT>
__device__ __forceinline__ void deq_fp6_group(uint32_t g, float (&v)[4]) {
  // the four 6-bit fields into the low bits of four bytes
  const uint32_t u = (g & 0x3Fu) | ((g << 2) & 0x3F00u) | ((g << 4) & 0x3F0000u) | ((g << 6) & 0x3F000000u);
  uint32_t lo, hi;
  if (FMT == 7) {
    asm("{\n\t.reg .b16 a;\n\tcvt.u16.u32 a, %1;\n\tcvt.rn.f16x2.e3m2x2 %0, a;\n\t}" : "=r"(lo) : "r"(u));
    asm("{\n\t.reg .b16 a;\n\tcvt.u16.u32 a, %1;\n\tcvt.rn.f16x2.e3m2x2 %0, a;\n\t}" : "=r"(hi) : "r"(u >> 16));
  } else {
    asm("{\n\t.reg .b16 a;\n\tcvt.u16.u32 a, %1;\n\tcvt.rn.f16x2.e2m3x2 %0, a;\n\t}" : "=r"(lo) : "r"(u));
    asm("{\n\t.reg .b16 a;\n\tcvt.u16.u32 a, %1;\n\tcvt.rn.f16x2.e2m3x2 %0, a;\n\t}" : "=r"(hi) : "r"(u >> 16));
  }
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&lo));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&hi));
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}

__device__ __forceinline__ uint32_t ldg_nc_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

template <int FMT>
__global__ void __launch_bounds__(256) gemv_fp6_kernel(const GemvParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t rb = p.K / 4 * 3;            // code bytes of a row
  const int64_t nch = p.K / 16;              // 12-byte chunks of a row
  for (int64_t n = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); n < p.N; n += warps) {
    float acc[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) acc[t] = 0.f;
    const uint8_t* wr = p.w + n * rb;
    for (int64_t c = lane; c < nch; c += 32) {
      const uint8_t* q = wr + 12 * c;        // 4-byte aligned: rows start at multiples of 12 bytes
      const uint32_t w0 = ldg_nc_u32(q), w1 = ldg_nc_u32(q + 4), w2 = ldg_nc_u32(q + 8);
      float v[16];
      {
        float g4[4];
        deq_fp6_group<FMT>(w0 & 0xFFFFFFu, g4);
        v[0] = g4[0]; v[1] = g4[1]; v[2] = g4[2]; v[3] = g4[3];
        deq_fp6_group<FMT>((w0 >> 24) | ((w1 & 0xFFFFu) << 8), g4);
        v[4] = g4[0]; v[5] = g4[1]; v[6] = g4[2]; v[7] = g4[3];
        deq_fp6_group<FMT>((w1 >> 16) | ((w2 & 0xFFu) << 16), g4);
        v[8] = g4[0]; v[9] = g4[1]; v[10] = g4[2]; v[11] = g4[3];
        deq_fp6_group<FMT>(w2 >> 8, g4);
        v[12] = g4[0]; v[13] = g4[1]; v[14] = g4[2]; v[15] = g4[3];
      }
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        if (t < p.M) {
          const uint16_t* xr = p.x + static_cast<int64_t>(t) * p.K + 16 * c;
          const uint4 a = ldg_nc_v4(xr), b = ldg_nc_v4(xr + 8);
          const uint32_t r[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
          float s = acc[t];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            s = fmaf(v[2 * e], __uint_as_float(r[e] << 16), s);
            s = fmaf(v[2 * e + 1], __uint_as_float(r[e] & 0xFFFF0000u), s);
          }
          acc[t] = s;
        }
      }
    }
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      if (t < p.M) {
        float s = acc[t];
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == t) store_out<FMT>(p, n, t, s);
      }
    }
  }
}

// ------------------------------------------------------------------------------------------- launcher
int gemv_max_k(int fmt) {
  if (fmt == 7 || fmt == 8) return 1 << 30;   // the fp6 product has no K ranges
  // at most MAX_RANGES K ranges per row
  return gemv::MAX_RANGES * gemv::RANGE_UNITS * gemv::UNIT * ((fmt == 2 || fmt == 9) ? 2 : 1);
}

template <int FMT, int MT, int G, int MINB, bool BOX = false, bool LR = false>
static cudaError_t launch_gemv_t(GemvParams p, int sms, int ctas_per_sm, int max_slots, bool pdl, cudaStream_t st,
                                 const CUtensorMap* tw = nullptr, const CUtensorMap* ts = nullptr) {
  using namespace gemv;
  auto kern = gemv_kernel<FMT, MT, G, MINB, BOX, LR>;
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_LIMIT);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  int limit = MINB >= 2 ? HALF_SM_SMEM : SMEM_LIMIT;
  int target = sms * ctas_per_sm;
  // cluster size: one CTA per row block's K span unless that leaves SMs idle or x does not fit
  auto smem_for = [&](int R, int slots, int C) {
    const int nloc0 = ranges_of_rank(p.nr, R, 0);
    const int rows_per_cluster = (p.nblocks + C - 1) / C;
    const int items = (R == 1 && p.nr == 1) ? 0 : rows_per_cluster * nloc0;
    return gemv_smem(FMT, p.M, MT, G, nloc0 * RANGE_UNITS, slots, items).total;
  };
  int R = 1;
  const int rmax = p.nr < MAX_CLUSTER ? p.nr : MAX_CLUSTER;
  auto clusters_for = [&](int R_) { int c = target / R_; return c < p.nblocks ? c : p.nblocks; };
  // box mode keeps at least two items in flight per CTA (its slots are the only ring a group has)
  const int fit_slots = BOX ? (2 * G <= max_slots ? 2 * G : G) : G;
  while (R < rmax && (smem_for(R, fit_slots, clusters_for(R)) > limit || clusters_for(R) * R < target / 2)) ++R;
  if (smem_for(R, G, clusters_for(R)) > limit && limit < SMEM_LIMIT) {   // one CTA per SM after all
    limit = SMEM_LIMIT;
    target = sms;
    R = 1;
    while (R < rmax && (smem_for(R, G, clusters_for(R)) > limit || clusters_for(R) * R < target / 2)) ++R;
  }
  int C = clusters_for(R);
  if (C < 1) C = 1;
  if (smem_for(R, G, C) > limit) return cudaErrorInvalidValue;
  int slots = G;                                     // a multiple of G (one slot set per group)
  while (slots + G <= max_slots && smem_for(R, slots + G, C) <= limit) slots += G;
  p.R = R;
  p.C = C;
  p.slots = slots;
  p.max_items = (R == 1 && p.nr == 1) ? 0 : ((p.nblocks + C - 1) / C) * ranges_of_rank(p.nr, R, 0);
  const size_t smem = static_cast<size_t>(smem_for(R, slots, C));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  int na = 0;
  cfg.gridDim = dim3(static_cast<unsigned>(C * R), 1, 1);
  if (R > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = static_cast<unsigned>(R);
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cfg.blockDim = dim3((G * GW + 1) * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  static const CUtensorMap none = {};
  return cudaLaunchKernelEx(&cfg, kern, p, tw ? *tw : none, ts ? *ts : none);
}

// Tensor maps of box mode: codes as a 3-D tensor (64 bytes of a unit, row, unit) whose box lands [unit][row][64 B]
// in shared memory; scales as a 2-D tensor (unit, row) when a scale row is a multiple of 16 bytes.
static bool encode_gemv_boxes(const void* codes, const void* scales, int64_t N, int64_t K, bool i4, CUtensorMap* tw,
                              CUtensorMap* ts, bool* scale_tma) {
  using namespace gemv;
  PFN_encodeTiled enc = get_encode();
  if (!enc || N > (1LL << 31)) return false;
  const int64_t row_bytes = i4 ? K / 2 : K;
  const int64_t units = row_bytes / UNIT;
  {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(UNIT), static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(units)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(UNIT)};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(UNIT), static_cast<cuuint32_t>(RB), static_cast<cuuint32_t>(RANGE_UNITS)};
    cuuint32_t es[3] = {1, 1, 1};
    if (enc(tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(codes), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return false;
  }
  *scale_tma = false;
  if (i4 && (units * 2) % 16 == 0) {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(units), static_cast<cuuint64_t>(N)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(units * 2)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(RANGE_UNITS), static_cast<cuuint32_t>(RB)};
    cuuint32_t es[2] = {1, 1};
    if (enc(ts, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(scales), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
      *scale_tma = true;
  }
  return true;
}

void prepare_gemv_maps(int fmt, const void* codes, const void* scales, int64_t N, int64_t K, GemvMaps* m) {
  m->ok = 0;
  m->stma = 0;
  bool stma = false;
  if (fmt == 2 && encode_gemv_boxes(codes, scales, N, K, true, &m->tw, &m->ts, &stma)) {
    m->ok = 1;
    m->stma = stma ? 1 : 0;
  }
}

cudaError_t launch_gemv(int fmt, const void* x, int64_t M, int64_t K, const void* codes, const void* scales,
                        int64_t N, const void* bias, int acc, void* y, int64_t ldy, int sms, bool pdl,
                        cudaStream_t st, const OutRanks* dst, const RmsPrologue* ln, const GemvMaps* maps) {
  GemvParams p;
  p.x = reinterpret_cast<const uint16_t*>(x);
  p.w = reinterpret_cast<const uint8_t*>(codes);
  p.s16 = reinterpret_cast<const __half*>(scales);
  p.bias = reinterpret_cast<const uint16_t*>(bias);
  p.y = reinterpret_cast<uint16_t*>(y);
  p.N = N; p.K = K; p.ldy = ldy;
  p.M = static_cast<int>(M);
  p.acc = acc;
  const int64_t row_bytes = (fmt == 2 || fmt == 9) ? K / 2 : K;
  p.total_units = static_cast<int>(row_bytes / gemv::UNIT);
  p.nblocks = static_cast<int>((N + gemv::RB - 1) / gemv::RB);
  p.nr = (p.total_units + gemv::RANGE_UNITS - 1) / gemv::RANGE_UNITS;
  p.R = 1; p.C = 1; p.slots = 2; p.max_items = 0;
  p.dst = dst ? *dst : OutRanks{};
  p.ln = ln ? ln->w : nullptr;
  p.ln_f32 = ln ? ln->w_f32 : 0;
  p.ln_vec = (ln && (reinterpret_cast<uintptr_t>(ln->w) & 15) == 0) ? 1 : 0;
  p.ln_eps = ln ? ln->eps : 0.f;
  p.ln_off = ln ? ln->off : 0.f;
  p.scale_tma = 0;
  p.pre = 1 << 30;
  if (fmt == 7 || fmt == 8) {
    if (ln) return cudaErrorNotSupported;     // the norm prologue lives in gemv_kernel's staging
    const int64_t want = (N + 7) / 8;         // one warp per row
    const unsigned grid = static_cast<unsigned>(want < 4LL * sms ? want : 4LL * sms);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return fmt == 7 ? cudaLaunchKernelEx(&cfg, gemv_fp6_kernel<7>, p) : cudaLaunchKernelEx(&cfg, gemv_fp6_kernel<8>, p);
  }
  // one token tile: three groups (12 warps + producer) and six ring slots; two token tiles: two groups
  // int4: one or two tokens on the integer tensor path (half the MMAs, a third of the dequantisation work;
  // [11008, 4096] at M = 2: 9.38 -> 8.78 us); more tokens on the bf16 path, whose n8 tile holds eight tokens
  // (the integer path measured 5 % slower at M = 4 and 25-60 % slower at M = 8: heavier staging, two tiles)
  if (fmt == 2) {
#ifndef LB_GEMV_NO_BOX
    if (M <= 2) {
      // box mode: one tensor copy per item (codes, and scales when their rows allow it); three groups, one slot
      // each ([28672, 8192]: 31.7 -> 29.2 us, [8192, 28672]: 40.3 -> 36.7 us against one copy per row)
      // a prepared weight brings its maps (encoded once); otherwise they are encoded for this launch
      GemvMaps local;
      if (!maps) {
        prepare_gemv_maps(fmt, codes, scales, N, K, &local);
        maps = &local;
      }
      const CUtensorMap& tw = maps->tw;
      const CUtensorMap& ts = maps->ts;
      if (maps->ok) {
        p.scale_tma = maps->stma;
        // one or two K ranges per row and a row block for every SM: six slots, so a CTA requests (almost) its
        // whole share of the weights at once, with the codes read from the slot unit by unit
        // ([11008, 4096]: 7.15 -> 6.68 us, [28672, 8192]: 25.1 -> 23.4 us); otherwise three slots
        // ([4096, 11008]: 10.2 against 11.0 us, [8192, 28672]: 31.7 against 49 us with six)
        if (p.nr <= 2 && p.nblocks >= sms) {
          p.pre = 1;   // then the activations' loads, then the rest ([11008, 4096]: 6.65 -> 6.45 us)
          return launch_gemv_t<20, 1, 3, 1, true, true>(p, sms, 1, 6, pdl, st, &tw, &ts);
        }
        return launch_gemv_t<20, 1, 3, 1, true>(p, sms, 1, 3, pdl, st, &tw, &ts);
      }
    }
#endif
    if (M <= 2) return launch_gemv_t<20, 1, 3, 1>(p, sms, 1, 6, pdl, st);
    // several K ranges per row (K > 4096) and more than four tokens: the ring holds four slots with two groups
    // against three with three groups once the larger activation staging is placed (measured on [4096, 11008]
    // at M = 8: 26.8 -> 21.6 us; single-range shapes are faster with three groups)
    if (M > 4 && M <= 8 && p.nr > 1) return launch_gemv_t<2, 1, 2, 1>(p, sms, 1, gemv::MAX_SLOTS, pdl, st);
    return M <= 8 ? launch_gemv_t<2, 1, 3, 1>(p, sms, 1, 6, pdl, st)
                  : launch_gemv_t<2, 2, 2, 1>(p, sms, 1, gemv::MAX_SLOTS, pdl, st);
  }
  if (fmt == 5)
    return M <= 8 ? launch_gemv_t<5, 1, 3, 1>(p, sms, 1, 6, pdl, st)
                  : launch_gemv_t<5, 2, 2, 1>(p, sms, 1, gemv::MAX_SLOTS, pdl, st);
  if (fmt == 6)
    return M <= 8 ? launch_gemv_t<6, 1, 3, 1>(p, sms, 1, 6, pdl, st)
                  : launch_gemv_t<6, 2, 2, 1>(p, sms, 1, gemv::MAX_SLOTS, pdl, st);
  if (fmt == 9)
    return M <= 8 ? launch_gemv_t<9, 1, 3, 1>(p, sms, 1, 6, pdl, st)
                  : launch_gemv_t<9, 2, 2, 1>(p, sms, 1, gemv::MAX_SLOTS, pdl, st);
  return M <= 8 ? launch_gemv_t<1, 1, 3, 1>(p, sms, 1, 6, pdl, st)
                : launch_gemv_t<1, 2, 2, 1>(p, sms, 1, gemv::MAX_SLOTS, pdl, st);
}

}  // namespace lb

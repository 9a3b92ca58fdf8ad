// Device helpers shared by the kernels: mbarriers with bounded waits, TMA bulk copies, tcgen05 wrappers,
// packed bf16/f16 arithmetic.  sm_100a only.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "apsi_b200 kernels are written for sm_100a only"
#endif

namespace lb {

// Device error word (LB_DEVERR_* bits), one per device; read and cleared by lb_device_errors().
// The library is compiled as one translation unit (lb_lib.cu), so this is its only definition.
__device__ int g_dev_errors = 0;


__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait that lets the hardware suspend the thread for up to `ns` nanoseconds while the phase is pending
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}
// Programmatic dependent launch: let the next kernel on the stream start its independent prologue, and wait
// for the previous kernel's results (both are no-ops when the launch did not opt in).
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits for the phase with the given parity to complete.  Each try lets the hardware suspend the thread while
// the phase is pending; after kWaitLimitNs of wall time (read from the global timer, so the bound does not
// depend on how long one try suspends), or at once when *abort is set, it records LB_DEVERR_WAIT_TIMEOUT, sets
// *abort so every other wait of the CTA returns at once, and returns false.  Callers carry on (their output
// is invalid), so no CTA barrier is skipped.
constexpr uint64_t kWaitLimitNs = 2000000000ull;   // 2 s
__device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0; i < (1u << 30); ++i) {
    if (mbar_try_wait_sleep(bar, parity, 1000000u)) return true;
    if (*abort) return false;
    if ((i & 15u) == 15u && global_ns() - t0 > kWaitLimitNs) break;
  }
  *abort = 1;
  atomicOr(&g_dev_errors, 1);
  return false;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait_sleep(bar, parity, 1000000u)) return true;   // usual case: completes within one try
  return mbar_wait_slow(bar, parity, abort);
}

// ------------------------------------------------------------------------------------------- TMA
// 1-D bulk copy global -> shared, completion counted in bytes on `bar`.  Sizes/addresses multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// L2 policy for data read once (streamed weights): evicted first, so it does not push out reused data.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// bulk_g2s with an L2 cache policy
__device__ __forceinline__ void bulk_g2s_hint(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Tiled 2-D tensor copy global -> shared (no multicast).  c0 is the innermost coordinate (in elements).
__device__ __forceinline__ void tma_load_2d(void* dst_smem, const void* tmap, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst_smem)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}
// Tiled 3-D tensor copy global -> shared with an L2 cache policy (no multicast).
__device__ __forceinline__ void tma_load_3d_hint(void* dst_smem, const void* tmap, int c0, int c1, int c2,
                                                 uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst_smem)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ------------------------------------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Arrives once on `bar` when every tcgen05.mma issued before by this thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]; kind::f16 (fp16 or bf16 inputs), fp32 accumulation.
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 32 lanes x 16 columns of 32 bits: thread t writes lane (base lane + t), columns [col, col + 16).
__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// Shared-memory matrix descriptor for a K-major operand written by TMA with 128-byte swizzle: rows of 128 B,
// 8-row atoms 1024 B apart.  `addr` is the shared address of the (1024-aligned) tile plus the K offset.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);        // start address
  d |= (uint64_t)1 << 16;                       // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;             // stride byte offset: next 8-row group
  d |= (uint64_t)1 << 46;                       // descriptor version for tcgen05
  d |= (uint64_t)2 << 61;                       // SWIZZLE_128B
  return d;
}

// Instruction descriptor of kind::f16 with fp16 A/B, fp32 D, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4)                              // D format F32
         | (0u << 7) | (0u << 10)               // A, B format F16
         | ((uint32_t)(N >> 3) << 17)           // N >> 3
         | ((uint32_t)(M >> 4) << 24);          // M >> 4
}

// ------------------------------------------------------------------------------------------- packed math
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t magic) {
  // (a & mask) | magic : immLut for (a & b) | c = 0xEA
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(magic));
  return d;
}
__device__ __forceinline__ uint32_t lop3_and_xor_or(uint32_t a, uint32_t mask, uint32_t c) {
  // (mask & (a ^ c)) | (~mask & c): immLut for b ? (a ^ c) : c with a=0xF0, b=0xCC, c=0xAA -> 0x6A
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(a), "r"(mask), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
__device__ __forceinline__ uint32_t bf2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t h2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// m16n8k16 bf16 tensor-core product, fp32 accumulate: d = a * b + c.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2],
                                               const float (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %11, %12, %13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "f"(c[0]), "f"(c[1]), "f"(c[2]),
        "f"(c[3]));
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t addr) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint4 lds_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

// fp4 e2m1: one word (8 codes, code 2j in the low nibble of byte j) -> the exact fp16 pairs (code 0, code 1),
// (2, 3), (4, 5), (6, 7) through the hardware conversion.
__device__ __forceinline__ void deq_fp4_word(uint32_t w, uint32_t (&p)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(p[0]), "=r"(p[1]), "=r"(p[2]), "=r"(p[3])
      : "r"(w));
}

// ---- RMSNorm in one fixed order, shared by the standalone norm and the norm prologue of the decode GEMV, so
// that a fused and an unfused normalised projection give the same bits.  A row of K bf16 values is cut into
// 16-byte chunks of 8 values; virtual thread v of 256 (eight warps of 32) adds the squares of chunks v, v + 256,
// v + 512, ... with fmaf in value order; each virtual warp adds its 32 lanes by the xor butterfly 16, 8, 4, 2, 1;
// the eight warp sums are added in warp order; fac = 1 / sqrt(sum / K + eps).
constexpr int RMS_VT = 256;   // virtual threads of the reduction

__device__ __forceinline__ float rms_chunk_fma(const uint4& v, float s) {
  const uint32_t r[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float a = __uint_as_float(r[e] << 16), b = __uint_as_float(r[e] & 0xFFFF0000u);
    s = fmaf(a, a, s);
    s = fmaf(b, b, s);
  }
  return s;
}

// chunk j of a row (values 8j .. 8j + 7, zeros past K); `vec`: the row is 16-byte aligned and K % 8 == 0
__device__ __forceinline__ uint4 rms_load_chunk(const uint16_t* row, int64_t K, int64_t j, bool vec) {
  if (vec) return ldg_nc_v4(row + 8 * j);
  uint32_t r[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int64_t k = 8 * j + 2 * e;
    const uint32_t a = k < K ? row[k] : 0u, b = k + 1 < K ? row[k + 1] : 0u;
    r[e] = a | (b << 16);
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

__device__ __forceinline__ float rms_butterfly(float s) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

__device__ __forceinline__ float rms_factor(float tot, int64_t K, float eps) {
  return 1.0f / sqrtf(tot / static_cast<float>(K) + eps);
}

// The whole reduction of one row by one warp (lane l plays virtual threads l, l + 32, ..., l + 224): each pass
// loads the next chunk of all eight virtual threads at once, so the loads of a pass are in flight together.
__device__ __forceinline__ float rms_row_factor_warp(const uint16_t* row, int64_t K, float eps, bool vec) {
  constexpr int NW = RMS_VT / 32;
  const int lane = threadIdx.x & 31;
  const int64_t nc = (K + 7) / 8;
  float s[NW];
#pragma unroll
  for (int w = 0; w < NW; ++w) s[w] = 0.f;
  for (int64_t j0 = lane; j0 < nc; j0 += RMS_VT) {
    uint4 v[NW];
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const int64_t j = j0 + 32 * w;
      v[w] = j < nc ? rms_load_chunk(row, K, j, vec) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int w = 0; w < NW; ++w)
      if (j0 + 32 * w < nc) s[w] = rms_chunk_fma(v[w], s[w]);
  }
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < NW; ++w) tot += rms_butterfly(s[w]);
  return rms_factor(tot, K, eps);
}

// The 8 RMSNorm weights at element k0 (float32: a, b; bf16: a), 16-byte aligned loads when `vec`.
struct RmsW {
  uint4 a, b;
};
__device__ __forceinline__ RmsW rms_load_w(const void* w, bool w_f32, int64_t k0, int64_t K, bool vec) {
  RmsW r;
  if (vec && w_f32) {
    r.a = ldg_nc_v4(static_cast<const float*>(w) + k0);
    r.b = ldg_nc_v4(static_cast<const float*>(w) + k0 + 4);
  } else if (vec) {
    r.a = ldg_nc_v4(static_cast<const uint16_t*>(w) + k0);
    r.b = make_uint4(0u, 0u, 0u, 0u);
  } else {
    uint32_t f[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int64_t k = k0 + e < K ? k0 + e : K - 1;
      f[e] = w_f32 ? __float_as_uint(static_cast<const float*>(w)[k])
                   : static_cast<uint32_t>(static_cast<const uint16_t*>(w)[k]);
    }
    if (w_f32) {
      r.a = make_uint4(f[0], f[1], f[2], f[3]);
      r.b = make_uint4(f[4], f[5], f[6], f[7]);
    } else {
      r.a = make_uint4(f[0] | (f[1] << 16), f[2] | (f[3] << 16), f[4] | (f[5] << 16), f[6] | (f[7] << 16));
      r.b = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  return r;
}

// The normalised chunk: each value bf16((x * fac) * (w + off)).
__device__ __forceinline__ uint4 rms_apply_chunk(const uint4& v, float fac, const RmsW& w, bool w_f32, float off) {
  float wf[8];
  if (w_f32) {
    wf[0] = __uint_as_float(w.a.x); wf[1] = __uint_as_float(w.a.y); wf[2] = __uint_as_float(w.a.z);
    wf[3] = __uint_as_float(w.a.w); wf[4] = __uint_as_float(w.b.x); wf[5] = __uint_as_float(w.b.y);
    wf[6] = __uint_as_float(w.b.z); wf[7] = __uint_as_float(w.b.w);
  } else {
    const uint32_t r[4] = {w.a.x, w.a.y, w.a.z, w.a.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) { wf[2 * e] = __uint_as_float(r[e] << 16); wf[2 * e + 1] = __uint_as_float(r[e] & 0xFFFF0000u); }
  }
  const uint32_t r[4] = {v.x, v.y, v.z, v.w};
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float ya = __uint_as_float(r[e] << 16) * fac * (wf[2 * e] + off);
    const float yb = __uint_as_float(r[e] & 0xFFFF0000u) * fac * (wf[2 * e + 1] + off);
    const __nv_bfloat162 h = __floats2bfloat162_rn(ya, yb);
    o[e] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

}  // namespace lb

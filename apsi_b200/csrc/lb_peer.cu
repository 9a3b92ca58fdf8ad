// Column-sharded linear with the gather fused into the product's epilogue, over NVLink peer memory.
//
// A layer of N output features is split over G ranks (one process per GPU); rank r owns columns
// [r Nl, (r + 1) Nl).  Instead of writing its [M, Nl] block locally and reassembling the full [M, N] output
// with an all-gather and an interleave, rank r's GEMV or GEMM epilogue stores each output value into column
// r Nl + n of EVERY rank's [M, ldy] output buffer: the local one and, through CUDA IPC mappings, the other
// ranks' (plain st.global over NVLink, no TMA, no multicast).  The transfer overlaps the products tile by tile
// and no interleave pass remains.  A small barrier kernel then tells every rank that this rank's stores are
// complete and waits until all ranks have said the same, so the full output may be read.
//
// Peer buffers: lb_peer_alloc (cudaMalloc + an IPC handle the caller exchanges between ranks), lb_peer_open /
// lb_peer_close on the other ranks, lb_peer_free by the owner.
//
// Barrier: each rank owns an array of G 32-bit flags in a peer buffer.  lb_rank_barrier(epoch) runs after the
// products in stream order, launched as their programmatic dependent (so the next static-weight product streams
// its weights while the barrier waits); its system-scope fence, followed by the flag stores (a release pattern),
// orders every store of those kernels (local and peer) before the flag it writes into slot `rank` of every rank's
// array, and it waits until every
// slot of its own array has reached `epoch` (acquire loads), i.e. every rank's stores are visible here.  The
// wait gives up after a time limit, sets LB_DEVERR_PEER_TIMEOUT in the device error word and returns, so a
// rank that never arrives is reported, not waited on for ever.  Epochs increase by one per call on every rank;
// the comparison is wrap-aware, so a rank that has already reached the next barrier does not stall a slower one.
// With epoch 0 the barrier takes its epoch from a counter in word G of this rank's own array (incremented on
// the device), so a captured CUDA graph that replays barriers stays in step on every rank.
#include <cstring>
#include "../../include/apsi_lowbit.h"
#include "lb_common.cuh"
#include "lb_kernels.h"

namespace lb {

struct BarrierParams {
  uint32_t* flags[kMaxRanks];   // rank g's flag array (G words + the epoch counter), local or IPC-mapped
  int G, rank;
  uint32_t epoch;
  uint64_t limit_ns;
};

__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void rank_barrier_kernel(const BarrierParams p) {
  // Launched as a programmatic dependent of the products: the next kernel on the stream (the following
  // static-weight GEMV) may launch now and stream its weights while this barrier waits for the other ranks;
  // everything it reads from earlier kernels waits for this grid to complete.  griddepcontrol.wait below
  // returns once the products before this barrier have completed and their stores are performed.
  pdl_launch_dependents();
  pdl_wait();
  if (threadIdx.x != 0) return;
  uint32_t* mine = p.flags[p.rank];
  uint32_t epoch = p.epoch;
  if (epoch == 0) {                         // device-side counter: only this thread of this rank touches it
    epoch = mine[p.G] + 1;
    if (epoch == 0) epoch = 1;
    mine[p.G] = epoch;
  }
  // one system-scope fence, then relaxed flag stores: the fence followed by a strong store is a release of
  // everything ordered before it (the products' stores included), so each flag needs no fence of its own
  // (a st.release per rank costs a fence per rank: about 1.5 us each).  acq_rel is the fence a release needs;
  // the sequentially consistent one measured the same or slower.
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  for (int g = 0; g < p.G; ++g) st_relaxed_sys(p.flags[g] + p.rank, epoch);
  const uint64_t t0 = global_ns();
  for (int g = 0; g < p.G; ++g) {
    for (uint32_t i = 0; static_cast<int32_t>(ld_acquire_sys(mine + g) - epoch) < 0; ++i) {
      if (i > (1u << 28) || global_ns() - t0 > p.limit_ns) {
        atomicOr(&g_dev_errors, LB_DEVERR_PEER_TIMEOUT);
        return;
      }
      __nanosleep(256);
    }
  }
}

}  // namespace lb

using namespace lb;

static_assert(sizeof(cudaIpcMemHandle_t) == LB_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" {

int lb_peer_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return fail(LB_E_ARG, "lb_peer_alloc: ptr, handle and a size are required");
  DevInfo* d;
  int r = current(&d);
  if (r) return r;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return fail(LB_E_DEVICE, "lb_peer_alloc: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(LB_E_DEVICE, "lb_peer_alloc: %s", cudaGetErrorString(e));
  }
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return LB_OK;
}

int lb_peer_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return fail(LB_E_ARG, "lb_peer_open: handle and ptr are required");
  DevInfo* d;
  int r = current(&d);
  if (r) return r;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(LB_E_DEVICE, "lb_peer_open: %s", cudaGetErrorString(e));
  *ptr = p;
  return LB_OK;
}

int lb_peer_close(void* ptr) {
  if (!ptr) return fail(LB_E_ARG, "lb_peer_close: NULL pointer");
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return fail(LB_E_DEVICE, "lb_peer_close: %s", cudaGetErrorString(e));
  return LB_OK;
}

int lb_peer_free(void* ptr) {
  if (!ptr) return fail(LB_E_ARG, "lb_peer_free: NULL pointer");
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return fail(LB_E_DEVICE, "lb_peer_free: %s", cudaGetErrorString(e));
  return LB_OK;
}

int lb_linear_sharded(int fmt, const void* x, int64_t M, int64_t K, const void* codes, const void* scales,
                      int64_t Nl, const void* bias, void* const* y_ranks, int G, int rank, int64_t ldy,
                      void* workspace, size_t ws_bytes, unsigned flags, void* stream) {
  if (G < 1 || G > kMaxRanks) return fail(LB_E_ARG, "lb_linear_sharded: G (%d) must be in 1..%d", G, kMaxRanks);
  if (rank < 0 || rank >= G) return fail(LB_E_ARG, "lb_linear_sharded: rank %d out of 0..%d", rank, G - 1);
  if (!y_ranks) return fail(LB_E_ARG, "lb_linear_sharded: y_ranks is NULL");
  if (Nl <= 0 || ldy < G * Nl)
    return fail(LB_E_ARG, "lb_linear_sharded: ldy (%lld) < G * Nl (%lld)", (long long)ldy, (long long)(G * Nl));
  OutRanks dst = {};
  for (int g = 0; g < G; ++g) {
    if (!y_ranks[g]) return fail(LB_E_ARG, "lb_linear_sharded: y_ranks[%d] is NULL", g);
    if (!aligned(y_ranks[g], 2)) return fail(LB_E_ALIGN, "lb_linear_sharded: y_ranks[%d] must be 2-byte aligned", g);
    dst.y[g] = static_cast<uint16_t*>(y_ranks[g]);
  }
  dst.n = G;
  dst.col0 = static_cast<int64_t>(rank) * Nl;
  return linear_impl(fmt, x, M, K, codes, scales, Nl, bias, 0, y_ranks[rank], ldy, workspace, ws_bytes, flags, stream,
                     &dst);
}

int lb_rank_barrier(uint32_t* const* flags_ranks, int G, int rank, uint32_t epoch, uint32_t timeout_ms, void* stream) {
  if (G < 1 || G > kMaxRanks) return fail(LB_E_ARG, "lb_rank_barrier: G (%d) must be in 1..%d", G, kMaxRanks);
  if (rank < 0 || rank >= G) return fail(LB_E_ARG, "lb_rank_barrier: rank %d out of 0..%d", rank, G - 1);
  if (!flags_ranks) return fail(LB_E_ARG, "lb_rank_barrier: flags_ranks is NULL");
  BarrierParams p = {};
  for (int g = 0; g < G; ++g) {
    if (!flags_ranks[g] || !aligned(flags_ranks[g], 4))
      return fail(LB_E_ARG, "lb_rank_barrier: flags_ranks[%d] is NULL or not 4-byte aligned", g);
    p.flags[g] = flags_ranks[g];
  }
  p.G = G;
  p.rank = rank;
  p.epoch = epoch;
  p.limit_ns = static_cast<uint64_t>(timeout_ms ? timeout_ms : 2000u) * 1000000ull;
  DevInfo* d;
  int r = current(&d);
  if (r) return r;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(1, 1, 1);
  cfg.blockDim = dim3(32, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return launched(cudaLaunchKernelEx(&cfg, rank_barrier_kernel, p), "rank_barrier");
}

}  // extern "C"

/*
 * apsi_lowbit.h -- C ABI of the B200 (sm_100a) low-bit quantized linear layer.
 *
 * Every entry point is extern "C", takes plain pointers and sizes, returns an int status (LB_OK == 0,
 * negative LB_E_* on error; lb_last_error() gives the message of the calling thread's last failure) and is
 * asynchronous on the given CUDA stream (`stream` is a cudaStream_t passed as void*, NULL = legacy default
 * stream).  All tensor pointers are DEVICE pointers owned by the caller.  Shapes are row-major:
 *
 *   W      [N, K]     weights, N output features, K input features (the HF / hub_gpu layout)
 *   x      [M, K]     bfloat16 activations, M tokens
 *   y      [M, ldy]   bfloat16 outputs (ldy >= N)
 *
 * Formats (LB_FMT_*):
 *   INT8_ROW   codes int8 [N, K]; scale16 IEEE binary16 [N]            (absmax/127 per output row)
 *   INT4_G128  packed uint8 [N, K/2]; scale16 binary16 [N, K/128]      (absmax/7 per 128 values along K;
 *              byte j of a row holds element 2j in the low nibble, element 2j+1 in the high nibble,
 *              two's complement)
 *   Q8_0_G32   words uint32 [N, K/4] (byte j of a word = value j); scale32 float [N, K/32]
 *   Q4_0_G32   words uint32 [N, K/8] (nibble j of a word = value j + 8); scale32 float [N, K/32]
 *   FP8_E4M3, FP8_E5M2, FP6_E3M2, FP6_E2M3, FP4_E2M1  minifloat codes (sign, exponent, mantissa; the
 *              reference's value tables), flat row-major: one byte per value (fp8), four values per three
 *              bytes (fp6, little-endian 24-bit word), two per byte (fp4, even index in the low nibble);
 *              scale32 float [R] per row, or one tensor scale
 *
 * Arguments are checked before anything is launched; a rejected call leaves the device untouched.
 * There is no CPU fallback: without an sm_100 device every compute call fails with LB_E_DEVICE.
 */
#ifndef APSI_LOWBIT_H
#define APSI_LOWBIT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LB_VERSION 10000 /* 1.0.0 */

/* status codes */
#define LB_OK 0
#define LB_E_ARG (-1)         /* null pointer, bad shape, bad format / dtype */
#define LB_E_ALIGN (-2)       /* pointer or leading dimension not aligned as required */
#define LB_E_DEVICE (-3)      /* no usable sm_100 device, or a CUDA runtime error during setup */
#define LB_E_LAUNCH (-4)      /* a kernel launch failed */
#define LB_E_WORKSPACE (-5)   /* workspace missing or smaller than lb_linear_workspace_size() */
#define LB_E_UNSUPPORTED (-6) /* valid request this build does not implement */

/* formats */
#define LB_FMT_INT8_ROW 1
#define LB_FMT_INT4_G128 2
#define LB_FMT_Q8_0_G32 3
#define LB_FMT_Q4_0_G32 4
#define LB_FMT_FP8_E4M3 5 /* minifloats: apsi/precision.py:70-76 (OCP fp8 / MX fp6, fp4 element formats) */
#define LB_FMT_FP8_E5M2 6
#define LB_FMT_FP6_E3M2 7
#define LB_FMT_FP6_E2M3 8
#define LB_FMT_FP4_E2M1 9

/* element types of weight inputs / dequantised outputs */
#define LB_DT_F32 0
#define LB_DT_BF16 1
#define LB_DT_F16 2

/* lb_linear_ex flags */
#define LB_LINEAR_STATIC_WEIGHTS 1u /* no kernel still running on the stream writes codes or scales */

/* device error word bits (lb_device_errors) */
#define LB_DEVERR_WAIT_TIMEOUT 1 /* a bounded device-side wait (mbarrier) gave up; the output is invalid */
#define LB_DEVERR_PEER_TIMEOUT 2 /* lb_rank_barrier gave up waiting for another rank; its output is incomplete */

/* ---------------------------------------------------------------------------------------------- runtime */

/* LB_VERSION of the loaded library.  Replaces nothing in the reference (library identity). */
int lb_version(void);

/* Message of the calling thread's most recent failed call ("" if none). */
const char* lb_last_error(void);

/* Checks that `device` is compute capability 10.x and caches its SM count and L2 size.
 * Replaces hub_gpu.runner() device selection / Runner.__init__ kernel load (apsi/hub_gpu.py:1772-1796,
 * 1366-1395).  Compute calls call it implicitly for the current device. */
int lb_init(int device);

/* Reads and clears the device error word of the current device (LB_DEVERR_* bits).  Synchronises
 * `stream` first.  Replaces the CUresult check after launches (apsi/native/cuda.py:213-223). */
int lb_device_errors(void* stream, int* bits_out);

/* ---------------------------------------------------------------------------------------------- quantise */

/* int8, one absmax/127 scale per output row.  w: [N, K] in `w_dtype` (LB_DT_F32 or LB_DT_BF16).
 * codes: int8 [N, K]; scale16: binary16 [N]; scale32 (may be NULL): float [N] -- the reference's float32
 * scale, bit-exact.  Codes are bit-exact with precision.quantize(W, "int8", axis=0).
 * Replaces precision.quantize / _scale_for for fmt int8, axis 0 (apsi/precision.py:205-246). */
int lb_quant_int8_rows(const void* w, int w_dtype, int64_t N, int64_t K, int8_t* codes, uint16_t* scale16,
                       float* scale32, void* stream);

/* int4, one absmax/7 scale per 128 values along K (K % 128 == 0).  packed: uint8 [N, K/2];
 * scale16: binary16 [N, K/128]; scale32 (may be NULL): float [N, K/128].  Bit-exact with
 * precision.quantize(W.reshape(-1, 128), "int4", axis=0) (apsi/precision.py:168-172, 205-246). */
int lb_quant_int4_g128(const void* w, int w_dtype, int64_t N, int64_t K, uint8_t* packed, uint16_t* scale16,
                       float* scale32, void* stream);

/* ggml-style int8 / int4 with one float scale per 32 values along K (K % 32 == 0), in hub_gpu's device
 * word layout.  Bit-exact with hub_gpu.qnumpy + the quant8 / quant4 kernels' packing
 * (apsi/hub_gpu.py:1215-1241, 734-801; launched by Runner._quant, apsi/hub_gpu.py:1478-1481). */
int lb_quant_q8_0_g32(const void* w, int w_dtype, int64_t N, int64_t K, uint32_t* words, float* scale32,
                      void* stream);
int lb_quant_q4_0_g32(const void* w, int w_dtype, int64_t N, int64_t K, uint32_t* words, float* scale32,
                      void* stream);

/* ---------------------------------------------------------------------------------------------- dequantise */

/* The g32 rounding in one pass: out[N, K] (float32, 16-byte aligned) = clip(rint(w * inv), lo, hi) * scale
 * per block of 32 along K, with hub_gpu.qnumpy's float32 scale (fmt LB_FMT_Q8_0_G32 or LB_FMT_Q4_0_G32).
 * Bit-exact with lowbit.round_weights / round_weights_torch on the rows, signed zeros included
 * (apsi/lowbit.py:37-50, 62-94; apsi/hub_gpu.py:1215-1241). */
int lb_round_g32(int fmt, const void* w, int w_dtype, int64_t N, int64_t K, float* out, void* stream);

/* out[N, K] = code * scale in `out_dtype` (LB_DT_F32: the exact float32 product, as precision.dequantize;
 * LB_DT_BF16: that product rounded to nearest even).  `scales` are `scale_dtype`: LB_DT_F16 (the stored
 * binary16 scales) or LB_DT_F32 (the reference's float32 scales, which makes the result bit-exact with
 * precision.dequantize); the G32 formats take LB_DT_F32 only.  Replaces precision.dequantize
 * (apsi/precision.py:249-274) and Runner._deq / the deq4, deq8 kernels (apsi/hub_gpu.py:918-950, 1483-1489). */
int lb_dequant(int fmt, const void* codes, const void* scales, int scale_dtype, int64_t N, int64_t K, void* out,
               int out_dtype, void* stream);

/* ---------------------------------------------------------------------------------------------- minifloats */

/* Bytes of the packed codes of n values in minifloat format fmt (-1 for other formats). */
int64_t lb_minifloat_bytes(int fmt, int64_t n);

/* Minifloat quantisation of R x C values w (LB_DT_F32 / LB_DT_BF16, row-major): precision.quantize(x, fmt,
 * scale="auto", axis=0 | None) (apsi/precision.py:205-246, with _minifloat_encode 109-130 and _pack4 / _pack6
 * 168-192).  per_row != 0 (axis=0): scale32[r] = float32(max|row r| / fmt.max), 1.0 when that maximum is 0 or
 * NaN, and the values of row r are divided by it.  per_row == 0 (axis=None): absmax[0] receives max|x| over the
 * tensor (NaN when any value is NaN) and the values are divided by the float64 scale absmax / fmt.max (1.0 when
 * 0 or NaN), as the reference does with its Python-float scale.  Codes: round to nearest on the grid, ties to
 * the even code, saturation at +-fmt.max, sign of -0.0 kept, NaN to the format's NaN code; packed flat
 * (lb_minifloat_bytes(fmt, R*C) bytes).  codes 8-byte aligned. */
int lb_quant_minifloat(int fmt, const void* w, int w_dtype, int64_t R, int64_t C, int per_row, uint8_t* codes,
                       float* scale32, float* absmax, void* stream);

/* out[r, c] = value(code) * scale (one float32 multiply; LB_DT_F32 or LB_DT_BF16 out), scale = scale32[r]
 * (per_row != 0) or tensor_scale: precision.dequantize of a minifloat QTensor (apsi/precision.py:249-274). */
int lb_dequant_minifloat(int fmt, const uint8_t* codes, int64_t R, int64_t C, int per_row, const float* scale32,
                         float tensor_scale, void* out, int out_dtype, void* stream);

/* ---------------------------------------------------------------------------------------------- GGUF */

/* GGUF blocks of 32 float32 values (n a multiple of 32): kind 8 = Q8_0 (34 bytes per block: binary16
 * d = amax / 127, 32 int8 codes sign(y) * floor(|y| + 0.5) of y = x / d), kind 4 = Q4_0 (18 bytes per block:
 * binary16 d = x[first argmax |x|] / -8, codes min(15, trunc(x / d + 8.5)), value j in the low and value j + 16
 * in the high nibble of byte j); float32 arithmetic as the reference's writer.  Replaces the GGUF codec of
 * modelio.save_gguf (apsi/modelio.py:56-81, _q8_0 / _q4_0); finite inputs. */
int lb_gguf_encode(int kind, const float* x, int64_t n, uint8_t* blocks, void* stream);

/* float32 values d * code of GGUF Q8_0 / Q4_0 blocks (apsi/modelio.py:84-95, _dq8_0 / _dq4_0). */
int lb_gguf_decode(int kind, const uint8_t* blocks, int64_t n, float* out, void* stream);

/* ---------------------------------------------------------------------------------------------- norm */

/* RMSNorm of activation rows, the prologue of a normalised projection: out[m, k] = bf16(x[m, k] *
 * (1 / sqrt(mean_k x[m, :]^2 + eps)) * (w[k] + off)), float32 arithmetic.  x, out: bf16 [M, K] (may alias);
 * w: [K] in w_dtype (LB_DT_F32 or LB_DT_BF16).  Replaces hub_gpu's rms op and the norm prologue of the
 * gemvq*n kernels behind _Base.linear(ln=...) (apsi/hub_gpu.py:1690-1693, 837-870, 1305-1315). */
int lb_rmsnorm(const void* x, int64_t M, int64_t K, const void* w, int w_dtype, float eps, float off, void* out,
               void* stream);

/* Bytes of device workspace lb_linear_rms needs for this shape (0 for M <= 16). */
int lb_linear_rms_workspace_size(int fmt, int64_t M, int64_t N, int64_t K, size_t* bytes);

/* A normalised projection: y (+)= rmsnorm(x; ln_w, eps, off) . deq(W)^T (+ bias), the result of lb_rmsnorm
 * followed by lb_linear_ex, bit for bit.  M <= 16: the norm runs inside the decode GEMV's activation staging
 * (one launch, no workspace, x itself is not modified); M > 16: lb_rmsnorm into the front of `workspace`, then
 * the GEMM.  ln_w: [K] in ln_dtype (LB_DT_F32 or LB_DT_BF16).  Replaces _Base.linear(x, W, ln=...) and its
 * gemvq*n kernels (apsi/hub_gpu.py:1305-1315, 837-870). */
int lb_linear_rms(int fmt, const void* x, int64_t M, int64_t K, const void* ln_w, int ln_dtype, float eps, float off,
                  const void* codes, const void* scales, int64_t N, const void* bias, int accumulate, void* y,
                  int64_t ldy, void* workspace, size_t ws_bytes, unsigned flags, void* stream);

/* The step between a decoder's fused QKV projection and its attention: split the [B T, (nh + 2 kvh) dh] bf16
 * projection into heads; optionally RMSNorm every q / k head (qn, kn: bf16 [dh] weights, or NULL); rotate the
 * first `rot` values of every q and k head with half-split pairs [a cos - b sin, b cos + a sin] (a = v[:rot/2],
 * b = v[rot/2:rot]; cos, sin: float32 tables [positions, rot/2]); write q[b, h, t, :] at
 * q + b q_sb + t q_st + h q_sh (elements) and k, v of token t into the caches at position p = *pos0 + t (pos0: a
 * device int64, so a captured graph can advance it) or start + t when pos0 is NULL:
 * cache[b, h, p, :] at b c_sb + h c_sh + p dh.  Float32 arithmetic, bf16 results.  Replaces hub_gpu's
 * qkv_prep op (apsi/hub_gpu.py:1547-1552, host form 1701-1723). */
int lb_qkv_prep(const void* qkv, int B, int T, int nh, int kvh, int dh, int rot, const float* cos, const float* sin,
                const void* qn, const void* kn, float eps, const int64_t* pos0, int64_t start, void* q,
                int64_t q_sb, int64_t q_st, int64_t q_sh, void* k_cache, void* v_cache, int64_t c_sb, int64_t c_sh,
                void* stream);
/* out[m, i] = act(gu[m, i]) * gu[m, I + i] for the fused [g | u] gate/up projection (bf16 [M, 2 I] -> [M, I]);
 * kind 0: silu g / (1 + exp(-g)); kind 1: gelu, tanh form.  Replaces hub_gpu's act_mul op
 * (apsi/hub_gpu.py:1598-1600, host form 1755-1762). */
int lb_act_mul(const void* gu, int64_t M, int64_t I, int kind, void* out, void* stream);


/* ---------------------------------------------------------------------------------------------- products */

/* Bytes of device workspace lb_linear needs for this shape (0 when none).  Replaces the scratch buffers of
 * _Base.ws (apsi/hub_gpu.py:1288-1295). */
int lb_linear_workspace_size(int fmt, int64_t M, int64_t N, int64_t K, size_t* bytes);

/* y[m, n] = sum_k x[m, k] * deq(W)[n, k] (+ bias[n]) (+ y[m, n] if accumulate), float32 accumulation,
 * bfloat16 output.  x: bf16 [M, K] (row stride K, 16-byte aligned); bias: bf16 [N] or NULL; y: bf16 with row
 * stride ldy.  M <= 16 runs the decode GEMV (integer codes exact in the tensor-core operands, scales applied
 * per group in float32; needs no workspace); larger M runs the tcgen05 GEMM (fp16 operands, x rescaled per
 * row by a power of two, float32 accumulation in tensor memory), whose converted activations live in
 * `workspace` (lb_linear_workspace_size() bytes, 256-byte aligned, contents need no initialisation).
 * x, codes and scales must be 16-byte aligned.  Formats: INT8_ROW and INT4_G128 (binary16 scales), FP8_E4M3
 * and FP8_E5M2 rows (codes uint8 [N, K], float32 scales [N]: the codes become exact fp16 operands), FP4_E2M1
 * rows (codes [N, K/2] as lb_quant_minifloat packs them, K % 128 == 0, float32 scales [N]; the codes become
 * exact fp16 operands through the hardware e2m1 conversion), FP6_E3M2 and FP6_E2M3 rows for M <= 16 only
 * (codes [N, 3K/4] as lb_quant_minifloat packs them, K % 16 == 0, float32 scales [N]; a CUDA-core product, the
 * codes exact in fp16); the other formats, and fp6 with M > 16, return LB_E_UNSUPPORTED.
 * Replaces precision.qmatmul / models.qlinear (apsi/precision.py:294-299, apsi/models.py:302-308) and
 * _Base.linear -> Runner.gemv / Runner.gemm with bias and acc (apsi/hub_gpu.py:1305-1315, 1491-1528). */
int lb_linear(int fmt, const void* x, int64_t M, int64_t K, const void* codes, const void* scales, int64_t N,
              const void* bias, int accumulate, void* y, int64_t ldy, void* workspace, size_t ws_bytes,
              void* stream);

/* lb_linear with flags.  LB_LINEAR_STATIC_WEIGHTS: the caller guarantees that no kernel still running on
 * `stream` writes `codes` or `scales` (true for weights quantised before the previous launch); the decode
 * GEMV is then launched with programmatic dependent launch and starts streaming weights while the previous
 * kernel finishes (x and y still wait for it).  Replaces the same reference call sites as lb_linear; the
 * overlap itself has no reference counterpart. */
int lb_linear_ex(int fmt, const void* x, int64_t M, int64_t K, const void* codes, const void* scales, int64_t N,
                 const void* bias, int accumulate, void* y, int64_t ldy, void* workspace, size_t ws_bytes,
                 unsigned flags, void* stream);

/* A weight prepared for repeated decode products (M <= 16).  lb_weight_create checks the format, codes, scales
 * and shape once, as lb_linear_ex would, on the current device, and encodes the tensor maps of the weight
 * stream once.  lb_weight_linear(w, x, M, y, ldy, flags, stream) then gives the bits of
 * lb_linear_ex(fmt, x, M, K, codes, scales, N, NULL, 0, y, ldy, NULL, 0, flags, stream) with fewer host
 * operations per call: it checks x, y, M and the device (the one the weight was prepared on) and launches.
 * M above 16 returns LB_E_UNSUPPORTED (the GEMM needs lb_linear's workspace).  The handle keeps the pointers,
 * not the memory: codes and scales must stay allocated until lb_weight_destroy.  It is the per-call path of
 * precision.qmatmul on one QTensor (apsi/precision.py:294-299, decode products of apsi/hub_gpu.py:1305-1315),
 * which has no separate preparation step in the reference. */
typedef struct lb_weight lb_weight;
int lb_weight_create(int fmt, const void* codes, const void* scales, int64_t N, int64_t K, lb_weight** out);
int lb_weight_linear(const lb_weight* w, const void* x, int64_t M, void* y, int64_t ldy, unsigned flags,
                     void* stream);
int lb_weight_destroy(lb_weight* w);

/* Bytes of the fixed device scratch behind lb_linear_noalloc (16 MiB + 64 KiB: the prefill path fits while
 * lb_linear_workspace_size(fmt, M, N, K) <= this, e.g. M = 2048, K = 4096). */
#define LB_NOALLOC_SCRATCH_BYTES 16842752

/* lb_linear without a workspace argument, allocating nothing: the prefill path (M > 16) uses one file-scope
 * device array per device instead (nothing in it needs to start at zero).  For callers that cannot allocate
 * at the call: engines whose free HBM is all handed to their own pool, loops that must not take the
 * synchronisation of cudaMalloc/cudaFree, bindings with no device allocator.  Shapes whose workspace exceeds
 * LB_NOALLOC_SCRATCH_BYTES fail with LB_E_WORKSPACE.  The array is reserved on every device where the library's
 * kernels are loaded (whether or not this entry point is called) and held until the process exits.  Calls
 * that overlap in time on one device (two streams or threads) race on the shared scratch; calls in order on one
 * stream are safe.  The scratch address is looked up on the first call in each CUDA context of a device (the
 * primary context, or a context made current through the driver API; a context re-created after
 * cudaDeviceReset counts as new): make that call outside stream capture.  No counterpart in the reference. */
int lb_linear_noalloc(int fmt, const void* x, int64_t M, int64_t K, const void* codes, const void* scales,
                      int64_t N, const void* bias, int accumulate, void* y, int64_t ldy, void* stream);

/* ---------------------------------------------------------------------------------------------- multi-GPU */

/* Reassembles column shards after an all-gather: src [G][M][Nl] (rank-major, bf16) -> dst [M][G*Nl].
 * No reference counterpart (the reference has no multi-GPU inference, apsi/hub_gpu.py:1772-1796). */
int lb_interleave_cols(const void* src, int G, int64_t M, int64_t Nl, void* dst, void* stream);

/* Bytes of a CUDA IPC memory handle as lb_peer_alloc writes it. */
#define LB_IPC_HANDLE_BYTES 64
/* Maximum ranks of a column-sharded layer. */
#define LB_MAX_RANKS 8

/* Device memory another process on the same node can map: `bytes` zeroed bytes on the current device, and the
 * CUDA IPC handle (LB_IPC_HANDLE_BYTES) the caller sends to the other ranks.  Free with lb_peer_free.
 * No reference counterpart (the reference has no multi-GPU path). */
int lb_peer_alloc(size_t bytes, void** ptr, void* handle);
/* Maps another process's lb_peer_alloc buffer into this process (peer access over NVLink); unmap with
 * lb_peer_close.  A handle from this same process cannot be opened. */
int lb_peer_open(const void* handle, void** ptr);
int lb_peer_close(void* ptr);
int lb_peer_free(void* ptr);

/* The column-sharded product with its gather fused in: this rank holds rows [rank Nl, (rank + 1) Nl) of the
 * layer's codes and scales (its own lb_quant_* output) and computes y[:, rank Nl + n] for n < Nl, storing each
 * value into EVERY rank's full output y_ranks[g] ([M, ldy] bf16, ldy >= G Nl; y_ranks is a host array of G
 * device pointers, the other ranks' buffers opened with lb_peer_open).  Same arithmetic as lb_linear on the
 * whole layer, so the assembled output is bit-identical to it; bias (bf16 [Nl], this rank's slice) as there;
 * no accumulate.  Call lb_rank_barrier afterwards before any rank reads its y.  Replaces the N-sharded linear
 * plus ncclAllGather of the scope's multi-GPU row; no reference counterpart. */
int lb_linear_sharded(int fmt, const void* x, int64_t M, int64_t K, const void* codes, const void* scales,
                      int64_t Nl, const void* bias, void* const* y_ranks, int G, int rank, int64_t ldy,
                      void* workspace, size_t ws_bytes, unsigned flags, void* stream);
/* Cross-rank barrier on `stream`: makes this rank's earlier stores (its lb_linear_sharded outputs) visible to
 * every rank, marks this rank's arrival with `epoch` in every rank's flag array and waits until all ranks have
 * arrived.  flags_ranks: host array of G device pointers, rank g's array of G uint32 (an lb_peer_alloc buffer,
 * zeroed; the others opened with lb_peer_open).  `epoch` starts at 1 and grows by one per barrier on every rank;
 * epoch 0 takes the next epoch from a counter in word G of this rank's array (arrays of G + 1 words), which keeps
 * barriers captured in a CUDA graph in step across replays.  The wait gives up after timeout_ms (0: 2000 ms) and
 * sets LB_DEVERR_PEER_TIMEOUT (read with lb_device_errors). */
int lb_rank_barrier(uint32_t* const* flags_ranks, int G, int rank, uint32_t epoch, uint32_t timeout_ms, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* APSI_LOWBIT_H */

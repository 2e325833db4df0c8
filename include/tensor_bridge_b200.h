/*
 * tensor_bridge_b200.h -- C ABI of the B200 (sm_100a) decode + GEMM path.
 *
 * The reference (tensor-bridge) exposes its hot path as C++ __global__
 * kernels that callers forward-declare and launch themselves
 * (bench/bench.cu:20-23, bench/bench_fused.cu:25-31,
 * bench/bench_formats.cu:30).  This header replaces those launch sites with
 * plain C entry points.  Conventions shared by every entry point:
 *
 *   - all pointers are DEVICE pointers owned by the caller, except where a
 *     parameter says "host";
 *   - every call is asynchronous on the given stream (NULL = legacy default
 *     stream, which is what the reference uses) and returns a status; a
 *     non-TB_OK status means nothing was launched;
 *   - matrices are row-major.  D[M x N] = A[M x K] * B^T with B stored
 *     [N x K] -- the reference's layout for gemm_fp16_wmma (A row-major,
 *     B "col-major K x N", src/gemm.cu:44-52).  For the weight-only case A is
 *     the quantized weight [out_features x in_features] and B the FP16
 *     activations [tokens x in_features], so N = tokens;
 *   - any M, N >= 1 is accepted (the reference needs multiples of 16); K
 *     must be a multiple of 16 (32 for packed FP4);
 *   - decoded values are bit-identical to the reference's conversion
 *     primitives (include/tensor_bridge/{fp8,fp4,bf16,tf32}.h), and GEMMs
 *     accumulate FP32 products of those FP16 values;
 *   - the library keeps no state besides cached launch attributes and a
 *     per-device error word (tb_device_error), and is safe to call from
 *     several host threads on different streams.
 */
#ifndef TENSOR_BRIDGE_B200_H
#define TENSOR_BRIDGE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t / CUstream. */
typedef struct CUstream_st* tb_stream_t;

typedef enum tb_status {
    TB_OK = 0,
    TB_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad enum, negative size */
    TB_ERR_SHAPE = 2,            /* shape not supported by this entry point */
    TB_ERR_ALIGNMENT = 3,        /* pointer or row pitch not aligned as required */
    TB_ERR_CUDA = 4,             /* a CUDA runtime or driver call failed */
    TB_ERR_LAUNCH = 5,           /* kernel launch failed */
    TB_ERR_TIMEOUT = 6,          /* a device-side bounded wait expired */
    TB_ERR_UNSUPPORTED = 7,      /* device is not sm_100, or format not supported here */
    TB_ERR_WORKSPACE = 8,        /* workspace missing or too small */
    TB_ERR_NCCL = 9              /* NCCL unavailable or an NCCL call failed */
} tb_status;

/* Storage formats.  Element counts are in values, not bytes. */
typedef enum tb_format {
    TB_FMT_F16 = 0,          /* IEEE binary16, 2 bytes */
    TB_FMT_E4M3 = 1,         /* FP8 E4M3, 1 byte (include/tensor_bridge/fp8.h) */
    TB_FMT_E5M2 = 2,         /* FP8 E5M2, 1 byte */
    TB_FMT_E2M1 = 3,         /* FP4 E2M1 packed two per byte, FIRST value in the HIGH
                                nibble (reference order, fp4.h:37-43) */
    TB_FMT_E2M1_UNPACKED = 4,/* FP4 E2M1 one value per byte in the low nibble (the
                                reference's decode_fp4_to_half input,
                                bench/bench_formats.cu:51-56) */
    TB_FMT_BF16 = 5,         /* bfloat16 bits, 2 bytes */
    TB_FMT_TF32 = 6,         /* TF32 carried in a 32-bit word (tf32.h:22) */
    TB_FMT_E2M1_HW = 7       /* FP4 E2M1 packed two per byte, FIRST value in the LOW
                                nibble (tensor-core order); native GEMM only */
} tb_format;

typedef enum tb_out_type {
    TB_OUT_F32 = 0,          /* FP32 output (the reference's only output type) */
    TB_OUT_F16 = 1           /* FP16 output, round-to-nearest-even */
} tb_out_type;

/* ---- status and device checks ------------------------------------------ */

/* Human-readable name of a status. */
const char* tb_status_string(tb_status s);

/* Detail of the most recent failure on the calling host thread ("" if none). */
const char* tb_last_error(void);

/* TB_OK if `device` is an sm_100 GPU this library was built for. */
tb_status tb_device_supported(int device);

/* Read (and optionally clear) the error word that kernels set when a bounded
 * device-side wait expires.  Synchronises the device.  *code = 0 means none. */
tb_status tb_device_error(int* code, int clear);

/* ---- decode streamers ---------------------------------------------------- */

/* dst[i] = decode(src[i]) as FP16 bits, i < n.  Bit-exact to the reference
 * primitive of `fmt`: fp8_e4m3_to_half (fp8.h:23-31), fp8_e5m2_to_half
 * (fp8.h:34-39), fp4_e2m1_to_half (fp4.h:33-35; packed order fp4.h:37-43),
 * bf16_to_half (bf16.h:22-34), tf32_to_half (tf32.h:22-34).  TB_FMT_F16 is a
 * copy.  Replaces the per-element decode kernels of src/gemm.cu:25-30 and
 * bench/bench_formats.cu:33-56 (their A half). */
tb_status tb_decode(tb_format fmt, const void* src, uint16_t* dst, size_t n, tb_stream_t stream);

/* Decode and transpose: src is [rows x cols] row-major in `fmt`, dst is
 * [cols x rows] row-major FP16.  Replaces the B half of the reference decode
 * kernels, which write B16[col*K + k] from B[k*N + col] (src/gemm.cu:29).
 * Packed FP4 needs an even `cols`. */
tb_status tb_decode_transposed(tb_format fmt, const void* src, uint16_t* dst,
                               int rows, int cols, tb_stream_t stream);

/* Block-scaled FP4 (the NVFP4 layout that fp4.h:6 names; the reference has no
 * kernel for it): dst[i] = e2m1(code i) * e4m3(scales[i / 16]) as FP16 bits,
 * i < n, n a multiple of 16.  `src` holds the codes packed two per byte in
 * the reference order (element 2j in the HIGH nibble of byte j, fp4.h:37-43;
 * codes as fp4_e2m1_to_half, fp4.h:33-35); `scales` holds one byte per 16
 * consecutive values, so a [rows x cols] matrix (cols a multiple of 16) has
 * [rows x cols/16] row-major scales.  Scale bytes are OCP E4M3 with
 * subnormals (exponent 0: m * 2^-9); 0x7F and 0xFF are NaN and give 0x7E00.
 * Every product is an FP16 value, so the decode is exact; a per-tensor FP32
 * scale goes into the GEMM's alpha (tb_gemm_f16). */
tb_status tb_decode_nvfp4(const uint8_t* src, const uint8_t* scales, uint16_t* dst, size_t n,
                          tb_stream_t stream);

/* Reference-shaped decode entry points: A [M x K] decoded straight into
 * A16 [M x K], B [K x N] decoded transposed into B16 [N x K].  Either pair may
 * be NULL to skip that operand.  Mirror, in order:
 *   decode_fp8_to_half      src/gemm.cu:25-30 (== decode_fp8_to_half_fmt,
 *                           bench/bench_formats.cu:45-50)
 *   decode_bf16_to_half     bench/bench_formats.cu:33-38
 *   decode_tf32_to_half     bench/bench_formats.cu:39-44
 *   decode_fp4_to_half      bench/bench_formats.cu:51-56 (one nibble per byte) */
tb_status tb_decode_fp8_to_half(const uint8_t* A, const uint8_t* B, uint16_t* A16, uint16_t* B16,
                                int M, int N, int K, tb_stream_t stream);
tb_status tb_decode_bf16_to_half(const uint16_t* A, const uint16_t* B, uint16_t* A16, uint16_t* B16,
                                 int M, int N, int K, tb_stream_t stream);
tb_status tb_decode_tf32_to_half(const uint32_t* A, const uint32_t* B, uint16_t* A16, uint16_t* B16,
                                 int M, int N, int K, tb_stream_t stream);
tb_status tb_decode_fp4_to_half(const uint8_t* A, const uint8_t* B, uint16_t* A16, uint16_t* B16,
                                int M, int N, int K, tb_stream_t stream);

/* ---- quantize (device-side; the reference quantizes on the host) -------- */

/* dst = Q(src[i] * scale) for i < n (scale 1: Q(src[i])), with Q the reference
 * quantizer of `fmt`: fp32_to_fp8_e4m3 (fp8.h:43-61), fp32_to_fp8_e5m2
 * (fp8.h:64-81), fp32_to_fp4_e2m1 (fp4.h:46-53; TB_FMT_E2M1 packs the first
 * value high, TB_FMT_E2M1_HW low), fp32_to_bf16 (bf16.h:37-48), fp32_to_tf32
 * (tf32.h:37-44), or FP16 round-to-nearest-even.  Replaces the host loops
 * `qA[i] = QUANT(hA[i] * ascale)` of bench/bench_formats.cu:64-65,131-132.
 * Bit-exact to the reference except for signaling-NaN inputs to the FP8
 * quantizers, whose reference result depends on the host's fminf. */
tb_status tb_quantize(tb_format fmt, const float* src, void* dst, size_t n, float scale, tb_stream_t stream);

/* *out (a device float) = max |src[i]| over the non-NaN values, the maxabs of
 * the per-tensor scale FORMAT_MAX / maxabs (bench/bench_formats.cu:128-130). */
tb_status tb_absmax(const float* src, size_t n, float* out, tb_stream_t stream);

/* ---- GEMMs (tcgen05 tensor cores, TMEM accumulators) --------------------- */

/* D = alpha * A * B^T.  A [M x K] FP16, B [N x K] FP16, FP32 accumulation.
 * Replaces gemm_fp16_wmma (src/gemm.cu:44-56), which is this call with
 * out = TB_OUT_F32 and alpha = 1. */
tb_status tb_gemm_f16(const uint16_t* A, const uint16_t* B, void* D, int M, int N, int K,
                      tb_out_type out, float alpha, tb_stream_t stream);

/* Weight-only fused GEMM: D = alpha * decode(A) * B^T, A stored in `a_fmt`
 * (E4M3, E5M2, E2M1, E2M1_UNPACKED, BF16, TF32), B FP16 [N x K].  The kernel
 * brings raw A tiles into shared memory with TMA and decodes them there to
 * FP16 operand tiles; decoded weights never reach global memory.  alpha is
 * the per-tensor dequantisation 1/scale that the reference applies on the
 * host (bench/bench_formats.cu:164).  The W_q @ X_fp16 case the reference
 * runs unfused (bench/bench_formats.cu:153-156); its fused kernel
 * gemm_fp8_fused_fp16 (src/gemm_fused.cu:24-49) quantizes both operands, see
 * tb_gemm_fp8_fused_fp16 for that one.
 * `workspace` (device, may be NULL when tb_gemm_fused_workspace returns 0)
 * holds split-K partial sums for short-and-wide shapes.
 * Few-token shapes (N <= 64; N <= 128 for the one-byte and FP4 formats)
 * run a kernel launched with programmatic dependent launch: it may start
 * while the previous kernel on `stream` runs, if that kernel allows it (the
 * same kernel and its split-K reduction do), and then reads one-byte and FP4
 * weights before that kernel has finished; B, D, the workspace and BF16/TF32
 * weights are accessed only after it has.  CUDA makes the previous
 * kernel's writes visible to this one only after the dependency wait, even
 * when that kernel never triggers early (tb_quantize included): so the
 * kernel launched just before this call on `stream` must not write its
 * one-byte or FP4 weights.  Put an event, a stream synchronisation, a copy
 * or any kernel launched without programmatic dependent launch between a
 * writer of the weights and the GEMM. */
tb_status tb_gemm_fused(tb_format a_fmt, const void* A, const uint16_t* B, void* D,
                        int M, int N, int K, tb_out_type out, float alpha,
                        void* workspace, size_t workspace_bytes, tb_stream_t stream);

/* Bytes of workspace tb_gemm_fused needs for this shape (0 if none). */
size_t tb_gemm_fused_workspace(tb_format a_fmt, int M, int N, int K);

/* No reference counterpart.  tb_gemm_fused without a workspace argument and
 * without allocating: split-K partial sums go to a fixed 20 MiB array compiled
 * into the library (one per device), for callers that may not allocate device
 * memory themselves, such as plugins under a runtime that owns all HBM through
 * its own pool and offers no workspace slot.  Shapes whose partial sums need
 * more than 20 MiB (tb_gemm_fused_workspace > 20 MiB; none on a 148-SM B200)
 * return TB_ERR_WORKSPACE.  The first call on each device does a one-time
 * set-up (looks up the array's device address) and should come before any
 * stream capture.  The 20 MiB are device memory that the CUDA driver commits
 * when it loads this part of the library on a device: at context creation
 * under CUDA_MODULE_LOADING=EAGER, otherwise (lazy loading, the default since
 * CUDA 12.2) during that first call, which then returns TB_ERR_CUDA if the
 * host has already reserved all free device memory.  A host that reserves its
 * memory pool up front should make one call (or run with eager loading)
 * before it reserves the pool.  All calls on a device share the array, which
 * keeps the last call's contents; calls that overlap in time on different
 * streams race on it. */
tb_status tb_gemm_fused_noalloc(tb_format a_fmt, const void* A, const uint16_t* B, void* D,
                                int M, int N, int K, tb_out_type out, float alpha,
                                tb_stream_t stream);

/* Both operands quantized, run natively by tcgen05 kind::f8f6f4 (qA @ qB of
 * bench/bench_formats.cu:140-150, without decoding to FP16):
 * D = alpha * A * B^T with A [M x K] in a_fmt and B [N x K] in b_fmt, each of
 * E4M3, E5M2 or E2M1_HW (mixed pairs allowed; with FP4, K % 128 == 0 and the
 * FP4 operand 32-byte aligned).  alpha
 * is 1/(scale_A*scale_B).  The tensor core reads E4M3 codes with exponent 0
 * as subnormals where the reference decoder flushes them to zero; the
 * reference quantizer (fp32_to_fp8_e4m3, fp8.h:58) never emits such codes.
 * Use tb_fp4_repack_hw to turn reference-packed FP4 into TB_FMT_E2M1_HW.
 * FP4 runs at the FP8 rate here (per-tensor scale, no block scales). */
tb_status tb_gemm_native(tb_format a_fmt, const void* A, tb_format b_fmt, const void* B, void* D,
                         int M, int N, int K, tb_out_type out, float alpha, tb_stream_t stream);

/* Block-scaled FP4 with both operands quantized (the NVFP4 layout that
 * fp4.h:6 names and docs/quantization-limits.md:14-33 argues for; the
 * reference has no kernel for it), run natively by tcgen05.mma
 * kind::mxf4nvf4.block_scale on pairs of SMs at the FP4 tensor rate:
 *   D[M x N] = alpha * (A .* SA) * (B .* SB)^T
 * A [M x K] and B [N x K] hold E2M1 codes packed two per byte with the FIRST
 * value in the LOW nibble (TB_FMT_E2M1_HW order; tb_fp4_repack_hw converts
 * reference-packed codes); SA [M x K/16] and SB [N x K/16] hold one scale
 * byte per 16 consecutive values of a row, row-major.  Scale bytes are
 * UE4M3: E4M3 with the sign bit clear, 0x00-0x7E (0x7F is NaN); a byte with
 * the sign bit set is outside this call's contract (tb_decode_nvfp4 accepts
 * every byte).  alpha carries the per-tensor FP32 scales (for two-level
 * quantization x = decode * g, alpha = gA * gB).  K % 256 == 0; all four
 * arrays 16-byte aligned; any M, N >= 1.  FP32 accumulation; FP32 or FP16
 * out.  Results equal, within FP32 accumulation error, the FP16 GEMM of the
 * operands decoded by tb_decode_nvfp4 (whose products are exact). */
tb_status tb_gemm_nvfp4(const uint8_t* A, const uint8_t* A_scales, const uint8_t* B, const uint8_t* B_scales, void* D,
                        int M, int N, int K, tb_out_type out, float alpha, tb_stream_t stream);

/* Swap the two nibbles of every byte: reference FP4 packing (first value high)
 * <-> tensor-core packing (first value low).  n_bytes bytes, may be in place. */
tb_status tb_fp4_repack_hw(const uint8_t* src, uint8_t* dst, size_t n_bytes, tb_stream_t stream);

/* Mirror of gemm_fp8_fused_fp16 (src/gemm_fused.cu:24-49): A [M x K] E4M3,
 * B [K x N] E4M3 (row-major, as the reference reads it), D [M x N] FP32, the
 * values of the reference's decode to FP16 and FP32-accumulated product.  Both
 * operands being E4M3, it runs on the FP8 tensor cores (tb_gemm_native)
 * without a decode: the codes of A, and of B transposed to [N x K], are
 * copied into `workspace` (M*K + N*K bytes rounded up, see
 * tb_gemm_fp8_fused_workspace) with the reference decoder's flush of the
 * subnormal codes to zero applied, so the tensor core's exact products are
 * those of the reference's FP16 operands.  A and the workspace 16-byte
 * aligned. */
tb_status tb_gemm_fp8_fused_fp16(const uint8_t* A, const uint8_t* B, float* D, int M, int N, int K,
                                 void* workspace, size_t workspace_bytes, tb_stream_t stream);
size_t tb_gemm_fp8_fused_workspace(int M, int N, int K);

/* ---- INT8 path (the reference's integer tensor-core path) ----------------
 *
 * E4M3 -> INT8 as src/gemm.cu:35-41 converts:
 * (int8_t)__float2int_rn(__half2float(fp8_e4m3_to_half(c)) * scale) -- the
 * reference decode to FP16, an FP32 product with the per-tensor scale (127 /
 * maxabs keeps every value in [-127, 127]), round to nearest even into an
 * int32 (clamped to the int32 range, NaN -> 0) and the low byte of that, so
 * out-of-range products wrap exactly as the reference's cast does. */

/* n codes, straight (decode_fp8_to_int8's A operand). */
tb_status tb_decode_e4m3_to_i8(const uint8_t* src, int8_t* dst, size_t n, float scale, tb_stream_t stream);

/* src [rows x cols] -> dst [cols x rows]: B8[col * K + k] of
 * decode_fp8_to_int8 (src/gemm.cu:39) with rows = K, cols = N. */
tb_status tb_decode_e4m3_to_i8_transposed(const uint8_t* src, int8_t* dst, int rows, int cols, float scale,
                                          tb_stream_t stream);

/* Mirror of decode_fp8_to_int8 (src/gemm.cu:35-41): A [M x K] straight into
 * A8, B [K x N] transposed into B8 [N x K]; either pair may be NULL. */
tb_status tb_decode_fp8_to_int8(const uint8_t* A, const uint8_t* B, int8_t* A8, int8_t* B8, int M, int N, int K,
                                float scale, tb_stream_t stream);

/* Replaces gemm_int8_wmma (src/gemm.cu:58-70): D [M x N] INT32 = A8 [M x K]
 * INT8 * B8^T, B8 [N x K] INT8 (the reference's column-major B), exact int32
 * accumulation on tcgen05.mma kind::i8.  K a multiple of 16, A and B 16-byte
 * aligned.  Any M, N (the reference needs multiples of 16). */
tb_status tb_gemm_i8(const int8_t* A, const int8_t* B, int32_t* D, int M, int N, int K, tb_stream_t stream);

/* Mirror of gemm_fp8_fused_int8 (src/gemm_fused.cu:52-81): A [M x K] and
 * B [K x N] E4M3, both converted to INT8 with `scale` as above, D [M x N]
 * INT32.  The converted operands go to `workspace`
 * (tb_gemm_fp8_fused_int8_workspace bytes), then the kind::i8 GEMM runs. */
tb_status tb_gemm_fp8_fused_int8(const uint8_t* A, const uint8_t* B, int32_t* D, int M, int N, int K, float scale,
                                 void* workspace, size_t workspace_bytes, tb_stream_t stream);
size_t tb_gemm_fp8_fused_int8_workspace(int M, int N, int K);

/* ---- column-sharded weight GEMM over NCCL -------------------------------- */
/* The reference is single-GPU; this is the B200 addition for weights too large
 * or slow for one GPU.  The weight's M rows (output features) are split into
 * world*chunks row blocks of Mc = M/(world*chunks) rows; rank r owns blocks
 * c*world + r for c = 0..chunks-1 (block-cyclic), stored back to back in
 * A_shard [chunks*Mc x K].  For each c the rank computes its block of D with
 * the fused kernel straight into D at global row (c*world + r)*Mc, then an
 * in-place NCCL all-gather of block group c (rows [c*world*Mc, (c+1)*world*Mc))
 * runs on `comm_stream` while block c+1 is computed on `stream`.  On return
 * (after both streams drain) every rank holds the full D [M x N].  `comm` is
 * an ncclComm_t from tb_nccl_comm_init; rank and world come from it.  M must
 * be a multiple of world*chunks*128. */
tb_status tb_gemm_sharded_fused(tb_format a_fmt, const void* A_shard, const uint16_t* B, void* D,
                                int M, int N, int K, tb_out_type out, float alpha, void* comm,
                                int chunks, tb_stream_t stream, tb_stream_t comm_stream);

/* The same sharded GEMM without a collective kernel: the fused kernel's
 * epilogue stores every finished output tile into each other rank's D through
 * peer-mapped memory (plain stores over NVLink), while the next tile's MMAs
 * run.  D is a buffer registered once with tb_peer_buffer_register; block
 * layout, shapes and the result are those of tb_gemm_sharded_fused, and
 * chunks = 1 is the natural choice (the overlap is per tile, not per block).
 * One process per GPU; the fused pair kernel must support the format (every
 * stored format except F16).  Collective: every rank calls it with the same
 * arguments, in the same order as its other calls on `comm`.  On `stream`, a
 * one-word NCCL all-reduce before the GEMM (no rank writes into a peer's D
 * before that peer has reached this call) and one after it (on completion
 * every rank's D is whole). */
tb_status tb_gemm_sharded_fused_p2p(tb_format a_fmt, const void* A_shard, const uint16_t* B, void* peer_buffer,
                                    int M, int N, int K, tb_out_type out, float alpha, int chunks,
                                    tb_stream_t stream);

/* Collective over `comm`: maps every rank's `bytes`-byte device buffer `buf`
 * (a cudaMalloc allocation or part of one, 16-byte aligned, the same size on
 * all ranks) into every other rank's process with CUDA IPC, and returns the
 * handle for tb_gemm_sharded_fused_p2p.  Synchronises `stream`.  A buffer
 * that one rank cannot export, or that does not match on every rank, or a
 * mapping that fails on one rank, fails the call on all ranks
 * (TB_ERR_INVALID_ARGUMENT or TB_ERR_CUDA), after the same collectives; a
 * failure before the exchange (an invalid argument, a 1 KB device allocation)
 * returns on that rank alone, like any collective called on some ranks only. */
tb_status tb_peer_buffer_register(void* comm, void* buf, size_t bytes, tb_stream_t stream, void** peer_buffer_out);
/* Collective: waits (on `stream`, synchronised) until every rank has reached
 * it, then unmaps the peers' buffers.  Call it on every rank before any rank
 * frees its buffer. */
tb_status tb_peer_buffer_release(void* peer_buffer, tb_stream_t stream);

/* NCCL plumbing (NCCL is loaded at run time; TB_ERR_NCCL if absent). */
tb_status tb_nccl_unique_id(uint8_t id_out[128]);
tb_status tb_nccl_comm_init(void** comm_out, int world, int rank, const uint8_t id[128]);
tb_status tb_nccl_comm_destroy(void* comm);

#ifdef __cplusplus
}
#endif

#endif /* TENSOR_BRIDGE_B200_H */

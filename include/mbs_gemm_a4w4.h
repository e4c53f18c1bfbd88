/*
 * mbs_gemm_a4w4.h -- C ABI of libmbs_gemm_kernel.so, the B200 (sm_100a)
 * MXFP4 "A4W4" GEMM and its quantiser.
 *
 * Every entry point is extern "C", takes plain device pointers, sizes and a
 * cudaStream_t passed as void*, never aborts, and returns an int status
 * (MBS_OK = 0).  Launches are asynchronous on the given stream; inputs are
 * borrowed for the duration of the stream work.
 *
 * Operand formats (the reference's input contract, unchanged):
 *   A        [M, K/2]  fp4x2 (uint8), row-major, element 2j in the low nibble
 *   B        [N, K/2]  fp4x2, preshuffled 16x16 ("flatB"):
 *              flatB(n,kp) = (n/16)*(K/64*512) + (kp/32)*512 + ((kp%32)/16)*256
 *                            + (n%16)*16 + kp%16
 *   A_scale  e8m0 (uint8), shuffled ("flatS"), Mpad x scaleN_pad bytes
 *   B_scale  e8m0, shuffled, roundup(N,32) x scaleN_pad bytes
 *              flatS(r,b) = (r%32)/16 + ((b%8)/4)*2 + (r%16)*4 + (b%4)*64
 *                           + (b/8)*256 + (r/32)*32*scaleN_pad
 *   out      bf16 [>= M, N] row-major; rows >= M are never written
 *   factors  optional uint8 [M] / [N]; byte b scales by f(b) = 1/(1 + b/256)
 *   scaleN_pad = roundup(ceil(K/32), 8), Mpad = roundup(M, 32)
 *
 * Shape rules: M >= 1, N % 16 == 0, K % 64 == 0 (the preshuffle needs whole
 * 64-element K tiles), all operand pointers 16-byte aligned.
 */
#ifndef MBS_GEMM_A4W4_H
#define MBS_GEMM_A4W4_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------- */
#define MBS_OK 0
#define MBS_ERR_INVALID_ARGUMENT 1  /* null pointer, non-positive size, bad pad */
#define MBS_ERR_UNSUPPORTED_SHAPE 2 /* N % 16 != 0, K % 64 != 0, too large     */
#define MBS_ERR_MISALIGNED 3        /* an operand is not 16-byte aligned        */
#define MBS_ERR_CUDA 4              /* CUDA runtime / driver error              */
#define MBS_ERR_WORKSPACE 5         /* caller workspace too small               */
#define MBS_ERR_DEVICE 6            /* no sm_100 device current                 */
#define MBS_ERR_DEVICE_TIMEOUT 7    /* a kernel wait ran out (see mbs_device_error) */

/* Short name of a status code. */
const char* mbs_status_string(int status);

/* Detail message of the last failing call on this host thread ("" if none). */
const char* mbs_last_error_message(void);

/* ---- GEMM ------------------------------------------------------------ */

/*
 * out[m][n] = bf16( (sum_k dq(A)[m][k] * dq(B)[n][k]) * f(AFactor[m]) * f(BFactor[n]) )
 *
 * Replaces the reference launcher `bool gemm_a4w4_mxfp4_launch(...)`
 * (kernel/gemm_a4w4.h:27-39, kernel/gemm_a4w4.hip:1044-1146) with the same
 * argument list.  Differences: returns an int status instead of bool, and
 * accepts MBS factors on every shape (the reference rejects factors when it
 * falls back to its single-wave kernel, kernel/gemm_a4w4.hip:1114-1115).
 * AFactor / BFactor may each be NULL (factor 1).
 *
 * Skinny and small problems use a stream-K schedule whose scratch buffer is
 * owned by the library: it is allocated with cudaMalloc on the first call per
 * (device, stream), so make that first call outside stream capture.  Callers
 * that manage memory themselves use mbs_gemm_a4w4_launch_ws.
 */
int gemm_a4w4_mxfp4_launch(const uint8_t* A, const uint8_t* B, const uint8_t* AScale,
                           const uint8_t* BScale, const uint8_t* AFactor, const uint8_t* BFactor,
                           void* out, int M, int N, int K, int Mpad, int scaleN_pad, void* stream);

/*
 * Bytes of scratch memory mbs_gemm_a4w4_launch_ws needs for this shape
 * (0 if the chosen schedule needs none).  Same call as the reference
 * launcher plus a caller workspace; no reference counterpart (the reference
 * kernel has no split-K/stream-K path).
 */
size_t mbs_gemm_a4w4_workspace_size(int M, int N, int K);

/*
 * Kernels one mbs_gemm_a4w4_launch_ws / gemm_a4w4_mxfp4_launch call of this
 * shape launches on the current device (2 on the CTA-pair path: the
 * scale-image pass and the GEMM; 1 otherwise).  Host-only, no CUDA work; -1
 * for a non-positive size.  No reference counterpart (the reference launches
 * one kernel per call).
 */
int mbs_gemm_a4w4_kernels_per_call(int M, int N, int K);

/*
 * Workspace layout shared by every schedule: the first
 * MBS_GEMM_WS_FLAG_BYTES bytes hold the stream-K completion flags (one word
 * per CTA), which must be zero when a launch starts; the rest is per-launch
 * scratch (stream-K partial tiles or the CTA-pair path's scale images) that
 * needs no initialisation.  Any workspace size returned by this library is
 * either 0 or at least MBS_GEMM_WS_FLAG_BYTES.
 */
#define MBS_GEMM_WS_FLAG_BYTES 4096

/*
 * As gemm_a4w4_mxfp4_launch, with caller-provided scratch memory.  The
 * workspace must be zero-filled before its first use; every launch that
 * completes leaves its flag words zero again, so the workspace can be reused
 * on the same stream, by any shape, without clearing.  A launch that stopped
 * with a device error (mbs_device_error) may leave flags set: zero the first
 * MBS_GEMM_WS_FLAG_BYTES bytes before reusing the workspace.  Launches that
 * overlap on the GPU must not share a workspace.
 */
int mbs_gemm_a4w4_launch_ws(const uint8_t* A, const uint8_t* B, const uint8_t* AScale,
                            const uint8_t* BScale, const uint8_t* AFactor, const uint8_t* BFactor,
                            void* out, int M, int N, int K, int Mpad, int scaleN_pad,
                            void* workspace, size_t workspace_bytes, void* stream);

/*
 * As mbs_gemm_a4w4_launch_ws, with an output epilogue:
 *   out[m][n] = bf16_rne( (acc[m][n] * (f(Af[m]) * f(Bf[n]))) * alpha + bias[n] )
 * each step an fp32 operation rounded to nearest (alpha = 1 and bias = NULL
 * give exactly the plain operator's result).  bias is bf16 [N] or NULL.
 * workspace may be NULL (then the library's own per-(device, stream)
 * workspace is used, as in gemm_a4w4_mxfp4_launch).  The alpha scale is the
 * output scaling of the reference's assembly kernel (asm_vs_wg_kernel.md:
 * 85-87); the bias has no reference counterpart.
 */
int mbs_gemm_a4w4_launch_ex(const uint8_t* A, const uint8_t* B, const uint8_t* AScale,
                            const uint8_t* BScale, const uint8_t* AFactor, const uint8_t* BFactor,
                            void* out, int M, int N, int K, int Mpad, int scaleN_pad, float alpha,
                            const void* bias, void* workspace, size_t workspace_bytes, void* stream);

/*
 * As mbs_gemm_a4w4_launch_ex, writing every output element to n_dst (1..8)
 * buffers at once: element (m, n) goes to out_dst[i] + m * ldc + n (bf16
 * elements) for each i, with ldc >= N and ldc % 8 == 0; out_dst is a host
 * array of device pointers, each 16-byte aligned.  For an N-sharded layer the
 * pointers are this GPU's copy of the full output and the peers' copies
 * (mapped through CUDA IPC or peer access), each offset to this rank's column
 * block, so the exchange of the output shards happens inside the GEMM's
 * epilogue, over NVLink, while the tensor cores work on the next tiles.  Each
 * kernel ends with a system-scope fence: once the launch has completed on
 * the stream (for example behind an NCCL barrier), every copy holds its
 * data.  No reference counterpart (the reference has no multi-GPU path);
 * replaces "GEMM, then NCCL all-gather" for BASELINE config[4].
 */
int mbs_gemm_a4w4_launch_multi(const uint8_t* A, const uint8_t* B, const uint8_t* AScale,
                               const uint8_t* BScale, const uint8_t* AFactor, const uint8_t* BFactor,
                               void* const* out_dst, int n_dst, long long ldc, int M, int N, int K,
                               int Mpad, int scaleN_pad, float alpha, const void* bias, void* workspace,
                               size_t workspace_bytes, void* stream);

/*
 * Dynamic-quant + GEMM in one call: bf16 activations x [M, ld_x] (row
 * stride ld_x elements, 16-byte aligned) are quantised to MXFP4 (the
 * per-1x32 arithmetic of mbs_quantize_mxfp4) and multiplied with the
 * preshuffled weight B, as mbs_quantize_mxfp4(x, shuffled) followed by
 * mbs_gemm_a4w4_launch_ws, with bit-identical results.  When the plan runs
 * on single CTAs (skinny and small M: decode, stream-K, cluster split-K)
 * the quantiser lives inside the GEMM kernel -- one launch.  Up to 8 rows,
 * each pipeline stage brings its bf16 rows and one warp converts them in
 * shared memory while the stage's weights stream in (no global A); more
 * rows are quantised by idle warps into the workspace while the producer
 * already streams the first weight stages, and the A loads wait for it (a
 * grid barrier, or for cluster split-K each CTA's own K range).  Large M
 * (CTA pairs) launches the stand-alone quantiser first.  The workspace (mbs_quant_gemm_a4w4_workspace_size,
 * 256-byte aligned) holds the quantised A and the GEMM's scratch; it must be
 * zero-filled before first use and is left reusable (including its first
 * MBS_GEMM_WS_FLAG_BYTES, as for mbs_gemm_a4w4_launch_ws).  Replaces the
 * quantise-then-GEMM sequence of the reference's drivers (bench_one.py:20-31,
 * test_gemm_a4w4.py:134-165) for BASELINE config[4]'s "fused dynamic-quant +
 * GEMM"; the reference has no fused kernel.
 */
size_t mbs_quant_gemm_a4w4_workspace_size(int M, int N, int K);
int mbs_quant_gemm_a4w4_launch(const void* x_bf16, int ld_x, const uint8_t* B, const uint8_t* BScale,
                               const uint8_t* AFactor, const uint8_t* BFactor, void* out, int M, int N, int K,
                               int scaleN_pad, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Macro-block-scaling variant: B's e8m0 scales are shared by 32-row x 32-K
 * blocks and given plainly as BScaleMacro[ceil(N/32)][mb_ld] with
 * mb_ld = roundup(K/32, 16).  A and A_scale are as above.  Spec-defined
 * extension; the reference has no such kernel.
 */
int mbs_gemm_a4w4_macro_launch_ws(const uint8_t* A, const uint8_t* B, const uint8_t* AScale,
                                  const uint8_t* BScaleMacro, const uint8_t* AFactor,
                                  const uint8_t* BFactor, void* out, int M, int N, int K, int Mpad,
                                  int scaleN_pad, int mb_ld, void* workspace,
                                  size_t workspace_bytes, void* stream);

/*
 * Allocation-free variant of mbs_gemm_a4w4_launch_ws for callers that may not
 * allocate device memory (for example a plugin whose host framework owns all
 * device allocations, or a loop where cudaMalloc's implicit synchronisation
 * is not acceptable).  No counterpart in the reference.
 *
 * Scratch comes from a static 8 MiB __device__ buffer inside the library,
 * which every GPU that loads the library keeps until the process exits.
 * Shapes whose schedule needs more scratch than that are rejected with
 * MBS_ERR_WORKSPACE (use mbs_gemm_a4w4_launch_ws for them); shapes that need
 * none never touch it.  The first call on each device looks up the buffer's
 * device address (cudaGetSymbolAddress), so make that first call before any
 * stream capture.  All calls share the one buffer and it keeps the last
 * call's contents: calls that overlap on the GPU (e.g. on two streams) race.
 * The caller still provides A, B, the scales, the factors and out.
 */
int mbs_gemm_a4w4_launch_noalloc(const uint8_t* A, const uint8_t* B, const uint8_t* AScale,
                                 const uint8_t* BScale, const uint8_t* AFactor,
                                 const uint8_t* BFactor, void* out, int M, int N, int K, int Mpad,
                                 int scaleN_pad, void* stream);

/*
 * Packed weights (optional, offline): the preshuffled weight and its shuffled
 * scales rearranged so that every (256-row tile, 256-element K stage) is one
 * contiguous 34 KB block -- the 32 KB tile in the exact shared-memory order
 * the tensor-core instruction reads, then its 2 KB of TMEM-ready scale
 * blocks.  The GEMM then streams each stage with a single bulk copy, which is
 * what skinny (decode) shapes need to approach HBM bandwidth.  Like the
 * reference's weight preshuffle this is a one-time step for static weights.
 * No reference counterpart.
 *
 * mbs_packed_weight_bytes: size of the packed buffer for an N x K weight.
 * mbs_pack_weight: B (flatB [N, K/2]) + BScale (flatS) -> packed.
 * mbs_gemm_a4w4_packed_launch_ws: as mbs_gemm_a4w4_launch_ws with the packed
 *   weight in place of B/BScale; workspace size from
 *   mbs_gemm_a4w4_packed_workspace_size.
 * mbs_quant_gemm_a4w4_packed_launch: dynamic quant + GEMM with the packed
 *   weight, as mbs_quant_gemm_a4w4_launch (bf16 x [M, ld_x], bit-identical
 *   to mbs_quantize_mxfp4 + mbs_gemm_a4w4_packed_launch_ws).  Up to 16 rows
 *   each pipeline stage converts its bf16 rows in shared memory (the packed
 *   scale blocks need no transpose, which frees a second converting warp);
 *   more rows run the stand-alone quantiser first.  Workspace (256-byte
 *   aligned, zero-filled before first use, left reusable) from
 *   mbs_quant_gemm_a4w4_packed_workspace_size.
 */
size_t mbs_packed_weight_bytes(int N, int K);
int mbs_pack_weight(const uint8_t* B, const uint8_t* BScale, int N, int K, int scaleN_pad,
                    uint8_t* packed, void* stream);
size_t mbs_gemm_a4w4_packed_workspace_size(int M, int N, int K);
int mbs_gemm_a4w4_packed_launch_ws(const uint8_t* A, const uint8_t* packedB, const uint8_t* AScale,
                                   const uint8_t* AFactor, const uint8_t* BFactor, void* out, int M,
                                   int N, int K, int Mpad, int scaleN_pad, void* workspace,
                                   size_t workspace_bytes, void* stream);
size_t mbs_quant_gemm_a4w4_packed_workspace_size(int M, int N, int K);
int mbs_quant_gemm_a4w4_packed_launch(const void* x_bf16, int ld_x, const uint8_t* packedB,
                                      const uint8_t* AFactor, const uint8_t* BFactor, void* out, int M,
                                      int N, int K, void* workspace, size_t workspace_bytes, void* stream);

/* ---- quantiser and layout kernels ------------------------------------ */

/*
 * bf16 [rows, K] (row stride ld_x elements) -> fp4x2 [rows, K/2] + e8m0 scales.
 * OCP MX per-1x32: scale = 2^(floor(log2 amax) - 2) (byte clamped at 0, 0xFF
 * for blocks holding Inf/NaN), values RNE onto the e2m1 grid saturating at 6.
 * shuffled == 0: scales plain [rows, K/32].  shuffled != 0: scales in the
 * flatS layout, roundup(rows,32) x scaleN_pad bytes, padding bytes = 127.
 * Replaces aiter's per_1x32 Triton quantiser (called at
 * test_gemm_a4w4.py:134-140, bench_one.py:20-25).  Requires K % 32 == 0.
 */
int mbs_quantize_mxfp4(const void* x_bf16, int rows, int K, int ld_x, uint8_t* fp4_out,
                       uint8_t* scale_out, int shuffled, void* stream);

/*
 * As mbs_quantize_mxfp4, fused with the MBS factor producer the reference
 * describes but does not ship (docs/kernel_advanced.md:120-129): per row,
 * factor_out[r] = b = the top 8 mantissa bits of 6.0 / max|x[r,:]| (IEEE
 * division, bits truncated; 0 for a zero, Inf or NaN max), and the row is
 * quantised as x * (1 + b/256) (exact in fp32; block scales from the fp32
 * amax).  Passing b as A_factor (or B_factor for weight rows) to the GEMM
 * multiplies the result by 1 / (1 + b/256), which undoes the scaling.
 */
int mbs_quantize_mxfp4_mbs(const void* x_bf16, int rows, int K, int ld_x, uint8_t* fp4_out,
                           uint8_t* scale_out, uint8_t* factor_out, int shuffled, void* stream);

/*
 * Macro-block quantiser: one scale per 32-row x 32-K block of x, written as
 * scale_out[ceil(rows/32)][roundup(K/32,16)] (padding 127).  No reference
 * counterpart (spec-defined).
 */
int mbs_quantize_mxfp4_macro(const void* x_bf16, int rows, int K, int ld_x, uint8_t* fp4_out,
                             uint8_t* scale_out, void* stream);

/*
 * Plain fp4x2 [N, K/2] -> flatB preshuffled [N, K/2].  Replaces aiter's
 * shuffle_weight(layout=(16,16)) (test_gemm_a4w4.py:141); layout decoded at
 * kernel/gemm_a4w4.hip:84-95.  Requires N % 16 == 0, K % 64 == 0.
 */
int mbs_shuffle_weight(const uint8_t* src, uint8_t* dst, int N, int K, void* stream);

/*
 * Plain scales [rows, K/32] -> flatS buffer roundup(rows,32) x scaleN_pad
 * (padding 127).  Replaces aiter's quant(shuffle=True) scale layout; decoded
 * at kernel/gemm_a4w4.hip:97-105.
 */
int mbs_shuffle_scales(const uint8_t* plain, uint8_t* shuffled, int rows, int K, void* stream);

/*
 * Measurement hook: on this host thread, record `before_main` / `after_main`
 * (cudaEvent_t passed as void*, or NULL to stop) on the launch stream right
 * before and right after the main GEMM kernel of every following GEMM call,
 * so a benchmark can time that kernel alone with CUDA events (a call may also
 * launch a small scale-layout kernel first).  No reference counterpart.
 */
int mbs_set_profile_events(void* before_main, void* after_main);

/*
 * Tuning knob: on this host thread, launch the following GEMMs on at most
 * max_ctas CTAs (0 = one per SM, the default), leaving SMs free for kernels
 * that must run at the same time, such as the NCCL kernels of an all-gather
 * overlapped with the GEMM.  Workspace sizes queried on this thread follow
 * the same limit.  No reference counterpart.
 */
int mbs_set_grid_limit(int max_ctas);

/*
 * Tuning and test hook: on this host thread, force parts of the schedule of
 * the following GEMM calls (and of the workspace-size and kernels-per-call
 * queries, which plan the same way), so that every schedule can be reached on
 * small shapes.  A field at its "auto" value keeps the planner's own choice;
 * ov == NULL clears every override.
 *   schedule   0 auto, 1 stream-K, 2 data-parallel
 *   grid       0 auto, else at most this many CTAs
 *   pair       -1 auto, 0 never CTA pairs, 1 CTA pairs whenever data-parallel
 *   swap       -1 auto, 1 weights as the 128-row operand when M <= 64
 *   pair_bn    0 auto, 256 or 384: CTA-pair tile width
 *   pair_wide  0 auto, else this many 384-wide column tiles, then 256-wide ones
 *   ksplit     -1 auto, 0 off, 2, 4 or 8: cluster split-K factor
 *   split_bn   0 auto (256), 128 or 256: split-K tile width (256 when M <= 64)
 * Returns MBS_ERR_INVALID_ARGUMENT (and changes nothing) for a value outside
 * these sets.  Replaces the reference's compile-time tile override
 * (-DMBS_FORCE_TILE_ENV, kernel/gemm_a4w4.hip:1094-1102) with an explicit
 * call, so the launch path reads no environment variable.
 */
typedef struct mbs_plan_override
{
    int schedule, grid, pair, swap, pair_bn, pair_wide, ksplit, split_bn;
} mbs_plan_override;
int mbs_set_plan_override(const mbs_plan_override* ov);

/*
 * Peer-memory plumbing for exchanging GEMM output shards between the GPUs of
 * one node (the N-sharded layer) with copy-engine
 * transfers over NVLink instead of SM kernels:
 *   mbs_ipc_alloc   cudaMalloc `bytes` on the current device and write its
 *                   CUDA IPC handle (64 bytes) to handle_out;
 *   mbs_ipc_open    map a peer's buffer from its handle (peer access enabled);
 *   mbs_ipc_close / mbs_ipc_free   undo the two;
 *   mbs_copy_async  one cudaMemcpyAsync of `bytes` between device pointers
 *                   (local or peer) on `stream`.
 * No reference counterpart (the reference has no multi-GPU path).
 */
int mbs_ipc_alloc(size_t bytes, void** ptr, void* handle_out);
int mbs_ipc_open(const void* handle, void** peer_ptr);
int mbs_ipc_close(void* peer_ptr);
int mbs_ipc_free(void* ptr);
int mbs_copy_async(void* dst, const void* src, size_t bytes, void* stream);

/*
 * Test hook for the failure path of the kernels' bounded waits: on this host
 * thread, while `on` != 0, the stream-K contributors of the following GEMM
 * calls write their partial tiles but never release their completion flags
 * (a flag that nothing sets).  The owner of each split tile then waits until
 * its limit (2 s of %globaltimer) runs out, records MBS_ERR_DEVICE_TIMEOUT in
 * the device error word and finishes its kernel without the partials, so the
 * output is wrong and mbs_device_error reports the timeout.  The wait is the
 * last step of the owner's kernel, with no copy or MMA in flight, and the
 * flag words stay zero.  No reference counterpart (the reference's only
 * failure path is its launcher's false return,
 * interface/gemm_a4w4_pybind.cpp:56-61).
 */
int mbs_set_withhold_release(int on);

/*
 * Sticky device-side error word of the current device: 0, or the code of a
 * kernel wait that ran out (MBS_ERR_DEVICE_TIMEOUT).  Synchronises the
 * device.  reset != 0 clears it.  No reference counterpart.
 */
int mbs_device_error(int* code_out, int reset);

/*
 * Diagnostic: the tensor-pipe peak of tcgen05.mma kind::mxf4 on the current
 * device, measured with every CTA pair issuing `groups` x 4 back-to-back
 * 256x256x64 pair MMAs (the prefill kernel's instruction) on operands
 * resident in shared memory and scales resident in TMEM.  Writes the
 * grid's TFLOP/s (CUDA events), cycles per MMA and the SM clock seen (MHz).
 * Blocks until done (synchronises `stream`).  groups in [16, 2^24].  This is
 * the roofline denominator a compute-bound GEMM is quoted against; the
 * reference has no counterpart (its MFMA probe, kernel/mfma_probe.hip, only
 * checks numerics).
 */
int mbs_mxf4_peak_probe(int groups, double* tflops, double* cycles_per_mma, double* sm_mhz, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MBS_GEMM_A4W4_H */

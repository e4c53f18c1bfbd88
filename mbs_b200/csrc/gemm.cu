// MXFP4 A4W4 GEMM for B200 (sm_100a): tcgen05.mma kind::mxf4 with e8m0
// block scales in TMEM, TMA-fed shared-memory pipeline, warp-specialised.
//
// Computes out[m][n] = bf16( sum_k dq(A)[m][k] dq(B)[n][k] * f(Af[m]) f(Bf[n]) )
// on the reference's input contract (plain row-major A, flatB-preshuffled B,
// flatS-shuffled e8m0 scales; kernel/gemm_a4w4.hip:19-25,84-105), the
// operation of the reference's gemm_a4w4_wg_kernel / gemm_a4w4_mfma_kernel
// (kernel/gemm_a4w4.hip:147-250, 344-1011).
//
// Roles in one 384-thread CTA (one CTA per SM, persistent):
//   warp 0      TMA producer: per K-stage (256 elements) loads the R tile
//               (MMA operand A, 128 rows), the C tile (MMA operand B, BN rows)
//               and both operands' raw scale bytes into one pipeline slot.
//   warp 1      TMEM allocator; lane 0 issues tcgen05.cp (scales -> TMEM) and
//               tcgen05.mma, and commits slot / accumulator barriers.
//   warp 2      scale transposer: rewrites the slot's raw scales (flatS or
//               macro-block layout) into the 32x16-byte blocks tcgen05.cp
//               copies to TMEM (row r of a 128-row block at byte
//               (r%32)*16 + (r/32)*4, one byte per 32-K group).
//   warps 4-11  epilogue: tcgen05.ld the fp32 accumulator, apply the MBS
//               factors, round to bf16 and store (or exchange stream-K partials).
//
// Operand roles.  Prefill (SWAP = false): R = activations A (plain rows,
// 128-byte-swizzled K-major tiles), C = weights B (flatB core matrices,
// no-swizzle K-major tiles).  Decode (SWAP = true, M <= 64): R = weights,
// C = activations, so the 128-row MMA dimension walks N and the small M sits
// in the MMA's N; the output is written transposed back to out[m][n].
//
// Shared-memory operand layouts the MMA reads:
//   plain     TMA box {128 B, rows} with 128-byte swizzle: row r at r*128 B,
//             8-row groups 1024 B apart (SBO), K step j at +32 B.
//   preshuf   the flatB buffer viewed as a 3-D tensor {256 B block of
//             16 rows x 16 B, row-tile (stride 8K), K chunk (stride 256)};
//             the box lands as [K chunk][row tile][16 rows x 16 B], i.e.
//             canonical no-swizzle K-major core matrices with
//             SBO = 128 B (8-row groups) and LBO = rows*16 B (K chunks).
//
// Schedules.  Data-parallel: CTA c takes tiles c, c+G, ...  Stream-K: the
// tiles x K-stages units are split evenly into G contiguous ranges; a tile cut
// between CTAs is finished by the CTA holding its first K-stage (the "owner",
// whose range ends there), which adds the fp32 partials the other CTAs (whose
// ranges start inside the tile) left in the workspace, flagged per CTA.
#include <cuda_bf16.h>

#include <cstring>
#include <mutex>
#include <unordered_map>

#include "common.h"
#include "mx_quant.cuh"
#include "ptx.cuh"

namespace mbs {
namespace gemm {

constexpr int BM = 128;          // MMA M: rows of the R operand per tile
constexpr int BK = 256;          // K elements per pipeline stage
constexpr int BKB = BK / 2;      // bytes per row per stage
constexpr int MMA_K = 64;        // K per tcgen05.mma kind::mxf4
constexpr int NUM_THREADS = 384;
constexpr int EPI_WARP0 = 4;
constexpr int NUM_EPI_WARPS = 8;
constexpr int NUM_EPI_THREADS = NUM_EPI_WARPS * 32;

constexpr int MAX_OUT = 8;  // output copies one launch writes (this GPU's and up to 7 peers')

struct Params
{
    int M, N, K;
    int tiles_r, tiles_c, k_stages, num_tiles;
    int sk;                // 1: stream-K over tiles x k_stages units
    long long sk_units;
    const uint8_t* a_factor;
    const uint8_t* b_factor;
    __nv_bfloat16* out;    // == outs[0]
    float* partials;       // [G][BN][BM] fp32, stream-K only
    unsigned* flags;       // [G], stream-K only; zero between launches
    unsigned* err;         // sticky device error word
    const uint8_t* packed_b;  // packed weights (C_PACKED configurations)
    int act_rows;          // rows per activation TMA box (the activation operand's tile rows, or M)
    float alpha;                  // output scale (1 = none)
    const __nv_bfloat16* bias;    // [N] added to every output row, or null
    int out_v8;                   // 1: `out` is 32-byte aligned, rows are stored 32 bytes per instruction
    int wide_c;                   // CTA pairs, 384-column configuration: column tiles [0, wide_c) are
                                  // 384 wide, the rest (up to tiles_c) 256 wide
    int img_b_blocks;             // ... 128-row blocks per K stage of the B scale images
    int ksplit;                   // single-CTA kernel, > 1: cluster split-K over clusters of ksplit CTAs
    int withhold_release;         // test hook: stream-K contributors never release their flags
    // Output copies: element (m, n) goes to outs[d] + m * ldc + n for every d < n_out (this GPU's
    // buffer and, for an N-sharded layer, peer GPUs' buffers reached over NVLink).
    long long ldc;
    int n_out;
    __nv_bfloat16* outs[MAX_OUT];
    // Fused activation quantiser (mbs_quant_gemm_a4w4_launch), single-CTA kernel only:
    // qmode 0 = A given; 1 = the grid quantises bf16 qx into qa / qsa (the A and A_scale
    // buffers the TMA maps read) behind a grid barrier (qbar); 2 = every CTA quantises
    // the A blocks of its own tile rows and K range (cluster split-K); 3 = each stage's
    // bf16 rows are quantised in shared memory (R_QUANT configurations).
    int qmode;
    int qx_ld;
    const __nv_bfloat16* qx;
    uint8_t* qa;
    uint8_t* qsa;
    int q_snp;
    unsigned* qbar;  // [arrived, departed], zero between launches
};

constexpr int align_up(int x, int a) { return (x + a - 1) / a * a; }

// R_ROWS_: rows of the R operand (A, non-swapped) actually loaded per stage.
// Skinny problems load only their M rows (32 or 64); the MMA still reads 128
// rows, the rest coming from whatever follows in shared memory, which only
// feeds accumulator rows that are never stored.
// C_PACKED_: the C operand (weights, non-swapped) comes from the packed
// weight format (pack_weight_kernel): per 256-row tile and K stage one
// contiguous block = the 32 KB tile in shared-memory order followed by its
// 2 KB of tcgen05.cp-ready scale blocks, loaded with one bulk copy.
// XQ_ (8 or 16; 0 = off): the activation rows (at most XQ_ of them) arrive
// as bf16 (a plain box of rows x BK values, 512 B per row, over the space of
// the A tile) and are quantised there in shared memory: the e2m1 codes go
// over the start of that staging, in the 128-byte-swizzled layout the MMA
// reads, the scales straight into the tcgen05.cp blocks (no raw activation
// scales, no global A).  XQ_ = 8: warp 2 converts; XQ_ = 16 (packed weights,
// whose scale blocks need no transpose): warps 2 and 3 convert 8 rows each.
constexpr int PACK_STAGE_BYTES = 256 * BKB + 4 * 512;

template <int BN_, bool SWAP_, bool W_MACRO_, int STAGES_, int R_ROWS_ = 128, bool C_PACKED_ = false,
          int XQ_ = 0>
struct Cfg
{
    static constexpr int BN = BN_;
    static constexpr bool SWAP = SWAP_;
    static constexpr int STAGES = STAGES_;
    static constexpr int R_ROWS = R_ROWS_;
    static constexpr bool C_PACKED = C_PACKED_;
    static constexpr int XQ = XQ_;
    static constexpr bool R_QUANT = XQ_ > 0;
    static_assert(R_ROWS == 128 || (!SWAP_ && (R_ROWS == 32 || R_ROWS == 64)), "R rows");
    static_assert(!C_PACKED || (!SWAP_ && !W_MACRO_ && BN_ == 256), "packed weights: non-swapped, BN 256");
    static_assert(XQ_ == 0 || ((XQ_ == 8 || (XQ_ == 16 && C_PACKED_)) && !SWAP_ && !W_MACRO_ && R_ROWS_ == 32),
                  "in-stage quantiser: 8 rows, or 16 with packed weights, on 32-row non-swapped tiles");
    static constexpr bool R_PRESHUF = SWAP;   // weights are the preshuffled operand
    static constexpr bool C_PRESHUF = !SWAP;
    static constexpr bool R_MACRO = SWAP && W_MACRO_;
    static constexpr bool C_MACRO = !SWAP && W_MACRO_;
    static constexpr int C_RB = BN >= 128 ? BN / 128 : 1;  // 128-row scale blocks of C

    static constexpr int R_DATA = R_ROWS * BKB;
    static constexpr int R_ROW_TX = R_QUANT ? BK * 2 : BKB;  // bytes the TMA brings per activation row
    // the A tile's space: its codes, or with the in-stage quantiser the bf16 rows they overwrite
    static constexpr int R_SPAN = XQ * BK * 2 > R_DATA ? XQ * BK * 2 : R_DATA;
    static constexpr int C_DATA = BN * BKB;
    static constexpr int R_RAW = R_QUANT ? 0 : R_MACRO ? (R_ROWS / 32) * 16 : (R_ROWS / 32) * 256;
    static constexpr int C_RAW = C_PACKED ? 0 : (C_MACRO ? (BN / 32) * 16 : (BN / 32) * 256);
    static constexpr int R_ATOM = 2 * 512;
    static constexpr int C_ATOM = 2 * C_RB * 512;

    // packed: [R data][C data][C atoms][R raw][R atoms] (C data + atoms contiguous)
    // else:   [R data][C data][R raw][C raw][R atoms][C atoms]
    static constexpr int R_DATA_OFF = 0;
    static constexpr int C_DATA_OFF = R_DATA_OFF + R_SPAN;
    static constexpr int R_RAW_OFF = C_PACKED ? C_DATA_OFF + C_DATA + C_ATOM : C_DATA_OFF + C_DATA;
    static constexpr int C_RAW_OFF = R_RAW_OFF + align_up(R_RAW, 128);
    static constexpr int R_ATOM_OFF = C_RAW_OFF + align_up(C_RAW, 128);
    static constexpr int C_ATOM_OFF = C_PACKED ? C_DATA_OFF + C_DATA : R_ATOM_OFF + R_ATOM;
    static constexpr int STAGE_END = C_PACKED ? R_ATOM_OFF + R_ATOM : C_ATOM_OFF + C_ATOM;
    static constexpr int STAGE_BYTES = align_up(STAGE_END, 1024);
    static constexpr uint32_t TX_BYTES = R_DATA + C_DATA + R_RAW + C_RAW + (C_PACKED ? C_ATOM : 0);
    static_assert(!C_PACKED || C_DATA + C_ATOM == PACK_STAGE_BYTES, "packed stage");

    static constexpr int SF_STAGE_COLS = 8 + 8 * C_RB;
    static constexpr int ACC_BUFS = (2 * BN + STAGES * SF_STAGE_COLS <= 512) ? 2 : 1;
    static constexpr int SF_BASE = ACC_BUFS * BN;
    static constexpr int TMEM_NEED = SF_BASE + STAGES * SF_STAGE_COLS;
    static constexpr int TMEM_COLS =
        TMEM_NEED <= 32 ? 32 : TMEM_NEED <= 64 ? 64 : TMEM_NEED <= 128 ? 128 : TMEM_NEED <= 256 ? 256 : 512;
    static_assert(TMEM_NEED <= 512, "TMEM budget");

    // barriers: full, sfready, empty [STAGES]; acc_full, acc_empty [2]; qready; xfull [STAGES when
    // R_QUANT]; tmem slot; abort
    static constexpr int XBARS = R_QUANT ? STAGES : 0;
    static constexpr int BAR_BYTES = (3 * STAGES + 5 + XBARS) * 8 + 16;
    static constexpr int EPI_BYTES = (BM + 2 * BN) * 4;  // epilogue factor + bias staging
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + BAR_BYTES + EPI_BYTES + 1024;  // +1024 alignment slack
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
    static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");

    // Cluster split-K: a CTA's buffer of S partial slices (S <= 8, each
    // 128 / S rows + 1 pad row of BN / 4 16-byte column groups) lives in the
    // idle pipeline stages.
    static constexpr bool SPLIT_OK = !SWAP && (R_ROWS + 8) * (BN / 4) * 16 <= STAGES * STAGE_BYTES;
};

// ------------------------------------------------------------------ schedule
struct Work
{
    int tile, k0, k1;
};

// floor(a * b / c) for non-negative operands; 32-bit division when the
// product fits (the common case), which costs far less than the 64-bit one.
__device__ __forceinline__ long long muldiv(long long a, long long b, long long c)
{
    const unsigned long long prod = (unsigned long long)a * (unsigned long long)b;
    if (prod <= 0xFFFFFFFFull && (unsigned long long)c <= 0xFFFFFFFFull)
        return (long long)((unsigned)prod / (unsigned)c);
    return (long long)(prod / (unsigned long long)c);
}

__device__ __forceinline__ long long sk_start(const Params& p, int c)
{
    return muldiv(c, p.sk_units, gridDim.x);
}

// Last CTA whose stream-K range starts before unit `tile_end`: sk_start(c) <
// tile_end  <=>  c * units < tile_end * G.
__device__ __forceinline__ int sk_last_starting_before(const Params& p, long long tile_end)
{
    const long long last = muldiv(tile_end * gridDim.x - 1, 1, p.sk_units);
    return last < (long long)gridDim.x - 1 ? (int)last : (int)gridDim.x - 1;
}

// idx-th work item of this CTA; false when exhausted.
__device__ __forceinline__ bool get_work(const Params& p, int idx, Work& w)
{
    if (p.ksplit > 1)
    {
        // cluster split-K: the ksplit CTAs of a cluster (consecutive blockIdx.x,
        // cluster rank = blockIdx.x % ksplit) share one tile, rank r taking K
        // stages [r * k_stages / ksplit, (r + 1) * k_stages / ksplit)
        if (idx > 0) return false;
        const int rank = (int)(blockIdx.x % (unsigned)p.ksplit);
        w.tile = (int)(blockIdx.x / (unsigned)p.ksplit);
        w.k0 = (int)muldiv(rank, p.k_stages, p.ksplit);
        w.k1 = (int)muldiv(rank + 1, p.k_stages, p.ksplit);
        return true;
    }
    if (!p.sk)
    {
        const long long t = (long long)blockIdx.x + (long long)idx * gridDim.x;
        if (t >= p.num_tiles) return false;
        w.tile = (int)t;
        w.k0 = 0;
        w.k1 = p.k_stages;
        return true;
    }
    const long long s = sk_start(p, blockIdx.x);
    const long long e = sk_start(p, blockIdx.x + 1);
    const int ks = p.k_stages;
    const long long t0 = muldiv(s, 1, ks);
    if (idx == 0)
    {
        if (s >= e) return false;
        w.tile = (int)t0;
        w.k0 = (int)(s - t0 * ks);
        w.k1 = (int)(w.k0 + (e - s) < ks ? w.k0 + (e - s) : ks);
        return true;
    }
    const long long u = (t0 + idx) * ks;
    if (u >= e) return false;
    w.tile = (int)(t0 + idx);
    w.k0 = 0;
    w.k1 = (int)(e - u < ks ? e - u : ks);
    return true;
}

__device__ __forceinline__ void raise_error(const Params& p, volatile int* abort_flag)
{
    *abort_flag = 1;
    atomicExch(p.err, (unsigned)MBS_ERR_DEVICE_TIMEOUT);
}

// One 16-column (32-byte) chunk of output row m, columns [n, n + 16), into
// every output copy.  The copy index stays a compile-time constant (the loop
// is unrolled over MAX_OUT and cut at n_out), so the pointers come straight
// from the parameter bank.
__device__ __forceinline__ void store_chunk16(const Params& p, long long m, int n, const uint32_t* w)
{
    const long long off = m * p.ldc + n;
#pragma unroll
    for (int d = 0; d < MAX_OUT; ++d)
    {
        if (d >= p.n_out) break;
        __nv_bfloat16* dst = p.outs[d] + off;
        if (p.out_v8)
        {
            st_global_v8(dst, w[0], w[1], w[2], w[3], w[4], w[5], w[6], w[7]);
        }
        else
        {
            uint4* d4 = reinterpret_cast<uint4*>(dst);
            d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
            d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
    }
}

// Debug instrumentation (build with -DMBS_TIMING=1): cycles per role and
// wait site, summed per CTA into g_mbs_timing and read with mbs_timing_read.
//   0 producer waits on `empty`      1 MMA waits on `acc_empty`
//   2 MMA waits on `full`            3 MMA waits on `sfready`
//   4 transposer waits on `full`     5 transposer work
//   6 epilogue waits on `acc_full`   7 epilogue work
//   8 stream-K owner flag wait       9 CTA lifetime (thread 0)
//  10 stages issued (producer)      11 MMA issue work
//  12 split-K: first cluster barrier 13 split-K: push + second barrier
//  14 kernel start -> past griddep_wait  15 split-K: finish
#ifndef MBS_TIMING
#define MBS_TIMING 0
#endif
#if MBS_TIMING
__device__ unsigned long long g_mbs_timing[16];
// per CTA (single-CTA kernel): SM id, start after the dependent-launch wait,
// last stage issued by the producer, CTA end (%globaltimer ns), stages issued
__device__ unsigned long long g_mbs_cta[1024 * 5];
#define MBS_TSTART() const long long _mbs_t0 = clock64()
#define MBS_TADD(acc, b) (acc)[b] += (unsigned long long)(clock64() - _mbs_t0)
#define MBS_TFLUSH(acc)                                              \
    do                                                               \
    {                                                                \
        for (int _b = 0; _b < 16; ++_b)                              \
            if ((acc)[_b]) atomicAdd(&g_mbs_timing[_b], (acc)[_b]);  \
    } while (0)
#else
#define MBS_TSTART() \
    do               \
    {                \
    } while (0)
#define MBS_TADD(acc, b) \
    do                   \
    {                    \
    } while (0)
#define MBS_TFLUSH(acc) \
    do                  \
    {                   \
    } while (0)
#endif

// f(b) = 1 / (1 + b/256): b fills the top 8 mantissa bits of 1.0f; the
// reciprocal is IEEE round-to-nearest (test_gemm_a4w4.py:47-51).
__device__ __forceinline__ float byte_to_factor(uint32_t b)
{
    return __frcp_rn(__uint_as_float(0x3F800000u | (b << 15)));
}

// Byte offset of scale (r, b) in a flatS buffer (kernel/gemm_a4w4.hip:97-105).
__device__ __forceinline__ long long flat_s_offset(int r, int b, int snp)
{
    const int r32 = r & 31, b8 = b & 7;
    return (long long)(r32 >> 4) + (long long)(b8 >> 2) * 2 + (long long)(r32 & 15) * 4 +
           (long long)(b8 & 3) * 64 + (long long)(b >> 3) * 256 + (long long)(r >> 5) * 32 * snp;
}

// Fused activation quantiser: the octets (8 consecutive K values) o in
// [0, nrows * width) of the slice rows [r_lo, r_lo + nrows) x octets
// [j_lo, j_lo + width), o = (r - r_lo) * width + (j - j_lo), taken 32 at a
// time by warp wbase, wbase + wstride, ...  j_lo and width are multiples of 4,
// so the 4 lanes of a 32-value block are 4 consecutive lanes and share the
// block's amax through two xor-shuffles (every lane runs them).  Writes the
// codes to qa ([M, K/2], plain) and the scale to qsa (flatS), with the same
// arithmetic as the stand-alone quantiser (mx_quant.cuh).
__device__ __forceinline__ void fused_quant_slice(const Params& p, int r_lo, int nrows, int j_lo, int width,
                                                  long long wbase, long long wstride)
{
    const int lane = threadIdx.x & 31;
    const long long total = (long long)nrows * width;
    for (long long base = wbase * 32; base < total; base += wstride * 32)
    {
        const long long o = base + lane;
        const bool valid = o < total;
        int r = 0, j = 0;
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        if (valid)
        {
            r = r_lo + (int)(o / width);
            j = j_lo + (int)(o - (long long)(r - r_lo) * width);
            const uint4 v = __ldcg(reinterpret_cast<const uint4*>(p.qx + (long long)r * p.qx_ld) + j);
            w[0] = v.x;
            w[1] = v.y;
            w[2] = v.z;
            w[3] = v.w;
        }
        uint32_t am = mx::amax_bits8(w);
        am = max(am, __shfl_xor_sync(0xffffffffu, am, 1));
        am = max(am, __shfl_xor_sync(0xffffffffu, am, 2));
        if (!valid) continue;
        const uint32_t sc = mx::scale_from_amax_bits(am);
        const bool nan_block = sc == 0xFFu;
        const float inv = __uint_as_float((254u - (nan_block ? 254u : sc)) << 23);
        reinterpret_cast<uint32_t*>(p.qa + (long long)r * (p.K >> 1))[j] = mx::encode8(w, inv, nan_block);
        if ((j & 3) == 0) p.qsa[flat_s_offset(r, j >> 2, p.q_snp)] = (uint8_t)sc;
    }
}

__device__ __forceinline__ void fence_proxy_async_global()
{
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// One operand's raw scale bytes for one K-stage (8 groups of 32 K) ->
// tcgen05.cp source blocks.  Output block (q, rb) covers rows 128*rb ..
// 128*rb+127 and K-groups 4q .. 4q+3 of the stage: 512 B with row r's four
// scale bytes at (r%32)*16 + ((r%128)/32)*4.
//   flatS input (kernel/gemm_a4w4.hip:97-105): per 32-row group g one 256 B
//     chunk, scale (r, b) at (b%4)*64 + (r%16)*4 + ((b/4)%2)*2 + (r%32)/16.
//     For fixed (g, r%16) the four words at (b%4)*64 hold, in byte p =
//     2*(b/4) + (r%32)/16, the scales of rows r and r+16 for both groups of
//     4: a 4x4 byte transpose gives the four output words.
//   macro input: per 32-row group 16 bytes covering 16 K-groups; this
//     stage's 8 start at byte 8*(ks&1); every row of the group shares them.
template <int ROWS, bool MACRO>
__device__ __forceinline__ void transpose_side(const uint8_t* raw, uint8_t* atoms, int ks, int lane)
{
    constexpr int RB = ROWS >= 128 ? ROWS / 128 : 1;
    if constexpr (!MACRO)
    {
        const uint32_t* raw32 = reinterpret_cast<const uint32_t*>(raw);
        constexpr int OPS = (ROWS / 32) * 16;
#pragma unroll
        for (int op = lane; op < OPS; op += 32)
        {
            const int g = op >> 4, rho = op & 15;
            const uint32_t w0 = raw32[g * 64 + rho];
            const uint32_t w1 = raw32[g * 64 + 16 + rho];
            const uint32_t w2 = raw32[g * 64 + 32 + rho];
            const uint32_t w3 = raw32[g * 64 + 48 + rho];
            const uint32_t t0 = __byte_perm(w0, w1, 0x5140);
            const uint32_t t1 = __byte_perm(w2, w3, 0x5140);
            const uint32_t t2 = __byte_perm(w0, w1, 0x7362);
            const uint32_t t3 = __byte_perm(w2, w3, 0x7362);
            const uint32_t o[4] = {__byte_perm(t0, t1, 0x5410), __byte_perm(t0, t1, 0x7632),
                                   __byte_perm(t2, t3, 0x5410), __byte_perm(t2, t3, 0x7632)};
#pragma unroll
            for (int pp = 0; pp < 4; ++pp)
            {
                const int r = 32 * g + 16 * (pp & 1) + rho;
                const int q = pp >> 1;
                *reinterpret_cast<uint32_t*>(atoms + (q * RB + (r >> 7)) * 512 + (r & 31) * 16 +
                                             ((r >> 5) & 3) * 4) = o[pp];
            }
        }
    }
    else
    {
        constexpr int OPS = ROWS * 2;
#pragma unroll
        for (int op = lane; op < OPS; op += 32)
        {
            const int r = op >> 1, q = op & 1;
            const uint32_t v =
                *reinterpret_cast<const uint32_t*>(raw + (r >> 5) * 16 + 8 * (ks & 1) + 4 * q);
            *reinterpret_cast<uint32_t*>(atoms + (q * RB + (r >> 7)) * 512 + (r & 31) * 16 +
                                         ((r >> 5) & 3) * 4) = v;
        }
    }
}

// In-stage activation quantiser (R_QUANT configurations), run on every
// stage once its bf16 rows landed (their own `xfull` barrier, so this runs
// ahead of the stage's weights).  The n <= XQ bf16 rows were staged by TMA
// as n x 512 B over the A tile's space (row r's BK = 256 values at r * 512).
// Each row becomes 128 B of e2m1 codes over the start of the same buffer --
// row r at r * 128, its 16-byte chunk b (32 values, one scale block) at
// b ^ (r % 8): the 128-byte swizzle of the MMA's K-major operand -- and 8
// e8m0 scales written straight into the tcgen05.cp blocks, scale (r, b) at
// (b / 4) * 512 + (r % 32) * 16 + (r / 32) * 4 + b % 4 (the
// transpose_side<32> output).  The arithmetic is the stand-alone
// quantiser's (mx_quant.cuh).
// Lane l takes whole blocks: block l % 8 of rows r0 + l / 8 + 4i, i < NI
// (its amax needs no other lane), and loads all of them before converting
// any.  The codes (rows below 4 of the staging) are written only after every
// reader is done: this warp's lanes (__syncwarp), or with two converting
// warps both warps (named barrier 2, which also ANDs their `ok`).  One warp
// converts ~8 rows per stage within the time the stage's weights take to
// stream in.
template <int NI, bool TWO_WARPS>
__device__ __forceinline__ bool quantise_rows(uint8_t* xs, uint8_t* atoms, int n, int r0, int lane, bool ok)
{
    const int q = lane >> 3, b = lane & 7;
    uint4 v[NI][4];
#pragma unroll
    for (int i = 0; i < NI; ++i)
    {
        const int r = min(r0 + q + 4 * i, n - 1);  // rows past n: any staged row (not stored)
        const uint4* src = reinterpret_cast<const uint4*>(xs + r * 512 + b * 64);
#pragma unroll
        for (int j = 0; j < 4; ++j) v[i][j] = src[j];
    }
    uint4 code[NI];
    uint32_t sc[NI];
#pragma unroll
    for (int i = 0; i < NI; ++i)
    {
        uint32_t w[4][4];
        uint32_t am = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j)
        {
            w[j][0] = v[i][j].x;
            w[j][1] = v[i][j].y;
            w[j][2] = v[i][j].z;
            w[j][3] = v[i][j].w;
            am = max(am, mx::amax_bits8(w[j]));
        }
        const uint32_t e = mx::scale_from_amax_bits(am);
        const bool nan_block = e == 0xFFu;
        const float inv = __uint_as_float((254u - (nan_block ? 254u : e)) << 23);
        code[i].x = mx::encode8(w[0], inv, nan_block);
        code[i].y = mx::encode8(w[1], inv, nan_block);
        code[i].z = mx::encode8(w[2], inv, nan_block);
        code[i].w = mx::encode8(w[3], inv, nan_block);
        sc[i] = e;
    }
    if constexpr (TWO_WARPS)
        ok = named_bar_and(2, 64, ok);  // both warps' reads before either's writes
    else
        __syncwarp();                   // every lane's reads before any lane's writes
    if (!ok) return false;
#pragma unroll
    for (int i = 0; i < NI; ++i)
    {
        const int r = r0 + q + 4 * i;
        if (r < n)
        {
            *reinterpret_cast<uint4*>(xs + r * 128 + ((b ^ (r & 7)) << 4)) = code[i];
            atoms[(b >> 2) * 512 + (r & 31) * 16 + (r >> 5) * 4 + (b & 3)] = (uint8_t)sc[i];
        }
    }
    return true;
}

// XQ 8: all n <= 8 rows by one warp
__device__ __forceinline__ void quantise_stage(uint8_t* xs, uint8_t* atoms, int n, int lane)
{
    if (n > 4)
        quantise_rows<2, false>(xs, atoms, n, 0, lane, true);
    else
        quantise_rows<1, false>(xs, atoms, n, 0, lane, true);
}

// Cluster split-K.  Cluster rank r finishes rows [r R, (r + 1) R) of the
// tile, R = R_ROWS / S (R_ROWS = 128, or 32 / 64 for skinny tiles, the rows
// that can hold outputs).  Each CTA's buffer (in its pipeline stages, idle once
// the whole cluster holds complete accumulators) has S slots, slot s holding
// rank s's partial of the rows this CTA finishes, stored by 16-byte column
// group q and row: group (s, q) is R + 1 rows of 16 bytes, so
//   byte offset of (slot s, group q, row lr) = ((s * BN/4 + q) * (R + 1) + lr) * 16.
// A warp storing its 32 accumulator rows' group q writes 512 contiguous
// bytes (stores into another CTA's shared memory move in packets; 16-byte
// pieces scattered over rows ran ~3x slower), and a warp reading 32
// consecutive groups of one row steps by R + 1 rows: distinct banks.
__device__ __forceinline__ int split_off(int s, int q, int lr, int rows, int c4)
{
    return ((s * c4 + q) * (rows + 1) + lr) * 16;
}

// The hand-over (epilogue threads, after a cluster barrier): each CTA pushes
// its fp32 partial straight from TMEM, rows [j R, (j + 1) R) into slot r of
// rank j's buffer; its own rows with plain shared stores (~3x the rate of
// stores into another CTA).  When R = R_ROWS / S >= 32 a warp's 32 rows have a
// single destination and the local/remote branch is warp-uniform; skinny
// tiles (R_ROWS = 32 or 64) with a larger S spread one warp's rows over
// several CTAs, which stays correct but diverges.  S is 2, 4 or 8 (the
// planner accepts nothing else), so R is a whole number of rows and every row
// has a destination rank below S.  An empty K range pushes zeros.
template <class CF>
__device__ __forceinline__ void split_push(const Params& p, const uint8_t* smem, uint32_t tmem_base, int warp,
                                           int lane, bool any)
{
    constexpr int COLS = CF::BN / 2;
    constexpr int C4 = CF::BN / 4;
    constexpr int NCH = COLS / 16;
    constexpr int BATCH = NCH < 4 ? NCH : 4;
    const int quarter = warp & 3, half = (warp - EPI_WARP0) >> 2;
    const int row = quarter * 32 + lane;  // accumulator row (TMEM lane)
    if (row >= CF::R_ROWS) return;        // skinny tiles: rows past R_ROWS hold no output
    const int S = p.ksplit, rows = CF::R_ROWS / S;
    const int rank = (int)(blockIdx.x % (unsigned)S);
    const int dst = row / rows, lr = row % rows;
    if (dst >= S) return;  // never taken for S in {2, 4, 8}; keeps mapa inside the cluster
    const bool local = dst == rank;
    const uint32_t rbase = mapa_shared(smem_u32(smem), (uint32_t)dst);
    uint8_t* lbase = const_cast<uint8_t*>(smem);
    const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + half * COLS;
#pragma unroll
    for (int b0 = 0; b0 < NCH; b0 += BATCH)
    {
        uint32_t v[BATCH][16];
#pragma unroll
        for (int b = 0; b < BATCH; ++b) tc_ld_32x32b_x16(taddr + (b0 + b) * 16, v[b]);
        tc_wait_ld();
#pragma unroll
        for (int b = 0; b < BATCH; ++b)
        {
#pragma unroll
            for (int t = 0; t < 4; ++t)
            {
                const int q = half * (COLS / 4) + (b0 + b) * 4 + t;  // 16-byte column group of the tile
                const int off = split_off(rank, q, lr, rows, C4);
                const uint4 val = any ? make_uint4(v[b][4 * t], v[b][4 * t + 1], v[b][4 * t + 2], v[b][4 * t + 3])
                                      : make_uint4(0u, 0u, 0u, 0u);
                if (local)
                    *reinterpret_cast<uint4*>(lbase + off) = val;
                else
                    st_shared_cluster_v4(rbase + (uint32_t)off, val.x, val.y, val.z, val.w);
            }
        }
    }
}

// The finish (all threads, after the pushes and a cluster barrier): rank r
// sums its R rows over the S slots of its own buffer in slot order 0, 1, ...
// (every run adds in the same order), applies factors, alpha and bias as the
// single-pass epilogue does and stores bf16: a warp covers 32 consecutive
// column groups of one row, 256 contiguous output bytes.
template <class CF>
__device__ __forceinline__ void split_finish(const Params& p, const uint8_t* smem, const float* epi_f, int et)
{
    constexpr int BN = CF::BN;
    constexpr int C4 = BN / 4;
    constexpr int NT = NUM_THREADS;
    constexpr int U = 8;
    const int S = p.ksplit;
    const int rank = (int)(blockIdx.x % (unsigned)S);
    const int rows = CF::R_ROWS / S;
    const int tile = (int)(blockIdx.x / (unsigned)S);
    const int tr = tile % p.tiles_r, tc = tile / p.tiles_r;
    const int r0 = tr * BM, c0 = tc * BN;
    const float* fr_s = epi_f;
    const float* fc_s = epi_f + BM;
    const float* bias_s = epi_f + BM + BN;
    const bool has_factor = (p.a_factor != nullptr) || (p.b_factor != nullptr);
    const bool has_alpha = p.alpha != 1.0f;
    const bool has_bias = p.bias != nullptr;
    const int units = rows * C4;
    for (int u0 = et; u0 < units; u0 += NT * U)
    {
        float4 a[U];
#pragma unroll
        for (int u = 0; u < U; ++u) a[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int src = 0; src < S; ++src)
        {
#pragma unroll
            for (int u = 0; u < U; ++u)
            {
                const int idx = u0 + u * NT;
                if (idx < units)
                {
                    const float4 b =
                        *reinterpret_cast<const float4*>(smem + split_off(src, idx % C4, idx / C4, rows, C4));
                    if (src == 0)
                    {
                        a[u] = b;
                    }
                    else
                    {
                        a[u].x += b.x;
                        a[u].y += b.y;
                        a[u].z += b.z;
                        a[u].w += b.w;
                    }
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
        {
            const int idx = u0 + u * NT;
            const int tl = rank * rows + idx / C4, c = (idx % C4) * 4;  // tile row, tile column
            const int m = r0 + tl, n = c0 + c;
            if (idx >= units || m >= p.M || n >= p.N) continue;
            float x[4] = {a[u].x, a[u].y, a[u].z, a[u].w};
            if (has_factor)
            {
#pragma unroll
                for (int t = 0; t < 4; ++t) x[t] = __fmul_rn(x[t], __fmul_rn(fr_s[tl], fc_s[c + t]));
            }
            if (has_alpha)
            {
#pragma unroll
                for (int t = 0; t < 4; ++t) x[t] = __fmul_rn(x[t], p.alpha);
            }
            if (has_bias)
            {
#pragma unroll
                for (int t = 0; t < 4; ++t) x[t] = __fadd_rn(x[t], bias_s[c + t]);
            }
            __nv_bfloat162 h0 = __floats2bfloat162_rn(x[0], x[1]);
            __nv_bfloat162 h1 = __floats2bfloat162_rn(x[2], x[3]);
            const uint2 v = make_uint2(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1));
            const long long off = (long long)m * p.ldc + n;
#pragma unroll
            for (int d = 0; d < MAX_OUT; ++d)
            {
                if (d >= p.n_out) break;
                *reinterpret_cast<uint2*>(p.outs[d] + off) = v;
            }
        }
    }
}

// ------------------------------------------------------------------ kernel
template <class CF>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    mxf4_gemm_kernel(const __grid_constant__ CUtensorMap tm_r, const __grid_constant__ CUtensorMap tm_c,
                     const __grid_constant__ CUtensorMap tm_rsf, const __grid_constant__ CUtensorMap tm_csf,
                     const Params p)
{
    constexpr int BN = CF::BN;
    constexpr int STAGES = CF::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * CF::STAGE_BYTES);
    uint64_t* sfready = full + STAGES;
    uint64_t* empty = sfready + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* qready = acc_empty + 2;  // fused quantiser: this CTA's share of A is written
    uint64_t* xfull = qready + 1;      // in-stage quantiser: the stage's bf16 rows landed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xfull + CF::XBARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* epi_f = reinterpret_cast<float*>(smem + STAGES * CF::STAGE_BYTES + CF::BAR_BYTES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    unsigned long long tacc[16] = {0};
#if MBS_TIMING
    const long long t_kernel0 = clock64();
#endif
    constexpr int QWARPS = NUM_THREADS / 32 - 2;  // warps 2.. quantise A before their own role

    if (threadIdx.x == 0)
    {
        for (int s = 0; s < STAGES; ++s)
        {
            mbar_init(&full[s], 1);
            mbar_init(&sfready[s], 2);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b)
        {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], NUM_EPI_WARPS);
        }
        mbar_init(qready, QWARPS);
        for (int s = 0; s < CF::XBARS; ++s) mbar_init(&xfull[s], 1);
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tmap(&tm_r);
        prefetch_tmap(&tm_rsf);
        if (!CF::C_PACKED)
        {
            prefetch_tmap(&tm_c);
            prefetch_tmap(&tm_csf);
        }
    }
    if (warp == 1)
    {
        tmem_alloc(tmem_slot, CF::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Programmatic dependent launch: this grid may have started while the
    // kernel ahead of it in the stream was still running.  Every thread waits
    // for that kernel here, before its first global-memory access (a no-op
    // for a plain launch), then lets the next kernel start its prologue on
    // the SMs this grid frees.
    griddep_wait();
    griddep_launch_dependents();
#if MBS_TIMING
    if (threadIdx.x == 0) tacc[14] = (unsigned long long)(clock64() - t_kernel0);
    if (threadIdx.x == 0 && blockIdx.x < 1024) g_mbs_cta[blockIdx.x * 5 + 1] = globaltimer_ns();
#endif

    if constexpr (!CF::SWAP && !CF::R_QUANT)
    {
        if (p.qmode != 0 && warp >= 2)
        {
            // ------------------------------------------------ fused activation quantiser
            // Warps 2.. write A (codes + flatS scales) before taking up their own
            // roles, while the producer already streams the first stages' weights.
            // qmode 1: the grid shares all of A (the producer then waits on a grid
            // barrier); qmode 2: each CTA writes the blocks of its own tile rows and
            // K range (CTAs of other clusters may write the same blocks, with the
            // same bytes).
            if (p.qmode == 1)
            {
                fused_quant_slice(p, 0, p.M, 0, p.K >> 3, (long long)blockIdx.x * QWARPS + (warp - 2),
                                  (long long)gridDim.x * QWARPS);
            }
            else
            {
                Work w0;
                if (get_work(p, 0, w0))
                {
                    const int r_lo = (w0.tile % p.tiles_r) * BM;
                    const int r_hi = min(p.M, r_lo + CF::R_ROWS);
                    const int j_lo = w0.k0 * (BK / 8);
                    const int j_hi = min(p.K >> 3, w0.k1 * (BK / 8));
                    if (r_hi > r_lo && j_hi > j_lo)
                        fused_quant_slice(p, r_lo, r_hi - r_lo, j_lo, j_hi - j_lo, warp - 2, QWARPS);
                }
            }
            fence_proxy_async_global();  // the TMA (async proxy) reads these bytes next
            __syncwarp();
            if (lane == 0) mbar_arrive(qready);
        }
    }

    if (warp == 0)
    {
        // ------------------------------------------------ TMA producer
        if (lane == 0)
        {
            int slot = 0;
            uint32_t phase = 0;
            // Fused quantiser: the first STAGES stages are armed and their weights
            // issued at once; their A tiles (and A scales) follow once A is written.
            int ndef = (!CF::SWAP && !CF::R_QUANT && p.qmode != 0) ? 0 : -1;  // -1: A is ready
            int def_slot[STAGES], def_r0[STAGES], def_ks[STAGES];
            auto a_ready = [&]() {
                bool ok = mbar_wait(qready, 0, nullptr);
                if (p.qmode == 1)
                {
                    __threadfence();  // this CTA's share of A (seen through qready) before the arrival
                    atomicAdd(&p.qbar[0], 1u);
                    const unsigned long long t0 = globaltimer_ns();
                    while (ld_acquire_gpu(&p.qbar[0]) < gridDim.x)
                    {
                        if (globaltimer_ns() - t0 > kWaitTimeoutNs)
                        {
                            ok = false;
                            break;
                        }
                    }
                    // the last CTA past the barrier leaves both words zero for the next launch
                    if (atomicAdd(&p.qbar[1], 1u) == gridDim.x - 1)
                    {
                        atomicExch(&p.qbar[0], 0u);
                        atomicExch(&p.qbar[1], 0u);
                    }
                }
                // a wait that ran out is reported; the loads still go out (to valid
                // addresses), so every armed stage completes and nothing is left in flight
                if (!ok) atomicExch(p.err, (unsigned)MBS_ERR_DEVICE_TIMEOUT);
                fence_proxy_async_global();
            };
            // The weights (C, or R when swapped) are read exactly once when the
            // other operand is a single tile: stream them evict-first.
            const bool w_once = CF::SWAP ? p.tiles_c == 1 : p.tiles_r == 1;
            const uint64_t pol_w = w_once ? l2_policy_evict_first() : l2_policy_evict_normal();
            const uint64_t pol_r = CF::SWAP ? pol_w : l2_policy_evict_normal();
            const uint64_t pol_c = CF::SWAP ? l2_policy_evict_normal() : pol_w;
            // A box of activation rows stops at M when one tile covers them all, so no
            // stage pays for out-of-bounds fill; expect only the bytes it brings.
            // In-stage quantiser: the bf16 rows complete `xfull`, the rest `full`.
            const uint32_t tx_bytes = CF::TX_BYTES - (CF::R_QUANT ? (uint32_t)CF::R_DATA
                                                                  : (uint32_t)((CF::SWAP ? BN : CF::R_ROWS) -
                                                                               p.act_rows) * BKB);
            const uint32_t x_tx = (uint32_t)p.act_rows * CF::R_ROW_TX;
            Work w;
            for (int i = 0; get_work(p, i, w); ++i)
            {
                const int tr = w.tile % p.tiles_r, tc = w.tile / p.tiles_r;
                const int r0 = tr * BM, c0 = tc * BN;
                for (int ks = w.k0; ks < w.k1; ++ks)
                {
                    bool ok_empty;
                    {
                        MBS_TSTART();
                        ok_empty = mbar_wait(&empty[slot], phase ^ 1, abort_flag);
                        MBS_TADD(tacc, 0);
                    }
                    if (!ok_empty)
                    {
                        raise_error(p, abort_flag);
                        goto producer_done;
                    }
#if MBS_TIMING
                    tacc[10] += 1;
#endif
                    uint8_t* st = smem + slot * CF::STAGE_BYTES;
                    if constexpr (CF::R_QUANT)
                    {
                        // bf16 activations (tm_r is their map): {BK values, rows}
                        mbar_arrive_expect_tx(&xfull[slot], x_tx);
                        tma_load_2d_hint(st + CF::R_DATA_OFF, &tm_r, &xfull[slot], ks * BK, r0, pol_r);
                    }
                    mbar_arrive_expect_tx(&full[slot], tx_bytes);
                    const bool defer = ndef >= 0;
                    if (defer)
                    {
                        def_slot[ndef] = slot;
                        def_r0[ndef] = r0;
                        def_ks[ndef] = ks;
                        ++ndef;
                    }
                    else if (CF::R_PRESHUF)
                        tma_load_3d_hint(st + CF::R_DATA_OFF, &tm_r, &full[slot], 0, r0 / 16, ks * 8, pol_r);
                    else if (CF::R_QUANT)
                        ;  // loaded above
                    else
                        tma_load_2d_hint(st + CF::R_DATA_OFF, &tm_r, &full[slot], ks * BKB, r0, pol_r);
                    if (CF::C_PACKED)
                        bulk_load_hint(st + CF::C_DATA_OFF,
                                       p.packed_b + ((size_t)tc * p.k_stages + ks) * PACK_STAGE_BYTES,
                                       PACK_STAGE_BYTES, &full[slot], pol_c);
                    else if (CF::C_PRESHUF)
                        tma_load_3d_hint(st + CF::C_DATA_OFF, &tm_c, &full[slot], 0, c0 / 16, ks * 8, pol_c);
                    else
                        tma_load_2d_hint(st + CF::C_DATA_OFF, &tm_c, &full[slot], ks * BKB, c0, pol_c);
                    if (defer || CF::R_QUANT)
                        ;  // A scales follow the deferred A tile, or come from the quantiser warps
                    else if (CF::R_MACRO)
                        tma_load_2d_hint(st + CF::R_RAW_OFF, &tm_rsf, &full[slot], 16 * (ks >> 1), r0 / 32, pol_r);
                    else
                        tma_load_3d_hint(st + CF::R_RAW_OFF, &tm_rsf, &full[slot], 0, ks, r0 / 32, pol_r);
                    if (CF::C_PACKED)
                        ;  // scale blocks arrived with the packed tile
                    else if (CF::C_MACRO)
                        tma_load_2d_hint(st + CF::C_RAW_OFF, &tm_csf, &full[slot], 16 * (ks >> 1), c0 / 32, pol_c);
                    else
                        tma_load_3d_hint(st + CF::C_RAW_OFF, &tm_csf, &full[slot], 0, ks, c0 / 32, pol_c);
                    if (++slot == STAGES)
                    {
                        slot = 0;
                        phase ^= 1;
                    }
                    if (ndef == STAGES)
                    {
                        // every slot is armed: the next stage needs a slot the MMAs free,
                        // and they need A
                        a_ready();
                        for (int d = 0; d < STAGES; ++d)
                        {
                            uint8_t* sd = smem + def_slot[d] * CF::STAGE_BYTES;
                            tma_load_2d_hint(sd + CF::R_DATA_OFF, &tm_r, &full[def_slot[d]], def_ks[d] * BKB,
                                             def_r0[d], pol_r);
                            tma_load_3d_hint(sd + CF::R_RAW_OFF, &tm_rsf, &full[def_slot[d]], 0, def_ks[d],
                                             def_r0[d] / 32, pol_r);
                        }
                        ndef = -1;
                    }
                }
            }
            if (ndef >= 0)
            {
                // fewer stages than slots (or no work: a grid barrier still needs this CTA)
                a_ready();
                for (int d = 0; d < ndef; ++d)
                {
                    uint8_t* sd = smem + def_slot[d] * CF::STAGE_BYTES;
                    tma_load_2d_hint(sd + CF::R_DATA_OFF, &tm_r, &full[def_slot[d]], def_ks[d] * BKB, def_r0[d],
                                     pol_r);
                    tma_load_3d_hint(sd + CF::R_RAW_OFF, &tm_rsf, &full[def_slot[d]], 0, def_ks[d], def_r0[d] / 32,
                                     pol_r);
                }
                ndef = -1;
            }
        producer_done:;
#if MBS_TIMING
            if (blockIdx.x < 1024)
            {
                unsigned smid_t;
                asm volatile("mov.u32 %0, %%smid;" : "=r"(smid_t));
                g_mbs_cta[blockIdx.x * 5 + 0] = smid_t;
                g_mbs_cta[blockIdx.x * 5 + 2] = globaltimer_ns();
                g_mbs_cta[blockIdx.x * 5 + 4] = tacc[10];
            }
#endif
        }
    }
    else if (warp == 1)
    {
        // ------------------------------------------------ MMA issuer
        if (lane == 0)
        {
            int slot = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            Work w;
            for (int i = 0; get_work(p, i, w); ++i)
            {
                bool ok_acc;
                {
                    MBS_TSTART();
                    ok_acc = mbar_wait(&acc_empty[acc], acc_phase ^ 1, abort_flag);
                    MBS_TADD(tacc, 1);
                }
                if (!ok_acc)
                {
                    raise_error(p, abort_flag);
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                bool ok = true;
                for (int ks = w.k0; ks < w.k1; ++ks)
                {
                    // `sfready` implies `full`: both transposer warps arrive on it
                    // only after their own wait on this stage's `full` (release /
                    // acquire through the two barriers; with the in-stage quantiser
                    // warp 3 still waits for `full`), so one barrier test per stage
                    // suffices here.
                    bool ok_sf;
                    {
                        MBS_TSTART();
                        ok_sf = mbar_wait(&sfready[slot], phase, abort_flag);
                        // 16-row in-stage quantiser: its warps arrive on `sfready` without
                        // waiting for the stage's weights, so this thread tests `full` too
                        if (CF::XQ == 16) ok_sf = mbar_wait(&full[slot], phase, abort_flag) && ok_sf;
                        MBS_TADD(tacc, 3);
                    }
                    if (!ok_sf)
                    {
                        raise_error(p, abort_flag);
                        ok = false;
                        break;
                    }
                    MBS_TSTART();
                    tc_fence_after();
                    const uint8_t* st = smem + slot * CF::STAGE_BYTES;
                    const uint32_t sf_r = tmem_base + CF::SF_BASE + slot * CF::SF_STAGE_COLS;
                    const uint32_t sf_c = sf_r + 8;
                    // scales: shared memory -> TMEM (32 rows x 16 B per block, x4 sub-partitions)
#pragma unroll
                    for (int q = 0; q < 2; ++q)
                        tc_cp_32x128b_warpx4(sf_r + 4 * q,
                                             make_smem_desc(smem_u32(st + CF::R_ATOM_OFF + q * 512), 0, 128, 0));
#pragma unroll
                    for (int a = 0; a < 2 * CF::C_RB; ++a)
                        tc_cp_32x128b_warpx4(sf_c + 4 * a,
                                             make_smem_desc(smem_u32(st + CF::C_ATOM_OFF + a * 512), 0, 128, 0));
                    const uint32_t r_base = smem_u32(st + CF::R_DATA_OFF);
                    const uint32_t c_base = smem_u32(st + CF::C_DATA_OFF);
#pragma unroll
                    for (int j = 0; j < BK / MMA_K; ++j)
                    {
                        if (ks * BK + j * MMA_K >= p.K) break;
                        const uint64_t a_desc =
                            CF::R_PRESHUF ? make_smem_desc(r_base + j * 2 * (BM * 16), BM * 16, 128, 0)
                                          : make_smem_desc(r_base + j * 32, 16, 1024, 2);
                        const uint64_t b_desc =
                            CF::C_PRESHUF ? make_smem_desc(c_base + j * 2 * (BN * 16), BN * 16, 128, 0)
                                          : make_smem_desc(c_base + j * 32, 16, 1024, 2);
                        const uint32_t id = (uint32_t)(j & 1) * 2;  // byte of the 32-bit scale column
                        const uint32_t q = (uint32_t)(j >> 1);      // which 4-group scale block
                        const uint32_t sfa = (sf_r + 4 * q) | (id << 30);
                        const uint32_t sfb = (sf_c + 4 * CF::C_RB * q) | (id << 30);
                        tc_mma_mxf4(d_tmem, a_desc, b_desc, make_idesc_mxf4(BM, BN, id, id), sfa, sfb,
                                    (ks > w.k0 || j > 0) ? 1u : 0u);
                    }
                    tc_commit(&empty[slot]);
                    MBS_TADD(tacc, 11);
                    if (++slot == STAGES)
                    {
                        slot = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                tc_commit(&acc_full[acc]);
                if (CF::ACC_BUFS == 2)
                {
                    acc ^= 1;
                    if (acc == 0) acc_phase ^= 1;
                }
                else
                {
                    acc_phase ^= 1;
                }
            }
        }
    }
    else if (CF::XQ == 16 && (warp == 2 || warp == 3))
    {
        // ------------------------------------------------ in-stage quantiser, 16 rows
        // (packed weights: their scale blocks arrive ready, nothing to transpose)
        // Warps 2 and 3 each convert 8 of the activation rows of every stage as
        // soon as they land, and arrive on `sfready`; a failed wait in either
        // warp reaches the other at the stage's barrier, so both stop together.
        const int h = warp - 2;
        int slot = 0;
        uint32_t phase = 0;
        bool ok = true;
        Work w;
        for (int i = 0; ok && get_work(p, i, w); ++i)
        {
            for (int ks = w.k0; ks < w.k1; ++ks)
            {
                bool ok_x;
                {
                    MBS_TSTART();
                    ok_x = mbar_wait(&xfull[slot], phase, abort_flag);
                    MBS_TADD(tacc, 4);
                }
                MBS_TSTART();
                uint8_t* st = smem + slot * CF::STAGE_BYTES;
                if (!quantise_rows<2, true>(st + CF::R_DATA_OFF, st + CF::R_ATOM_OFF, p.act_rows, 8 * h, lane, ok_x))
                {
                    if (lane == 0) raise_error(p, abort_flag);
                    ok = false;
                    break;
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sfready[slot]);
                MBS_TADD(tacc, 5);
                if (++slot == STAGES)
                {
                    slot = 0;
                    phase ^= 1;
                }
            }
        }
    }
    else if (warp == 2 || warp == 3)
    {
        // ------------------------------------------------ scale transposers
        // warp 2 rewrites the R operand's scales, warp 3 the C operand's; with
        // the 8-row in-stage quantiser warp 2 quantises the activation rows instead.
        const bool r_side = warp == 2;
        int slot = 0;
        uint32_t phase = 0;
        Work w;
        for (int i = 0; get_work(p, i, w); ++i)
        {
            bool ok = true;
            for (int ks = w.k0; ks < w.k1; ++ks)
            {
                if (CF::R_QUANT && r_side)
                {
                    // the stage's activation rows, quantised as soon as they land
                    bool ok_x;
                    {
                        MBS_TSTART();
                        ok_x = mbar_wait(&xfull[slot], phase, abort_flag);
                        MBS_TADD(tacc, 4);
                    }
                    if (!ok_x)
                    {
                        if (lane == 0) raise_error(p, abort_flag);
                        ok = false;
                        break;
                    }
                    MBS_TSTART();
                    uint8_t* st = smem + slot * CF::STAGE_BYTES;
                    quantise_stage(st + CF::R_DATA_OFF, st + CF::R_ATOM_OFF, p.act_rows, lane);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sfready[slot]);
                    MBS_TADD(tacc, 5);
                }
                else
                {
                    bool ok_full;
                    {
                        MBS_TSTART();
                        ok_full = mbar_wait(&full[slot], phase, abort_flag);
                        MBS_TADD(tacc, 4);
                    }
                    if (!ok_full)
                    {
                        if (lane == 0) raise_error(p, abort_flag);
                        ok = false;
                        break;
                    }
                    MBS_TSTART();
                    uint8_t* st = smem + slot * CF::STAGE_BYTES;
                    if (r_side && !CF::R_QUANT)
                        transpose_side<CF::R_ROWS, CF::R_MACRO>(st + CF::R_RAW_OFF, st + CF::R_ATOM_OFF, ks, lane);
                    else if (!CF::C_PACKED)
                        transpose_side<BN, CF::C_MACRO>(st + CF::C_RAW_OFF, st + CF::C_ATOM_OFF, ks, lane);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sfready[slot]);
                    MBS_TADD(tacc, 5);
                }
                if (++slot == STAGES)
                {
                    slot = 0;
                    phase ^= 1;
                }
            }
            if (!ok) break;
        }
    }
    else if (warp >= EPI_WARP0)
    {
        // ------------------------------------------------ epilogue
        // Each thread owns one accumulator row (TMEM lane) and half of the
        // BN columns.  The output path drains its columns from TMEM into
        // registers (scaled, rounded to bf16), releases the accumulator so
        // the next tile's MMAs can start, and only then stores.
        const int e = warp - EPI_WARP0;
        const int quarter = warp & 3;         // TMEM lanes [32*quarter, 32*quarter + 32)
        const int half = e >> 2;              // which half of the BN columns
        const int row = quarter * 32 + lane;  // accumulator row (TMEM lane)
        const int et = threadIdx.x - EPI_WARP0 * 32;  // 0 .. NUM_EPI_THREADS-1
        constexpr int COLS = BN / 2;
        constexpr int NCH = COLS / 16;
        constexpr int BATCH = NCH < 4 ? NCH : 4;
        // stream-K partial slots hold only the rows that can be valid
        constexpr int PR = CF::SWAP ? BM : CF::R_ROWS;
        // an owner sums its contributors' partials in the idle pipeline stages when they fit
        constexpr bool STAGE_PARTIALS = PR * BN * 4 <= STAGES * CF::STAGE_BYTES;
        const bool has_factor = (p.a_factor != nullptr) || (p.b_factor != nullptr);
        const bool has_alpha = p.alpha != 1.0f;
        const bool has_bias = p.bias != nullptr;
        // R rows are activations (non-swap) or weights (swap); C columns the other.
        const uint8_t* r_factor = CF::SWAP ? p.b_factor : p.a_factor;
        const uint8_t* c_factor = CF::SWAP ? p.a_factor : p.b_factor;
        const int r_extent = CF::SWAP ? p.N : p.M;
        const int c_extent = CF::SWAP ? p.M : p.N;
        float* fr_s = epi_f;            // [BM] row factors of the current tile
        float* fc_s = epi_f + BM;       // [BN] column factors
        float* bias_s = epi_f + BM + BN;  // [BN] column bias (non-swapped)
        int acc = 0;
        uint32_t acc_phase = 0;
        Work w;
        for (int i = 0; get_work(p, i, w); ++i)
        {
            const int tr = w.tile % p.tiles_r, tc = w.tile / p.tiles_r;
            const int r0 = tr * BM, c0 = tc * BN;
            const bool nonowner = p.sk && w.k0 > 0;
            const bool owner = p.sk && w.k0 == 0 && w.k1 < p.k_stages;
            if ((has_factor || (has_bias && !CF::SWAP)) && !nonowner)
            {
                named_bar_sync(1, NUM_EPI_THREADS);  // previous tile's readers are done
                if (et < BM)
                {
                    const int r = r0 + et;
                    fr_s[et] = (r_factor != nullptr && r < r_extent) ? byte_to_factor(r_factor[r]) : 1.0f;
                }
                if (et < BN)
                {
                    const int c = c0 + et;
                    fc_s[et] = (c_factor != nullptr && c < c_extent) ? byte_to_factor(c_factor[c]) : 1.0f;
                    if (!CF::SWAP)
                        bias_s[et] = (has_bias && c < c_extent) ? __bfloat162float(p.bias[c]) : 0.0f;
                }
                named_bar_sync(1, NUM_EPI_THREADS);
            }
            bool ok_acc;
            {
                MBS_TSTART();
                ok_acc = mbar_wait(&acc_full[acc], acc_phase, abort_flag);
                MBS_TADD(tacc, 6);
            }
            // all epilogue warps take the same branch, so none is left behind in a named barrier
            ok_acc = named_bar_and(1, NUM_EPI_THREADS, ok_acc);
            if (!ok_acc)
            {
                if (lane == 0) raise_error(p, abort_flag);
                break;
            }
            MBS_TSTART();
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN + half * COLS;
            const bool row_valid = r0 + row < r_extent;
            if (CF::SPLIT_OK && p.ksplit > 1)
            {
                // cluster split-K: the accumulator stays in TMEM until the whole
                // cluster has its own (split_push after the role loops)
            }
            else if (nonowner)
            {
                float* part = p.partials + (size_t)blockIdx.x * (PR * BN);
#pragma unroll 1
                for (int c = 0; c < COLS; c += 16)
                {
                    uint32_t v[16];
                    tc_ld_32x32b_x16(taddr + c, v);
                    tc_wait_ld();
                    if (row_valid && row < PR)
                    {
#pragma unroll
                        for (int t = 0; t < 16; ++t)
                            __stcg(part + (size_t)(half * COLS + c + t) * PR + row, __uint_as_float(v[t]));
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[acc]);
                __threadfence();
                named_bar_sync(1, NUM_EPI_THREADS);
                // (the failure-path test withholds the release: the owner's bounded wait then runs out)
                if (et == 0 && !p.withhold_release) st_release_gpu(&p.flags[blockIdx.x], 1u);
            }
            else
            {
                int c_first = 0, c_last = -1;  // contributing CTAs [c_first, c_last]
                const float* psum = nullptr;   // their partials summed, [BN][PR] in shared memory
                if (owner)
                {
                    const long long tile_end = (long long)(w.tile + 1) * p.k_stages;
                    c_first = blockIdx.x + 1;
                    c_last = sk_last_starting_before(p, tile_end);
                    if (et == 0)
                    {
#if MBS_TIMING
                        const long long t_flag0 = clock64();
#endif
                        const unsigned long long t0 = globaltimer_ns();
                        for (int c = c_first; c <= c_last; ++c)
                        {
                            while (ld_acquire_gpu(&p.flags[c]) == 0u)
                            {
                                if (*abort_flag || globaltimer_ns() - t0 > kWaitTimeoutNs)
                                {
                                    raise_error(p, abort_flag);
                                    break;
                                }
                            }
                        }
#if MBS_TIMING
                        tacc[8] += (unsigned long long)(clock64() - t_flag0);
#endif
                    }
                    named_bar_sync(1, NUM_EPI_THREADS);
                    // An owner item ends this CTA's range, so it is the CTA's last item: with its
                    // accumulator full, no load or MMA touches the pipeline stages any more.  The
                    // contributors' partials are summed there first, every thread keeping eight
                    // independent 16-byte loads in flight, so the tile costs about one DRAM round
                    // trip; the drain loop then adds them from shared memory.  (Per-thread loads
                    // inside the drain loop would pay a round trip per column chunk.)
                    if constexpr (STAGE_PARTIALS)
                    {
                        constexpr int N4 = PR * BN / 4;
                        constexpr int U = 8;
                        float4* sum4 = reinterpret_cast<float4*>(smem);
                        const float4* part4 = reinterpret_cast<const float4*>(p.partials);
                        for (int base = et; base < N4; base += NUM_EPI_THREADS * U)
                        {
                            float4 a[U];
#pragma unroll
                            for (int u = 0; u < U; ++u) a[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                            // two contributors per round trip: both sets of loads are in
                            // flight before the adds, which keep the contributors' order
                            for (int cc = c_first; cc <= c_last; cc += 2)
                            {
                                const bool two = cc + 1 <= c_last;
                                const float4* src0 = part4 + (size_t)cc * N4;
                                const float4* src1 = part4 + (size_t)(two ? cc + 1 : cc) * N4;
                                float4 b0[U], b1[U];
#pragma unroll
                                for (int u = 0; u < U; ++u)
                                {
                                    const int e4 = base + u * NUM_EPI_THREADS;
                                    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
                                    b0[u] = e4 < N4 ? __ldcg(src0 + e4) : z;
                                    b1[u] = (two && e4 < N4) ? __ldcg(src1 + e4) : z;
                                }
#pragma unroll
                                for (int u = 0; u < U; ++u)
                                {
                                    a[u].x += b0[u].x;
                                    a[u].y += b0[u].y;
                                    a[u].z += b0[u].z;
                                    a[u].w += b0[u].w;
                                    if (two)
                                    {
                                        a[u].x += b1[u].x;
                                        a[u].y += b1[u].y;
                                        a[u].z += b1[u].z;
                                        a[u].w += b1[u].w;
                                    }
                                }
                            }
#pragma unroll
                            for (int u = 0; u < U; ++u)
                            {
                                const int e4 = base + u * NUM_EPI_THREADS;
                                if (e4 < N4) sum4[e4] = a[u];
                            }
                        }
                        named_bar_sync(1, NUM_EPI_THREADS);
                        psum = reinterpret_cast<const float*>(smem);
                    }
                }
                uint32_t packed[COLS / 2];
                const float fr = has_factor ? fr_s[row] : 1.0f;
                // swapped: the bias runs along the R rows (output columns n = r0 + row)
                const float brow = (CF::SWAP && has_bias && row_valid) ? __bfloat162float(p.bias[r0 + row]) : 0.0f;
#pragma unroll
                for (int b0 = 0; b0 < NCH; b0 += BATCH)
                {
                    uint32_t v[BATCH][16];
#pragma unroll
                    for (int b = 0; b < BATCH; ++b) tc_ld_32x32b_x16(taddr + (b0 + b) * 16, v[b]);
                    tc_wait_ld();
#pragma unroll
                    for (int b = 0; b < BATCH; ++b)
                    {
                        const int cb = half * COLS + (b0 + b) * 16;  // first tile column of the chunk
                        float x[16];
#pragma unroll
                        for (int t = 0; t < 16; ++t) x[t] = __uint_as_float(v[b][t]);
                        if constexpr (STAGE_PARTIALS)
                        {
                            if (psum != nullptr && row < PR)
                            {
#pragma unroll
                                for (int t = 0; t < 16; ++t) x[t] += psum[(cb + t) * PR + row];
                            }
                        }
                        else if (row < PR)
                        {
                            for (int cc = c_first; cc <= c_last; ++cc)
                            {
                                const float* part = p.partials + (size_t)cc * (PR * BN);
#pragma unroll
                                for (int t = 0; t < 16; ++t) x[t] += __ldcg(part + (size_t)(cb + t) * PR + row);
                            }
                        }
                        if (has_factor)
                        {
#pragma unroll
                            for (int t = 0; t < 16; ++t) x[t] = __fmul_rn(x[t], __fmul_rn(fr, fc_s[cb + t]));
                        }
                        if (has_alpha)
                        {
#pragma unroll
                            for (int t = 0; t < 16; ++t) x[t] = __fmul_rn(x[t], p.alpha);
                        }
                        if (has_bias)
                        {
#pragma unroll
                            for (int t = 0; t < 16; ++t) x[t] = __fadd_rn(x[t], CF::SWAP ? brow : bias_s[cb + t]);
                        }
#pragma unroll
                        for (int t = 0; t < 8; ++t)
                        {
                            __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * t], x[2 * t + 1]);
                            packed[(b0 + b) * 8 + t] = *reinterpret_cast<uint32_t*>(&h);
                        }
                    }
                }
                // accumulator drained: let the next tile's MMAs in
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[acc]);
                if (row_valid)
                {
                    if (!CF::SWAP)
                    {
                        const int m = r0 + row;
#pragma unroll
                        for (int ch = 0; ch < NCH; ++ch)
                        {
                            const int n = c0 + half * COLS + ch * 16;
                            if (n < p.N) store_chunk16(p, m, n, packed + ch * 8);
                        }
                    }
                    else
                    {
                        const int n = r0 + row;
#pragma unroll
                        for (int t = 0; t < COLS; ++t)
                        {
                            const int m = c0 + half * COLS + t;
                            if (m < p.M)
                            {
                                const uint32_t pr = packed[t >> 1];
                                const unsigned short hbits = (t & 1) ? (unsigned short)(pr >> 16)
                                                                     : (unsigned short)(pr & 0xFFFFu);
#pragma unroll
                                for (int d = 0; d < MAX_OUT; ++d)
                                {
                                    if (d >= p.n_out) break;
                                    p.outs[d][(long long)m * p.ldc + n] = __ushort_as_bfloat16(hbits);
                                }
                            }
                        }
                    }
                }
                if (owner)
                {
                    named_bar_sync(1, NUM_EPI_THREADS);
                    if (et == 0)
                        for (int c = c_first; c <= c_last; ++c) p.flags[c] = 0u;
                }
            }
            MBS_TADD(tacc, 7);
            if (CF::ACC_BUFS == 2)
            {
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
            }
            else
            {
                acc_phase ^= 1;
            }
        }
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    __syncwarp();
    if constexpr (CF::SPLIT_OK)
    {
        if (p.ksplit > 1)
        {
            // Every role loop above ends (its waits are bounded), so every thread
            // of every CTA of the cluster reaches both barriers.
#if MBS_TIMING
            const long long t_red0 = clock64();
#endif
            cluster_sync();  // every CTA of the cluster: accumulator complete, stages idle
#if MBS_TIMING
            const long long t_red1 = clock64();
#endif
            if (warp >= EPI_WARP0)
            {
                Work w;
                const bool any = get_work(p, 0, w) && w.k1 > w.k0;
                split_push<CF>(p, smem, tmem_base, warp, lane, any);
            }
            tc_fence_before();
            cluster_sync();  // every slice in place
            tc_fence_after();
#if MBS_TIMING
            const long long t_red2 = clock64();
#endif
            split_finish<CF>(p, smem, epi_f, threadIdx.x);
#if MBS_TIMING
            if (threadIdx.x == EPI_WARP0 * 32)
            {
                tacc[12] += (unsigned long long)(t_red1 - t_red0);
                tacc[13] += (unsigned long long)(t_red2 - t_red1);
                tacc[15] += (unsigned long long)(clock64() - t_red2);
            }
#endif
        }
    }
    // output copies in other GPUs' memory: make this thread's stores visible
    // system-wide before the grid completes (a barrier on the stream follows)
    if (p.n_out > 1) __threadfence_system();
    __syncwarp();
    if (warp == 1) tmem_dealloc(tmem_base, CF::TMEM_COLS);
#if MBS_TIMING
    if (threadIdx.x == 0) tacc[9] = (unsigned long long)(clock64() - t_kernel0);
    if (threadIdx.x == 0 && blockIdx.x < 1024) g_mbs_cta[blockIdx.x * 5 + 3] = globaltimer_ns();
    if (lane == 0 && (warp <= 2 || warp == EPI_WARP0)) MBS_TFLUSH(tacc);
#else
    (void)tacc;
#endif
}


// ====================================================================== packing
// Reference weight layout (flatB + flatS) -> packed format.  Packed block
// (tile t of 256 rows, K stage ks), PACK_STAGE_BYTES long:
//   [0, 32 KB)  tile bytes in the shared-memory order the MMA reads:
//               16-byte row slice (row tile nt, K chunk c) at (c*16 + nt)*256,
//               i.e. flatB offset (t*16 + nt)*8K + (8ks + c)*256
//   [32, 34 KB) scale blocks (q, rb) at 32 KB + (2q + rb)*512, row r of the
//               tile at (r%32)*16 + ((r%128)/32)*4, byte k = scale
//               (256t + r, 8ks + 4q + k)  (the transpose_side<256> output)
// Rows past N and K chunks past K/32 are zero.
__global__ void __launch_bounds__(256) pack_weight_kernel(const uint8_t* __restrict__ B,
                                                          const uint8_t* __restrict__ BS, int N, int K, int snp,
                                                          int ks_count, long long nblocks,
                                                          uint8_t* __restrict__ packed)
{
    constexpr int V_PER_BLOCK = (256 * BKB) / 16 + 512;  // 16-byte tile pieces + scale words
    const long long total = nblocks * V_PER_BLOCK;
    const int chunks = K / 32;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x)
    {
        const long long blk = i / V_PER_BLOCK;
        const int v = (int)(i - blk * V_PER_BLOCK);
        const int t = (int)(blk / ks_count), ks = (int)(blk - (long long)t * ks_count);
        uint8_t* dst = packed + blk * PACK_STAGE_BYTES;
        if (v < (256 * BKB) / 16)
        {
            const int piece = v >> 4, sub = v & 15;  // 256-byte slice, 16-byte part
            const int c = piece >> 4, nt = piece & 15;
            const int ntile = t * 16 + nt, chunk = ks * 8 + c;
            uint4 val = make_uint4(0, 0, 0, 0);
            if (ntile * 16 < N && chunk < chunks)
                val = __ldg(reinterpret_cast<const uint4*>(B + (long long)ntile * ((long long)K * 8) +
                                                           (long long)chunk * 256) + sub);
            reinterpret_cast<uint4*>(dst)[v] = val;
        }
        else
        {
            const int wi = v - (256 * BKB) / 16;  // scale word 0..511
            const int a = wi >> 7, rr = (wi & 127) >> 2, g4 = wi & 3;  // atom, row-in-32, group
            const int q = a >> 1, rb = a & 1;
            const int r = 128 * rb + 32 * g4 + rr;
            const int row = 256 * t + r;
            uint32_t word = 0;
            if (row < N)
            {
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    word |= (uint32_t)BS[flat_s_offset(row, 8 * ks + 4 * q + k, snp)] << (8 * k);
            }
            *reinterpret_cast<uint32_t*>(dst + 256 * BKB + a * 512 + rr * 16 + g4 * 4) = word;
        }
    }
}

// ====================================================================== CTA pair
// Prefill kernel on CTA pairs (cluster of 2).  A pair tile is 256 rows of A
// by BN = 256 or 384 columns: per 64-K step one tcgen05.mma.cta_group::2 of
// 256 x 256 and, for BN = 384, a second one of 256 x 128 on the same A.  Each
// CTA contributes 128 rows of A and half of each MMA's B rows (128, plus 64)
// from its own shared memory and holds its 128 x BN accumulator in its own
// TMEM (accumulator column j = output column c0 + j).  Per SM the pair halves
// the B bytes TMA writes into shared memory compared with a single-CTA tile,
// and BN = 384 moves 20 % fewer operand bytes per FLOP than 256 (44 vs 35 KB
// per stage for 1.5x the MMA work).
//
// Scales reach it as "scale images" written by scale_image_kernel: per K
// stage and 128-row block of A or B, the two 512-byte 32x16B blocks
// tcgen05.cp.32x128b.warpx4 copies into TMEM (the copy replicates them to all
// four lane quarters).  Every image is reused by all tiles of its rows, so
// building them once per call costs a few microseconds and removes all scale
// work from the GEMM.
//
// Protocol (leader = cluster rank 0):
//   * both producers wait on their own `empty` slot (the leader's commit
//     multicasts to both), then TMA their A tile, B rows, A-scale image and
//     the tile's B-scale images with .cta_group::2, completing on the
//     LEADER's `full` barrier, which the leader's producer arms with both
//     CTAs' bytes;
//   * the leader's scale-copy thread (warp 2) waits on `full` and on its TMEM
//     scale slot being free (for BN = 384 there are fewer scale slots than
//     stages: the slot of stage g is free once the MMAs of stage g - SF_SLOTS
//     completed, i.e. that stage's `empty` commit), issues
//     tcgen05.cp.cta_group::2 (each CTA's shared memory -> its own TMEM) and
//     commits to the leader's `sfready`;
//   * the leader's MMA thread waits on `sfready` (committed only after the
//     copy thread saw `full`, so it implies the operands landed), issues the
//     pair MMAs and multicasts its commits to both CTAs' `empty` / `acc_full`.
//     (Keeping tcgen05.cp out of the MMA thread matters: a thread that issues
//     copies right after an mbarrier wait stalls ~120 cycles per stage, one
//     that issues only MMAs does not.)
//   * each CTA's epilogue drains its own TMEM and arrives on the leader's
//     `acc_empty` (16 warps).

constexpr int IMG_BLOCK = 2 * 512;  // scale image of 128 rows per K stage: [q] 32x16B blocks

// flatS scales (or macro-block B scales) -> scale images
//   img[ks][blk][q][l][16 B]: word w of row l, byte k = SF(128 blk + 32 w + l, 8 ks + 4 q + k)
// i.e. per (K stage, 128-row block, K-group set q) the 32x16B block
// tcgen05.cp.32x128b.warpx4 takes.  K-stage-major, so one stage's blocks of
// consecutive rows are contiguous (one TMA box loads a tile's B blocks).
// Rows outside the scale buffer give 0.
// One thread per (K stage, 128-row block, row-in-16 rho): it loads the 16
// flatS words of the block's four 32-row groups at that rho (word k*16 + rho
// of each group's 256-byte chunk holds the scales of rows rho and rho + 16
// for the K-group k of both sets of 4), transposes them with byte
// permutes and writes the four 16-byte rows (rho and rho + 16, both q).
// Macro-block B scales are shared by all rows of a 32-row group, so their
// image rows are copies.
__global__ void __launch_bounds__(256) scale_image_kernel(const uint8_t* __restrict__ sa, int a_rows_buf,
                                                          int a_blocks, const uint8_t* __restrict__ sb,
                                                          int b_rows_buf, int b_blocks, int snp, int ks_count,
                                                          int b_macro, int mb_ld, uint8_t* __restrict__ img_a,
                                                          uint8_t* __restrict__ img_b)
{
    // the GEMM behind this kernel may start now: it loads its first operand
    // stages and waits for this grid before it reads any image
    griddep_launch_dependents();
    const long long na = (long long)a_blocks * ks_count * 16;
    const long long nb = (long long)b_blocks * ks_count * 16;
    for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < na + nb;
         t += (long long)gridDim.x * blockDim.x)
    {
        const bool is_a = t < na;
        long long u = is_a ? t : t - na;
        const int rho = (int)(u & 15);
        u >>= 4;
        const int nblk = is_a ? a_blocks : b_blocks;
        const long long blk = u % nblk;
        const int ks = (int)(u / nblk);
        const long long row0 = blk * 128;
        const int rows_buf = is_a ? a_rows_buf : b_rows_buf;
        const uint8_t* src = is_a ? sa : sb;
        uint32_t o[4][4];  // [group][p], p = 2q + h
        if (!is_a && b_macro)
        {
#pragma unroll
            for (int g = 0; g < 4; ++g)
            {
                const long long r = row0 + 32 * g;
                uint32_t w0 = 0, w1 = 0;
                if (r < rows_buf)
                {
                    const uint8_t* m = src + (r >> 5) * mb_ld + 8 * ks;
                    w0 = (uint32_t)m[0] | ((uint32_t)m[1] << 8) | ((uint32_t)m[2] << 16) | ((uint32_t)m[3] << 24);
                    w1 = (uint32_t)m[4] | ((uint32_t)m[5] << 8) | ((uint32_t)m[6] << 16) | ((uint32_t)m[7] << 24);
                }
                o[g][0] = o[g][1] = w0;  // q = 0, both h
                o[g][2] = o[g][3] = w1;  // q = 1
            }
        }
        else
        {
#pragma unroll
            for (int g = 0; g < 4; ++g)
            {
                const long long r = row0 + 32 * g;  // 32-row group start
                uint32_t w[4] = {0, 0, 0, 0};
                if (r < rows_buf)
                {
                    const uint32_t* chunk =
                        reinterpret_cast<const uint32_t*>(src + (r >> 5) * 32 * (long long)snp + (long long)ks * 256);
#pragma unroll
                    for (int k = 0; k < 4; ++k) w[k] = __ldg(chunk + k * 16 + rho);
                }
                const uint32_t t0 = __byte_perm(w[0], w[1], 0x5140);
                const uint32_t t1 = __byte_perm(w[2], w[3], 0x5140);
                const uint32_t t2 = __byte_perm(w[0], w[1], 0x7362);
                const uint32_t t3 = __byte_perm(w[2], w[3], 0x7362);
                o[g][0] = __byte_perm(t0, t1, 0x5410);
                o[g][1] = __byte_perm(t0, t1, 0x7632);
                o[g][2] = __byte_perm(t2, t3, 0x5410);
                o[g][3] = __byte_perm(t2, t3, 0x7632);
            }
        }
        uint8_t* img = (is_a ? img_a : img_b) + ((long long)ks * nblk + blk) * IMG_BLOCK;
#pragma unroll
        for (int pp = 0; pp < 4; ++pp)
        {
            const int h = pp & 1, q = pp >> 1;
            const uint4 v4 = make_uint4(o[0][pp], o[1][pp], o[2][pp], o[3][pp]);
            *reinterpret_cast<uint4*>(img + q * 512 + (16 * h + rho) * 16) = v4;
        }
    }
}

template <int STAGES_, int BN_, bool XCHG_ = false>
struct CfgPair
{
    // XCHG: the output goes to several copies (mbs_gemm_a4w4_launch_multi, other GPUs'
    // memory among them); each epilogue warp stages 32 rows x 64 columns at a time in
    // shared memory and writes them out as 128-byte row segments
    static constexpr bool XCHG = XCHG_;
    static constexpr int BN = BN_;           // pair tile columns
    static constexpr int N2 = BN - 256;      // columns of the second MMA (0 or 128)
    static_assert(N2 == 0 || N2 == 128, "pair tiles are 256 or 384 columns wide");
    static constexpr int B1_ROWS = 128;      // B rows per CTA for the N = 256 MMA
    static constexpr int B2_ROWS = N2 / 2;   // ... for the N = 128 MMA
    static constexpr int STAGES = STAGES_;
    static constexpr int B_BLOCKS = BN / 128;  // 128-row scale image blocks of B per stage
    static constexpr int A_DATA = BM * BKB;
    static constexpr int B1_DATA = B1_ROWS * BKB;
    static constexpr int B2_DATA = B2_ROWS * BKB;
    static constexpr int A_DATA_OFF = 0;
    static constexpr int B1_DATA_OFF = A_DATA;
    static constexpr int B2_DATA_OFF = B1_DATA_OFF + B1_DATA;
    static constexpr int A_IMG_OFF = B2_DATA_OFF + B2_DATA;
    static constexpr int B_IMG_OFF = A_IMG_OFF + IMG_BLOCK;
    static constexpr int STAGE_BYTES = align_up(B_IMG_OFF + B_BLOCKS * IMG_BLOCK, 1024);
    static constexpr uint32_t TX = A_DATA + B1_DATA + B2_DATA + (1 + B_BLOCKS) * IMG_BLOCK;  // per CTA
    // TMEM: accumulator columns [0, BN); then per scale slot SFA [q] (4 columns
    // each), SFB of the N = 256 MMA [q] (8 each), SFB of the N = 128 MMA [q] (4 each)
    static constexpr int SFB1_OFF = 8;
    static constexpr int SFB2_OFF = 24;
    static constexpr int SF_STAGE_COLS = 8 + 16 + (N2 ? 8 : 0);
    static constexpr int SF_BASE = BN;  // one accumulator buffer
    static constexpr int SF_SLOTS_MAX = (512 - BN) / SF_STAGE_COLS;
    static constexpr int SF_SLOTS = STAGES < SF_SLOTS_MAX ? STAGES : SF_SLOTS_MAX;
    static constexpr int TMEM_COLS = 512;
    static_assert(SF_BASE + SF_SLOTS * SF_STAGE_COLS <= 512, "TMEM budget");
    // full, sfready, empty [STAGES]; acc_full, acc_empty; tmem slot; abort
    static constexpr int BAR_BYTES = (3 * STAGES + 2) * 8 + 16;
    static constexpr int EPI_BYTES = (BM + 2 * BN) * 4;  // factor + bias staging
    static constexpr int XCHG_WARP_BYTES = 32 * 64 * 2;   // 32 rows x 64 bf16 columns
    static constexpr int XCHG_OFF = align_up(STAGES * STAGE_BYTES + BAR_BYTES + EPI_BYTES, 128);
    static constexpr int XCHG_BYTES = XCHG ? NUM_EPI_WARPS * XCHG_WARP_BYTES : 0;
    static constexpr int SMEM_BYTES = XCHG_OFF + XCHG_BYTES + 1024;
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
    static_assert(XCHG_OFF % 16 == 0, "staging alignment");
};

template <class CF>
__global__ void __launch_bounds__(NUM_THREADS, 1) __cluster_dims__(2, 1, 1)
    mxf4_gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                          const __grid_constant__ CUtensorMap tm_b2, const __grid_constant__ CUtensorMap tm_ia,
                          const __grid_constant__ CUtensorMap tm_ib, const Params p)
{
    constexpr int BN = CF::BN;
    constexpr int STAGES = CF::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * CF::STAGE_BYTES);
    uint64_t* sfready = full + STAGES;  // leader: a stage's scales are in TMEM
    uint64_t* empty = sfready + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint64_t* acc_empty = acc_full + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* epi_f = reinterpret_cast<float*>(smem + STAGES * CF::STAGE_BYTES + CF::BAR_BYTES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int cluster = blockIdx.x >> 1;
    const int nclusters = gridDim.x >> 1;
    unsigned long long tacc[16] = {0};
#if MBS_TIMING
    const long long t_kernel0 = clock64();
#endif

    if (threadIdx.x == 0)
    {
        for (int s = 0; s < STAGES; ++s)
        {
            mbar_init(&full[s], 1);
            mbar_init(&sfready[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 2 * NUM_EPI_WARPS);
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tmap(&tm_a);
        prefetch_tmap(&tm_b);
        if (CF::N2) prefetch_tmap(&tm_b2);
        prefetch_tmap(&tm_ia);
        prefetch_tmap(&tm_ib);
    }
    if (warp == 1)
    {
        tmem_alloc_pair(tmem_slot, CF::TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();  // barriers of both CTAs initialised, TMEM allocated in both
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int tiles_r2 = (p.M + 2 * BM - 1) / (2 * BM);
    // Column tiles: all BN wide, or, in the 384-column configuration, the
    // first p.wide_c 384 wide and the rest 256 wide (a 256-wide tile issues
    // only the N = 256 MMA and skips the second MMA's B rows), so that the
    // rounds of tiles over the clusters come out even.
    const int tiles_c = CF::N2 ? p.tiles_c : (p.N + BN - 1) / BN;
    const int ntiles = tiles_r2 * tiles_c;
    auto col0 = [&](int tc) {
        return CF::N2 ? (tc < p.wide_c ? tc * 384 : p.wide_c * 384 + (tc - p.wide_c) * 256) : tc * BN;
    };
    auto is_wide = [&](int tc) { return CF::N2 != 0 && tc < p.wide_c; };

    if (warp == 0)
    {
        if (lane == 0)
        {
            const uint32_t full0 = mapa_shared(smem_u32(full), 0);  // leader's full[0]
            // image blocks per K stage
            const int a_blocks = tiles_r2 * 2, b_blocks = CF::N2 ? p.img_b_blocks : tiles_c * CF::B_BLOCKS;
            int slot = 0;
            uint32_t phase = 0;
#if MBS_TIMING
            tacc[12] += (unsigned long long)(clock64() - t_kernel0);  // prologue
#endif
            // The scale images are written by the kernel launched just
            // before this one, which may still be running (programmatic
            // dependent launch).  The first STAGES stages get their operands
            // at once and their images after griddep_wait(); every later
            // stage waits for an MMA that needed those images, so only this
            // thread has to wait.  `full` is armed for operands and images
            // together, so it completes only when both have landed.
            auto load_images = [&](int g) {
                const int t = cluster + (g / p.k_stages) * nclusters, ks = g % p.k_stages;
                const int rb = (t % tiles_r2) * 2 + (int)rank, tc = t / tiles_r2;
                uint8_t* st = smem + (g % STAGES) * CF::STAGE_BYTES;
                const uint32_t fbar = full0 + (g % STAGES) * 8;
                tma_load_2d_pair(st + CF::A_IMG_OFF, &tm_ia, fbar, 0, (ks * a_blocks + rb) * (IMG_BLOCK / 256));
                tma_load_2d_pair(st + CF::B_IMG_OFF, &tm_ib, fbar, 0,
                                 (ks * b_blocks + col0(tc) / 128) * (IMG_BLOCK / 256));
            };
            int g = 0;  // stage index in this cluster's sequence
            for (int t = cluster; t < ntiles; t += nclusters)
            {
                const int tr = t % tiles_r2, tc = t / tiles_r2;
                const int rb = tr * 2 + (int)rank;  // this CTA's 128-row block of A
                // this CTA's B rows: half of the N = 256 MMA's, half of the N = 128 MMA's
                const int nb1 = col0(tc) + (int)rank * CF::B1_ROWS;
                const int nb2 = col0(tc) + 256 + (int)rank * CF::B2_ROWS;
                const bool wide = is_wide(tc);
                for (int ks = 0; ks < p.k_stages; ++ks, ++g)
                {
                    if (g == STAGES)
                    {
                        griddep_wait();
                        for (int d = 0; d < STAGES; ++d) load_images(d);
                    }
                    bool ok_empty;
                    {
                        MBS_TSTART();
                        ok_empty = mbar_wait(&empty[slot], phase ^ 1, abort_flag);
                        MBS_TADD(tacc, 0);
                    }
                    if (!ok_empty)
                    {
                        raise_error(p, abort_flag);
                        goto pair_producer_done;
                    }
                    uint8_t* st = smem + slot * CF::STAGE_BYTES;
                    const uint32_t fbar = full0 + slot * 8;
                    if (leader) mbar_arrive_expect_tx(&full[slot], 2 * (wide ? CF::TX : CF::TX - CF::B2_DATA));
                    tma_load_2d_pair(st + CF::A_DATA_OFF, &tm_a, fbar, ks * BKB, rb * BM);
                    tma_load_3d_pair(st + CF::B1_DATA_OFF, &tm_b, fbar, 0, nb1 / 16, ks * 8);
                    if (wide) tma_load_3d_pair(st + CF::B2_DATA_OFF, &tm_b2, fbar, 0, nb2 / 16, ks * 8);
                    if (g >= STAGES) load_images(g);
#if MBS_TIMING
                    tacc[10] += 1;
#endif
                    if (++slot == STAGES)
                    {
                        slot = 0;
                        phase ^= 1;
                    }
                }
            }
            if (g <= STAGES)
            {
                // a sequence of at most STAGES stages never reached the wait
                // above (it runs at the top of stage STAGES): its images are owed
                griddep_wait();
                for (int d = 0; d < g; ++d) load_images(d);
            }
        pair_producer_done:;
        }
    }
    else if (warp == 1)
    {
        if (lane == 0 && leader)
        {
            int slot = 0, sfs = 0;  // operand slot, TMEM scale slot
            uint32_t phase = 0;
            uint32_t acc_phase = 0;
#if MBS_TIMING
            const long long t_loop0 = clock64();
#endif
            for (int t = cluster; t < ntiles; t += nclusters)
            {
                const bool wide = is_wide(t / tiles_r2);
                bool ok_acc;
                {
                    MBS_TSTART();
                    ok_acc = mbar_wait(acc_empty, acc_phase ^ 1, abort_flag);
                    MBS_TADD(tacc, 1);
                }
                if (!ok_acc)
                {
                    raise_error(p, abort_flag);
                    break;
                }
                tc_fence_after();
                bool ok = true;
                for (int ks = 0; ks < p.k_stages; ++ks)
                {
                    // `sfready` implies `full`: the scale-copy thread commits it only
                    // after it has waited for this stage's `full` (which completes
                    // once all of the stage's bytes -- operands and scale images --
                    // have landed) and its copies of those images have completed.
                    // One barrier test per stage instead of two keeps this thread,
                    // whose waits leave the tensor pipe idle, ~4 % faster.
                    bool ok_in;
                    {
                        MBS_TSTART();
                        ok_in = mbar_wait(&sfready[slot], phase, abort_flag);
                        MBS_TADD(tacc, 3);
                    }
                    if (!ok_in)
                    {
                        raise_error(p, abort_flag);
                        ok = false;
                        break;
                    }
                    MBS_TSTART();
                    tc_fence_after();
                    const uint8_t* st = smem + slot * CF::STAGE_BYTES;
                    const uint32_t sf_a = tmem_base + CF::SF_BASE + sfs * CF::SF_STAGE_COLS;
                    const uint32_t a_base = smem_u32(st + CF::A_DATA_OFF);
                    const uint32_t b1_base = smem_u32(st + CF::B1_DATA_OFF);
                    const uint32_t b2_base = smem_u32(st + CF::B2_DATA_OFF);
#pragma unroll
                    for (int j = 0; j < BK / MMA_K; ++j)
                    {
                        if (ks * BK + j * MMA_K >= p.K) break;
                        const uint64_t a_desc = make_smem_desc(a_base + j * 32, 16, 1024, 2);
                        const uint32_t id = (uint32_t)(j & 1) * 2;
                        const uint32_t q = (uint32_t)(j >> 1);
                        const uint32_t sfa = (sf_a + 4 * q) | (id << 30);
                        const uint32_t acc = (ks > 0 || j > 0) ? 1u : 0u;
                        const uint64_t b1_desc =
                            make_smem_desc(b1_base + j * 2 * (CF::B1_ROWS * 16), CF::B1_ROWS * 16, 128, 0);
                        tc_mma_mxf4_pair(tmem_base, a_desc, b1_desc, make_idesc_mxf4(2 * BM, 256, id, id), sfa,
                                         (sf_a + CF::SFB1_OFF + 8 * q) | (id << 30), acc);
                        if (wide)
                        {
                            const uint64_t b2_desc =
                                make_smem_desc(b2_base + j * 2 * (CF::B2_ROWS * 16), CF::B2_ROWS * 16, 128, 0);
                            tc_mma_mxf4_pair(tmem_base + 256, a_desc, b2_desc, make_idesc_mxf4(2 * BM, CF::N2, id, id),
                                             sfa, (sf_a + CF::SFB2_OFF + 4 * q) | (id << 30), acc);
                        }
                    }
                    tc_commit_pair_mc(&empty[slot], 0x3);
                    MBS_TADD(tacc, 11);
                    if (++slot == STAGES)
                    {
                        slot = 0;
                        phase ^= 1;
                    }
                    if (++sfs == CF::SF_SLOTS) sfs = 0;
                }
                if (!ok) break;
                {
                    MBS_TSTART();
                    tc_commit_pair_mc(acc_full, 0x3);
                    MBS_TADD(tacc, 14);
                }
                acc_phase ^= 1;
            }
#if MBS_TIMING
            tacc[13] = (unsigned long long)clock64();  // last issue time, turned into a tail below
            tacc[15] = tacc[13] - (unsigned long long)t_loop0;
#endif
        }
    }
    else if (warp == 2)
    {
        // ------------------------------------------------ scale copies (leader)
        // A thread that issues tcgen05.cp right after observing an mbarrier
        // stalls far longer than one that only issues MMAs, so the scale
        // images go to TMEM from here, one stage ahead of the MMA thread,
        // which then waits on sfready (cheap) instead.
        if (lane == 0 && leader)
        {
            int slot = 0, sfs = 0, eslot = 0;
            uint32_t phase = 0, ephase = 0;
            long long g = 0;
            for (int t = cluster; t < ntiles; t += nclusters)
            {
                bool ok = true;
                for (int ks = 0; ks < p.k_stages; ++ks, ++g)
                {
                    // the scale slot of stage g was last read by the MMAs of
                    // stage g - SF_SLOTS (their `empty` commit); with a scale
                    // slot per operand slot, `full` already implies it
                    bool ok_wait = mbar_wait(&full[slot], phase, abort_flag);
                    if (CF::SF_SLOTS < STAGES && g >= CF::SF_SLOTS)
                    {
                        ok_wait = ok_wait && mbar_wait(&empty[eslot], ephase, abort_flag);
                        if (++eslot == STAGES)
                        {
                            eslot = 0;
                            ephase ^= 1;
                        }
                    }
                    if (!ok_wait)
                    {
                        raise_error(p, abort_flag);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint8_t* st = smem + slot * CF::STAGE_BYTES;
                    const uint32_t sf_a = tmem_base + CF::SF_BASE + sfs * CF::SF_STAGE_COLS;
                    // SFA: one 32x16B block per K-group set q; SFB: per q, one per 128-row block
#pragma unroll
                    for (int q = 0; q < 2; ++q)
                    {
                        tc_cp_32x128b_warpx4_pair(sf_a + 4 * q,
                                                  make_smem_desc(smem_u32(st + CF::A_IMG_OFF + q * 512), 0, 128, 0));
#pragma unroll
                        for (int b = 0; b < CF::B_BLOCKS; ++b)
                        {
                            const uint32_t col = b < 2 ? CF::SFB1_OFF + 8 * q + 4 * b : CF::SFB2_OFF + 4 * q;
                            tc_cp_32x128b_warpx4_pair(
                                sf_a + col,
                                make_smem_desc(smem_u32(st + CF::B_IMG_OFF + b * IMG_BLOCK + q * 512), 0, 128, 0));
                        }
                    }
                    tc_commit_pair_mc(&sfready[slot], 0x1);
                    if (++slot == STAGES)
                    {
                        slot = 0;
                        phase ^= 1;
                    }
                    if (++sfs == CF::SF_SLOTS) sfs = 0;
                }
                if (!ok) break;
            }
        }
    }
    else if (warp >= EPI_WARP0)
    {
        const int e = warp - EPI_WARP0;
        const int quarter = warp & 3;
        const int half = e >> 2;
        const int row = quarter * 32 + lane;
        const int et = threadIdx.x - EPI_WARP0 * 32;
        constexpr int COLS = BN / 2;
        constexpr int NCH = COLS / 16;
        constexpr int BATCH = COLS > 128 ? 2 : 4;  // 384-column tiles hold 96 packed words per thread
        const bool has_factor = (p.a_factor != nullptr) || (p.b_factor != nullptr);
        const bool has_alpha = p.alpha != 1.0f;
        const bool has_bias = p.bias != nullptr;
        const uint32_t acc_empty0 = mapa_shared(smem_u32(acc_empty), 0);
        float* fr_s = epi_f;
        float* fc_s = epi_f + BM;
        float* bias_s = epi_f + BM + BN;
        uint32_t acc_phase = 0;
        for (int t = cluster; t < ntiles; t += nclusters)
        {
            const int tr = t % tiles_r2, tc = t / tiles_r2;
            const int r0 = tr * 2 * BM + (int)rank * BM;
            const int c0 = col0(tc);
            const int c_end = c0 + (CF::N2 && !is_wide(tc) ? 256 : BN);  // columns this tile computes
            if (has_factor || has_bias)
            {
                named_bar_sync(1, NUM_EPI_THREADS);
                if (et < BM)
                {
                    const int r = r0 + et;
                    fr_s[et] = (p.a_factor != nullptr && r < p.M) ? byte_to_factor(p.a_factor[r]) : 1.0f;
                }
                for (int j = et; j < BN; j += NUM_EPI_THREADS)
                {
                    const int c = c0 + j;
                    fc_s[j] = (p.b_factor != nullptr && c < p.N) ? byte_to_factor(p.b_factor[c]) : 1.0f;
                    bias_s[j] = (has_bias && c < p.N) ? __bfloat162float(p.bias[c]) : 0.0f;
                }
                named_bar_sync(1, NUM_EPI_THREADS);
            }
            bool ok_acc;
            {
                MBS_TSTART();
                ok_acc = mbar_wait(acc_full, acc_phase, abort_flag);
                MBS_TADD(tacc, 6);
            }
            // all epilogue warps take the same branch, so none is left behind in a named barrier
            ok_acc = named_bar_and(1, NUM_EPI_THREADS, ok_acc);
            if (!ok_acc)
            {
                if (lane == 0) raise_error(p, abort_flag);
                break;
            }
            MBS_TSTART();
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + half * COLS;
            uint32_t packed[COLS / 2];
            const float fr = has_factor ? fr_s[row] : 1.0f;
#pragma unroll
            for (int b0 = 0; b0 < NCH; b0 += BATCH)
            {
                uint32_t v[BATCH][16];
#pragma unroll
                for (int b = 0; b < BATCH; ++b) tc_ld_32x32b_x16(taddr + (b0 + b) * 16, v[b]);
                tc_wait_ld();
#pragma unroll
                for (int b = 0; b < BATCH; ++b)
                {
                    const int cb = half * COLS + (b0 + b) * 16;
                    float x[16];
#pragma unroll
                    for (int u = 0; u < 16; ++u) x[u] = __uint_as_float(v[b][u]);
                    if (has_factor)
                    {
#pragma unroll
                        for (int u = 0; u < 16; ++u) x[u] = __fmul_rn(x[u], __fmul_rn(fr, fc_s[cb + u]));
                    }
                    if (has_alpha)
                    {
#pragma unroll
                        for (int u = 0; u < 16; ++u) x[u] = __fmul_rn(x[u], p.alpha);
                    }
                    if (has_bias)
                    {
#pragma unroll
                        for (int u = 0; u < 16; ++u) x[u] = __fadd_rn(x[u], bias_s[cb + u]);
                    }
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                    {
                        __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * u], x[2 * u + 1]);
                        packed[(b0 + b) * 8 + u] = *reinterpret_cast<uint32_t*>(&h);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
            {
                if (leader)
                    mbar_arrive(acc_empty);
                else
                    mbar_arrive_cluster(acc_empty0);
            }
            const int m = r0 + row;
            if constexpr (CF::XCHG)
            {
                // 64 columns at a time: each thread puts its row's eight 16-byte pieces
                // into the warp's staging block (piece q of row r at slot q ^ (r & 7), so
                // 8 consecutive lanes hit 8 different bank groups), then lane l writes
                // piece l & 7 of row 4i + (l >> 3): 8 lanes cover 128 contiguous bytes
                // of one output row, which is what NVLink moves efficiently (32-byte
                // pieces scattered over 32 rows ran ~4x slower to another GPU).
                uint4* stg = reinterpret_cast<uint4*>(smem + CF::XCHG_OFF + e * CF::XCHG_WARP_BYTES);
#pragma unroll
                for (int grp = 0; grp < COLS / 64; ++grp)
                {
                    __syncwarp();
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                    {
                        const uint32_t* w = packed + grp * 32 + q * 4;
                        stg[lane * 8 + (q ^ (lane & 7))] = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                    __syncwarp();
                    const int q = lane & 7;
                    const int n = c0 + half * COLS + grp * 64 + q * 8;
                    const bool col_ok = n < p.N && n < c_end;
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                    {
                        const int rr = 4 * i + (lane >> 3);  // row of the warp's 32
                        const uint4 v = stg[rr * 8 + (q ^ (rr & 7))];
                        const long long mm = (long long)r0 + quarter * 32 + rr;
                        if (col_ok && mm < p.M)
                        {
                            const long long off = mm * p.ldc + n;
#pragma unroll
                            for (int d = 0; d < MAX_OUT; ++d)
                            {
                                if (d >= p.n_out) break;
                                *reinterpret_cast<uint4*>(p.outs[d] + off) = v;
                            }
                        }
                    }
                }
            }
            else if (m < p.M)
            {
#pragma unroll
                for (int ch = 0; ch < NCH; ++ch)
                {
                    const int n = c0 + half * COLS + ch * 16;
                    if (n < p.N && n < c_end) store_chunk16(p, m, n, packed + ch * 8);
                }
            }
            MBS_TADD(tacc, 7);
            acc_phase ^= 1;
        }
    }

    if (p.n_out > 1) __threadfence_system();  // output copies in other GPUs' memory
    __syncwarp();
    tc_fence_before();
    cluster_sync();  // no remote arrive or pair MMA can still target this CTA
    tc_fence_after();
    __syncwarp();
    if (warp == 1) tmem_dealloc_pair(tmem_base, CF::TMEM_COLS);
#if MBS_TIMING
    if (threadIdx.x == 0) tacc[9] = (unsigned long long)(clock64() - t_kernel0);
    if (tacc[13]) tacc[13] = (unsigned long long)clock64() - tacc[13];  // last issue -> exit
    if (lane == 0 && (warp <= 1 || warp == EPI_WARP0)) MBS_TFLUSH(tacc);
#else
    (void)tacc;
#endif
}

}  // namespace gemm
}  // namespace mbs

// ====================================================================== host
namespace mbs {
namespace gemm {
namespace {

struct Problem
{
    const uint8_t *A, *B, *AS, *BS, *AF, *BF;
    void* out;
    int M, N, K, Mpad, snp, mb_ld;
    bool macro;
    bool packed = false;  // B is in the packed format (BS unused)
    float alpha = 1.0f;   // output scale
    const void* bias = nullptr;  // bf16 [N] or null
    // extra output copies (mbs_gemm_a4w4_launch_multi): out_dst[0..n_dst) with row stride ldc;
    // n_dst == 0 means the single buffer `out` with row stride N
    void* const* out_dst = nullptr;
    int n_dst = 0;
    long long ldc = 0;
    // fused activation quantiser (mbs_quant_gemm_a4w4_launch): A / AS point into the
    // workspace and are written by the GEMM itself from bf16 qx [M, qx_ld]
    const void* qx = nullptr;
    int qx_ld = 0;
    unsigned* qbar = nullptr;
};

// The output copies of a launch: `out` alone with row stride N, or the
// caller's list (validated by run()).
void set_outputs(Params& p, const Problem& pb)
{
    const int n = pb.n_dst > 0 ? pb.n_dst : 1;
    p.n_out = n;
    p.ldc = pb.n_dst > 0 ? pb.ldc : pb.N;
    bool v8 = (p.ldc * 2) % 32 == 0;
    for (int d = 0; d < MAX_OUT; ++d)
    {
        void* ptr = d < n ? (pb.n_dst > 0 ? pb.out_dst[d] : pb.out) : nullptr;
        p.outs[d] = static_cast<__nv_bfloat16*>(ptr);
        if (d < n && (reinterpret_cast<uintptr_t>(ptr) & 31) != 0) v8 = false;
    }
    p.out = p.outs[0];
    p.out_v8 = v8 ? 1 : 0;  // every copy's rows start 32-byte aligned: 32-byte stores
}

struct Plan
{
    int bn;
    int r_rows;  // rows of A loaded per stage (non-swapped single-CTA path)
    bool swap, sk, pair;
    int pair_bn;  // CTA-pair configuration: 256-column tiles, or 384 (mixed with 256)
    int pair_tiles_c, pair_wide_c;  // ... column tiles, of which the first pair_wide_c 384 wide
    int pair_img_b_blocks;          // ... 128-row B scale image blocks per K stage
    int ksplit;                     // single-CTA kernel: cluster split-K factor (1 = none)
    int G, tiles_r, tiles_c, k_stages;
    size_t ws_bytes;
};

// Measurement hook (mbs_set_profile_events): events recorded on the launch
// stream immediately before and after the main GEMM kernel of the next calls.
thread_local cudaEvent_t g_ev_before = nullptr, g_ev_after = nullptr;

// Upper bound on the CTAs of the next GEMM launches from this host thread
// (0 = one per SM): leaves SMs free for kernels that must run alongside, such
// as the NCCL kernels of an overlapped all-gather.
thread_local int g_grid_limit = 0;

// Test hook (mbs_set_withhold_release): stream-K contributors of the next
// launches from this host thread never release their completion flags.
thread_local int g_withhold_release = 0;


int record_before(cudaStream_t s)
{
    if (g_ev_before == nullptr) return MBS_OK;
    cudaError_t e = cudaEventRecord(g_ev_before, s);
    return e == cudaSuccess ? MBS_OK : cuda_fail(e, "cudaEventRecord (profile)");
}

int record_after(cudaStream_t s)
{
    if (g_ev_after == nullptr) return MBS_OK;
    cudaError_t e = cudaEventRecord(g_ev_after, s);
    return e == cudaSuccess ? MBS_OK : cuda_fail(e, "cudaEventRecord (profile)");
}

int env_int(const char* name, int dflt)
{
    const char* v = getenv(name);
    return (v != nullptr && *v != 0) ? atoi(v) : dflt;
}

// Schedule overrides of the following plans on this host thread
// (mbs_set_plan_override; "auto" values keep the planner's own choice).  The
// launch path reads no environment variable: the tests reach every schedule
// on small shapes through this explicit, thread-local hook.
constexpr mbs_plan_override kAutoOverride = {0, 0, -1, -1, 0, 0, -1, 0};
thread_local mbs_plan_override g_ov = kAutoOverride;

// The pair GEMM starts behind its scale-image pre-pass by programmatic
// dependent launch; MBS_PAIR_PDL=0 launches it in plain stream order.
bool pair_pdl_enabled()
{
    static const bool on = env_int("MBS_PAIR_PDL", 1) != 0;
    return on;
}

// The single-CTA GEMM may start while the kernel before it in the stream
// finishes (programmatic dependent launch); MBS_PDL=0 launches it in plain
// stream order.
bool pdl_enabled()
{
    static const bool on = env_int("MBS_PDL", 1) != 0;
    return on;
}

// Workspace of the CTA-pair path: the A and B scale images.
size_t pair_image_a_bytes(int M, int K)
{
    const size_t blocks = (size_t)((M + 2 * BM - 1) / (2 * BM)) * 2;
    return blocks * ((K + BK - 1) / BK) * IMG_BLOCK;
}


struct Plan;
size_t sk_partial_bytes(const Plan& pl);

// Every workspace starts with the stream-K flag words at a fixed place, so
// that no schedule's scratch (partials, scale images) ever lands on another
// schedule's flags when one workspace serves several shapes.
constexpr size_t kFlagBytes = MBS_GEMM_WS_FLAG_BYTES;
// stream-K flag words [0, kMaxGrid); the last two words are the fused
// quantiser's grid barrier (arrived, departed)
constexpr int kMaxGrid = (int)(kFlagBytes / sizeof(unsigned)) - 2;
constexpr int kQuantBarrierWord = kMaxGrid;

// Path and schedule choice.  Skinny M (decode) loads only its 32 or 64
// activation rows per stage and uses stream-K so every SM streams an equal
// share of the weights; larger M runs data-parallel tiles (stream-K only for
// a very deep K over few tiles).
// The thread's plan override (mbs_set_plan_override) can force the schedule,
// the grid, CTA pairs, the swapped form, pair tile widths and cluster split-K.
Plan make_plan(int M, int N, int K, int num_sms, bool packed = false)
{
    Plan pl{};
    // Skinny M keeps the weights in the N = 256 operand (one 128x256x64 MMA
    // per 8 KB of weights) and loads only the activation rows that exist;
    // An override swap = 1 selects the swapped form (weights as the 128-row operand).
    const mbs_plan_override& ov = g_ov;
    pl.swap = false;
    if (ov.swap == 1 && M <= 64 && !packed) pl.swap = true;
    pl.bn = pl.swap ? (M <= 32 ? 32 : 64) : 256;
    pl.r_rows = pl.swap ? 128 : (M <= 32 ? 32 : (M <= 64 ? 64 : 128));
    pl.k_stages = (K + BK - 1) / BK;
    if (pl.swap)
    {
        pl.tiles_r = (N + BM - 1) / BM;
        pl.tiles_c = (M + pl.bn - 1) / pl.bn;
    }
    else
    {
        pl.tiles_r = (M + BM - 1) / BM;
        pl.tiles_c = (N + pl.bn - 1) / pl.bn;
    }
    const long long tiles = (long long)pl.tiles_r * pl.tiles_c;
    // Cluster split-K for few 128-row tiles: the S CTAs of a cluster run one
    // tile's K stages in S ranges and add their fp32 partials through
    // distributed shared memory, so S times the SMs stream the operands and no
    // partial touches global memory.  Tiles are 128 x 256 or 128 x 128 (the
    // narrower tile doubles the clusters and halves each CTA's hand-over, but
    // moves 1.5x the operand bytes per FLOP).  Among (BN, S) in {256, 128} x
    // {2, 4} whose CTAs fit on the SMs, the plan takes the least estimated
    // time per CTA,
    //   6.1 us + 0.0132 us/KB * operand KB + 0.0497 us/KB * KB handed to other CTAs,
    // a fit to back-to-back B200 timings (1024x1024x5120 16.9 us on CTA
    // pairs -> 13.8 at 256 x S4 -> 12.5 at 128 x S2; 256x1024x8192 22.3 ->
    // 11.5 at 128 x S4; 1024x1024x2048 12.3 -> 9.3 at 128 x S2;
    // 128x7168x16384 29.4 -> 21.3 at 256 x S4).  A split needs 8 or more K
    // stages (256x512x1024, 4 stages: 8.0 -> 9.9 us at S = 2); clusters of 8
    // fit too few at a time.  The schedule overrides below turn it off; an
    // override ksplit = S forces S (2, 4 or 8, checked when the override is
    // set, so R_ROWS / S is always a whole number of rows) with split_bn = 128
    // or 256 (256 for skinny tiles, whose configurations exist only at 256),
    // ksplit = 0 turns it off.
    pl.ksplit = 1;
    {
        const int force_split = ov.ksplit;
        const bool overridden = ov.schedule != 0 || ov.grid != 0 || ov.pair == 1;
        int lim = num_sms;
        if (g_grid_limit > 0 && g_grid_limit < lim) lim = g_grid_limit;
        int split_bn = 256;
        if (!pl.swap && force_split > 1)
        {
            if ((force_split == 2 || force_split == 4 || force_split == 8) && force_split <= pl.k_stages &&
                tiles * force_split < (1LL << 31))
            {
                pl.ksplit = force_split;
                split_bn = (ov.split_bn == 128 && !packed && pl.r_rows == 128) ? 128 : 256;
            }
        }
        else if (!pl.swap && pl.r_rows == 128 && force_split != 0 && !overridden && pl.k_stages >= 8)
        {
            double best = 1e300;
            for (int bn : {256, 128})
            {
                if (bn == 128 && packed) continue;  // packed weights come in 256-row tiles
                const long long t = (long long)pl.tiles_r * ((N + bn - 1) / bn);
                const double stage_kb = bn == 256 ? 51.0 : 34.0;  // A + B tiles + raw scales per K stage
                for (int S : {2, 4})
                {
                    if (t * S > lim || pl.k_stages < 2 * S) continue;
                    const double per_cta = 6.1 + 0.0132 * ((pl.k_stages + S - 1) / S) * stage_kb +
                                           0.0497 * (double)(S - 1) / S * (bn / 2);
                    if (per_cta < best)
                    {
                        best = per_cta;
                        pl.ksplit = S;
                        split_bn = bn;
                    }
                }
            }
        }
        else if (!pl.swap && pl.r_rows < 128 && force_split != 0 && !overridden)
        {
            // Skinny (decode) tiles with room for every tile's split on the SMs:
            // the stream-K owner of a tile otherwise waits for its contributors'
            // partials through L2 (16x8192x8192: streaming done at ~5 us, the
            // last owner at ~15 us).  The largest S in 8, 4, 2 leaving every CTA
            // 4 or more K stages, clusters of 8 only for up to 8 tiles (more of
            // them do not fit at a time).  Back to back: 16x8192x8192 16.4 ->
            // 12.6 us, 32x4096x4096 13.9 -> 9.2, 16x1024x8192 14.9 -> 9.7 (S = 8),
            // 64x14336x4096 16.5 -> 13.0.
            for (int S : {8, 4, 2})
            {
                if (S == 8 && tiles > 8) continue;
                if (tiles * S <= lim && pl.k_stages >= 4 * S)
                {
                    pl.ksplit = S;
                    break;
                }
            }
        }
        if (pl.ksplit > 1)
        {
            pl.bn = split_bn;
            pl.tiles_c = (N + split_bn - 1) / split_bn;
            pl.sk = false;
            pl.pair = false;
            pl.G = (int)((long long)pl.tiles_r * pl.tiles_c * pl.ksplit);
            pl.ws_bytes = 0;
            return pl;
        }
    }
    // Stream-K where its partial tiles are small (skinny activations: 32- or
    // 64-row partials, an HBM-bound stream) or where a data-parallel tile
    // would run a very deep K alone on a mostly idle GPU.  With 128-row
    // tiles every contributor moves a 128 KB fp32 partial, which measured
    // 10-30 % slower than data-parallel tiles at M in 128..2048 even when
    // those leave SMs idle.
    pl.sk = pl.swap || pl.r_rows < 128 || (tiles * 4 <= num_sms && pl.k_stages >= 64);
    const int force = ov.schedule;
    if (force == 1) pl.sk = true;
    if (force == 2) pl.sk = false;
    int G = num_sms < kMaxGrid ? num_sms : kMaxGrid;
    if (g_grid_limit > 0 && g_grid_limit < G) G = g_grid_limit;
    const int fg = ov.grid;
    if (fg > 0 && fg < G) G = fg;
    const long long units = pl.sk ? tiles * pl.k_stages : tiles;
    // Stream-K ranges of at least 8 K-stages (16 for 128-row partials) per
    // CTA: with shorter ones the partial traffic of the many contributors to
    // each tile outweighs the extra SMs (full decode shapes keep every SM).
    if (pl.sk && !pl.swap && fg == 0)
    {
        const long long per = units / (pl.r_rows == 128 ? 16 : 8);
        const long long cap = per > tiles ? per : tiles;
        if (cap < G) G = (int)cap;
    }
    pl.G = (int)(units < G ? units : G);
    pl.ws_bytes = pl.sk ? kFlagBytes + sk_partial_bytes(pl) : 0;
    // Data-parallel problems with at least 4 pair tiles run on CTA pairs
    // (256-row tiles; their workspace holds the scale images); below that the
    // scale-image pre-pass (a second launch) costs more than the pair saves.
    const long long tr2 = (M + 2 * BM - 1) / (2 * BM);
    const long long t2 = tr2 * ((N + 255) / 256);
    const int force_pair = ov.pair;
    pl.pair = !packed && !pl.swap && !pl.sk && force_pair != 0 && (t2 >= 4 || force_pair == 1);
    if (pl.pair)
    {
        // 384-column tiles do 1.5x the MMA work of 256-column ones for 1.26x
        // the bytes and measure ~1.39x the time.  Two configurations: all
        // tiles 256 wide (6 pipeline stages), or nw 384-wide column tiles
        // followed by 256-wide ones (5 stages of 44 KB; a 256-wide tile
        // there measures ~1.1x a 256-wide tile of the first).  Tiles go to
        // the clusters round-robin, wide ones first; take the layout whose
        // busiest cluster has the least work.  An override pair_bn = 256 / 384
        // forces all-256 / all-384 tiles, pair_wide = nw a given mix.
        const int c = G / 2;
        const int force_bn = ov.pair_bn;
        const int force_wide = ov.pair_wide;
        auto busiest = [&](long long T, long long A, double w_wide, double w_narrow) {
            double mx = 0;
            const long long cl = T < c ? T : c;
            for (long long k = 0; k < cl; ++k)
            {
                const long long n_k = (T - 1 - k) / c + 1;
                const long long a_k = k < A ? (A - 1 - k) / c + 1 : 0;
                const double load = (double)a_k * w_wide + (double)(n_k - a_k) * w_narrow;
                if (load > mx) mx = load;
            }
            return mx;
        };
        const double cost256 = busiest(t2, 0, 1.0, 1.0);
        double best = 1e300;
        int best_nw = 0, best_nn = 0;
        const int max_wide = (N + 383) / 384;
        for (int nw = 1; nw <= max_wide; ++nw)
        {
            const int rest = N - nw * 384;
            const int nn = rest > 0 ? (rest + 255) / 256 : 0;
            if (force_wide > 0 && nw != (force_wide < max_wide ? force_wide : max_wide)) continue;
            if (force_bn == 384 && nw != max_wide) continue;
            const double cost = busiest(tr2 * (nw + nn), tr2 * nw, 1.39, 1.1);
            if (cost < best)
            {
                best = cost;
                best_nw = nw;
                best_nn = nn;
            }
        }
        const bool use384 = force_bn == 384 || force_wide > 0 || (force_bn != 256 && best < cost256);
        pl.pair_bn = use384 ? 384 : 256;
        pl.pair_wide_c = use384 ? best_nw : 0;
        pl.pair_tiles_c = use384 ? best_nw + best_nn : (N + 255) / 256;
        const long long tp = tr2 * pl.pair_tiles_c;
        // B scale images: whole tiles of 128-row blocks, plus one block so the
        // last 256-wide tile's 3-block image box stays inside the buffer
        pl.pair_img_b_blocks = use384 ? (best_nw * 384 + best_nn * 256) / 128 + 1 : pl.pair_tiles_c * 2;
        const size_t ia = pair_image_a_bytes(M, K);
        const size_t ib = (size_t)pl.pair_img_b_blocks * pl.k_stages * IMG_BLOCK;
        // TMA row coordinates of the images are 32-bit
        if (ia / 256 < (size_t)INT32_MAX && ib / 256 < (size_t)INT32_MAX)
        {
            pl.G = 2 * (int)(tp < c ? tp : c);
            pl.ws_bytes = kFlagBytes + ia + ib;
        }
        else
        {
            pl.pair = false;
        }
    }
    return pl;
}

// Stream-K partials: one [BN][rows] fp32 slot per CTA, rows = the rows of
// the R operand that can hold valid outputs.
size_t sk_partial_bytes(const Plan& pl)
{
    const int rows = pl.swap ? BM : pl.r_rows;
    return (size_t)pl.G * rows * pl.bn * sizeof(float);
}

int validate(const Problem& pb)
{
    if (!pb.A || !pb.B || !pb.AS || (!pb.BS && !pb.packed) || !pb.out)
        return fail(MBS_ERR_INVALID_ARGUMENT, "gemm_a4w4: A, B, scales and out must be non-NULL");
    if (pb.M <= 0 || pb.N <= 0 || pb.K <= 0)
        return fail(MBS_ERR_INVALID_ARGUMENT, "gemm_a4w4: M, N, K must be positive (M=%d N=%d K=%d)",
                    pb.M, pb.N, pb.K);
    if (pb.N % 16 != 0)
        return fail(MBS_ERR_UNSUPPORTED_SHAPE, "gemm_a4w4: N must be a multiple of 16, got %d", pb.N);
    if (pb.K % 64 != 0)
        return fail(MBS_ERR_UNSUPPORTED_SHAPE,
                    "gemm_a4w4: K must be a multiple of 64 (whole preshuffle K tiles), got %d", pb.K);
    if (pb.M > (1 << 30) || pb.N > (1 << 30) || pb.K > (1 << 24))
        return fail(MBS_ERR_UNSUPPORTED_SHAPE, "gemm_a4w4: problem too large");
    if (pb.Mpad < pb.M || pb.Mpad % 32 != 0)
        return fail(MBS_ERR_INVALID_ARGUMENT, "gemm_a4w4: Mpad (%d) must be a multiple of 32 >= M (%d)",
                    pb.Mpad, pb.M);
    if (pb.snp % 8 != 0 || pb.snp < pb.K / 32)
        return fail(MBS_ERR_INVALID_ARGUMENT,
                    "gemm_a4w4: scaleN_pad (%d) must be a multiple of 8 >= K/32 (%d)", pb.snp, pb.K / 32);
    if (pb.macro && (pb.mb_ld % 16 != 0 || pb.mb_ld < pb.K / 32))
        return fail(MBS_ERR_INVALID_ARGUMENT, "gemm_a4w4: mb_ld (%d) must be a multiple of 16 >= K/32",
                    pb.mb_ld);
    if (!aligned16(pb.A) || !aligned16(pb.B) || !aligned16(pb.AS) || (!pb.packed && !aligned16(pb.BS)) ||
        !aligned16(pb.out))
        return fail(MBS_ERR_MISALIGNED, "gemm_a4w4: A, B, scales and out must be 16-byte aligned");
    if (pb.n_dst > 0)
    {
        if (pb.n_dst > MAX_OUT)
            return fail(MBS_ERR_INVALID_ARGUMENT, "gemm_a4w4: at most %d output copies, got %d", MAX_OUT,
                        pb.n_dst);
        if (pb.ldc < pb.N || pb.ldc % 8 != 0 || pb.ldc > (1LL << 40))
            return fail(MBS_ERR_INVALID_ARGUMENT,
                        "gemm_a4w4: ldc (%lld) must be a multiple of 8 and at least N (%d)", pb.ldc, pb.N);
        for (int d = 0; d < pb.n_dst; ++d)
        {
            if (pb.out_dst[d] == nullptr)
                return fail(MBS_ERR_INVALID_ARGUMENT, "gemm_a4w4: output copy %d is NULL", d);
            if (!aligned16(pb.out_dst[d]))
                return fail(MBS_ERR_MISALIGNED, "gemm_a4w4: output copy %d is not 16-byte aligned", d);
        }
    }
    return MBS_OK;
}

// Row capacity of the GEMM's in-stage quantiser for these bf16 activations:
// 8 (one converting warp), 16 (two, with packed weights), or 0 (A is
// quantised in global memory: by the GEMM's idle warps or, for packed
// weights, by the stand-alone quantiser first).
int in_stage_quant(const Problem& pb, const Plan& pl)
{
    if (pb.qx == nullptr || pl.swap || pl.pair || pb.macro || pl.r_rows != 32 || pl.bn != 256) return 0;
    if (pb.M <= 8) return 8;
    return pb.packed && pb.M <= 16 ? 16 : 0;
}

// Rows per activation TMA box: the activation operand's rows per tile, cut to
// M when a single tile holds them all (TMA zero-fill of the rows past M costs
// stream time; those shared-memory rows only feed accumulator rows that are
// never stored).
int act_box_rows(const Problem& pb, const Plan& pl)
{
    const int tile_rows = pl.swap ? pl.bn : pl.r_rows;
    return pb.M < tile_rows ? pb.M : tile_rows;
}

// TMA descriptors for the four operands of one launch (with the in-stage
// quantiser, tm_r maps the bf16 activations and the activation-scale map is
// unused).
int make_maps(const Problem& pb, const Plan& pl, CUtensorMap* tm_r, CUtensorMap* tm_c,
              CUtensorMap* tm_rsf, CUtensorMap* tm_csf, bool x_in_stage = false)
{
    const int r_rows = pl.swap ? BM : pl.r_rows, c_rows = pl.bn;
    const int act_rows = pl.swap ? c_rows : r_rows;
    const int w_rows = pl.swap ? r_rows : c_rows;
    CUtensorMap* act_map = pl.swap ? tm_c : tm_r;
    CUtensorMap* w_map = pl.swap ? tm_r : tm_c;
    CUtensorMap* act_sf = pl.swap ? tm_csf : tm_rsf;
    CUtensorMap* w_sf = pl.swap ? tm_rsf : tm_csf;
    const uint64_t Kp = (uint64_t)pb.K / 2;
    int st;
    if (x_in_stage)
    {  // bf16 activations [M, K] (row stride qx_ld) for the in-stage quantiser:
       // plain boxes of {BK values, rows}; values past K read as zero
        const uint64_t dims[2] = {(uint64_t)pb.K, (uint64_t)pb.M};
        const uint64_t strides[1] = {(uint64_t)pb.qx_ld * 2};
        const uint32_t box[2] = {BK, (uint32_t)act_box_rows(pb, pl)};
        st = encode_tmap(act_map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void*)pb.qx, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st) return st;
        memset(act_sf, 0, sizeof(CUtensorMap));  // the scales come from the quantiser warps
    }
    else
    {  // activations: plain [M, K/2], 128-byte swizzled boxes of {128 B, rows}
        const uint64_t dims[2] = {Kp, (uint64_t)pb.M};
        const uint64_t strides[1] = {Kp};
        const uint32_t box[2] = {BKB, (uint32_t)act_box_rows(pb, pl)};
        st = encode_tmap(act_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)pb.A, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
        if (st) return st;
    }
    if (pb.packed)
    {  // weights and their scales come from the packed buffer by bulk copies
        memset(w_map, 0, sizeof(CUtensorMap));
        memset(w_sf, 0, sizeof(CUtensorMap));
    }
    if (!pb.packed)
    {  // weights: flatB as {256 B block, row tile (16 rows), K chunk (16 B)}
        const uint64_t dims[3] = {256, (uint64_t)pb.N / 16, (uint64_t)pb.K / 32};
        const uint64_t strides[2] = {(uint64_t)pb.K * 8, 256};
        const uint32_t box[3] = {256, (uint32_t)w_rows / 16, BK / 32};
        st = encode_tmap(w_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, (void*)pb.B, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st) return st;
    }
    if (!x_in_stage)
    {  // activation scales: flatS as {256 B chunk, K-stage, 32-row group}
        const uint64_t dims[3] = {256, (uint64_t)pb.snp / 8, (uint64_t)pb.Mpad / 32};
        const uint64_t strides[2] = {256, (uint64_t)pb.snp * 32};
        const uint32_t box[3] = {256, 1, (uint32_t)act_rows / 32};
        st = encode_tmap(act_sf, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, (void*)pb.AS, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st) return st;
    }
    if (pb.packed)
    {
    }
    else if (!pb.macro)
    {  // weight scales: flatS, roundup(N,32) rows
        const uint64_t dims[3] = {256, (uint64_t)pb.snp / 8, (uint64_t)(pb.N + 31) / 32};
        const uint64_t strides[2] = {256, (uint64_t)pb.snp * 32};
        const uint32_t box[3] = {256, 1, (uint32_t)w_rows / 32};
        st = encode_tmap(w_sf, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, (void*)pb.BS, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    else
    {  // weight macro scales: [ceil(N/32), mb_ld], boxes of {16 K-groups, row groups}
        const uint64_t dims[2] = {(uint64_t)pb.mb_ld, (uint64_t)(pb.N + 31) / 32};
        const uint64_t strides[1] = {(uint64_t)pb.mb_ld};
        const uint32_t box[2] = {16, (uint32_t)w_rows / 32};
        st = encode_tmap(w_sf, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)pb.BS, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    return st;
}

// TMA descriptors of the CTA-pair kernel: A boxes of 128 rows, B boxes of the
// CTA's 128 (and 64) rows, and the scale images as rows of 256 bytes (one
// 128-row block of A, a tile's 2 or 3 blocks of B).
int make_maps_pair(const Problem& pb, int pair_bn, void* img_a, size_t img_a_bytes, void* img_b,
                   size_t img_b_bytes, CUtensorMap* tm_a, CUtensorMap* tm_b, CUtensorMap* tm_b2, CUtensorMap* tm_ia,
                   CUtensorMap* tm_ib)
{
    const uint64_t Kp = (uint64_t)pb.K / 2;
    int st;
    {
        const uint64_t dims[2] = {Kp, (uint64_t)pb.M};
        const uint64_t strides[1] = {Kp};
        const uint32_t box[2] = {BKB, BM};
        st = encode_tmap(tm_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)pb.A, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
        if (st) return st;
    }
    for (int which = 0; which < 2; ++which)
    {
        const int rows = which == 0 ? 128 : 64;
        CUtensorMap* m = which == 0 ? tm_b : tm_b2;
        if (which == 1 && pair_bn == 256)
        {
            *m = *tm_b;  // unused
            break;
        }
        const uint64_t dims[3] = {256, (uint64_t)pb.N / 16, (uint64_t)pb.K / 32};
        const uint64_t strides[2] = {(uint64_t)pb.K * 8, 256};
        const uint32_t box[3] = {256, (uint32_t)rows / 16, BK / 32};
        st = encode_tmap(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, (void*)pb.B, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st) return st;
    }
    {
        const uint64_t dims[2] = {256, (uint64_t)(img_a_bytes / 256)};
        const uint64_t strides[1] = {256};
        const uint32_t box[2] = {256, IMG_BLOCK / 256};
        st = encode_tmap(tm_ia, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, img_a, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st) return st;
    }
    {
        const uint64_t dims[2] = {256, (uint64_t)(img_b_bytes / 256)};
        const uint64_t strides[1] = {256};
        const uint32_t box[2] = {256, (uint32_t)(pair_bn / 128) * (IMG_BLOCK / 256)};
        st = encode_tmap(tm_ib, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, img_b, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    return st;
}

template <class CF>
int launch_pair(const Problem& pb, const Plan& pl, const DeviceInfo& dev, void* ws, cudaStream_t stream)
{
    static bool attr_done[64] = {false};
    static std::mutex mu;
    auto kernel = mxf4_gemm_pair_kernel<CF>;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!attr_done[dev.device])
        {
            cudaError_t e =
                cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, CF::SMEM_BYTES);
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute (pair)");
            attr_done[dev.device] = true;
        }
    }
    const size_t ia = pair_image_a_bytes(pb.M, pb.K);
    const size_t ib = (size_t)pl.pair_img_b_blocks * pl.k_stages * IMG_BLOCK;
    uint8_t* img_a = static_cast<uint8_t*>(ws) + kFlagBytes;
    uint8_t* img_b = img_a + ia;
    CUtensorMap tm_a, tm_b, tm_b2, tm_ia, tm_ib;
    int st = make_maps_pair(pb, CF::BN, img_a, ia, img_b, ib, &tm_a, &tm_b, &tm_b2, &tm_ia, &tm_ib);
    if (st) return st;
    // 1) scale images
    {
        const int a_blocks = (int)(ia / ((size_t)pl.k_stages * IMG_BLOCK));
        const int b_blocks = (int)(ib / ((size_t)pl.k_stages * IMG_BLOCK));
        const long long threads = (long long)(a_blocks + b_blocks) * pl.k_stages * 16;
        long long blocks = (threads + 255) / 256;
        if (blocks > (long long)dev.num_sms * 8) blocks = (long long)dev.num_sms * 8;
        scale_image_kernel<<<(int)blocks, 256, 0, stream>>>(pb.AS, pb.Mpad, a_blocks, pb.BS,
                                                            round_up(pb.N, 32), b_blocks, pb.snp, pl.k_stages,
                                                            pb.macro ? 1 : 0, pb.mb_ld, img_a, img_b);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_fail(e, "scale image launch");
    }
    // 2) the GEMM on CTA pairs
    Params p{};
    p.M = pb.M;
    p.N = pb.N;
    p.K = pb.K;
    p.k_stages = pl.k_stages;
    p.a_factor = pb.AF;
    p.b_factor = pb.BF;
    set_outputs(p, pb);
    p.alpha = pb.alpha;
    p.bias = static_cast<const __nv_bfloat16*>(pb.bias);
    p.tiles_c = pl.pair_tiles_c;
    p.wide_c = pl.pair_wide_c;
    p.img_b_blocks = pl.pair_img_b_blocks;
    p.err = device_error_word(dev.device);
    if (p.err == nullptr) return fail(MBS_ERR_CUDA, "device error word unavailable");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pl.G);
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = CF::SMEM_BYTES;
    cfg.stream = stream;
    // programmatic dependent launch: the GEMM may start while the image
    // pre-pass runs (cluster shape comes from __cluster_dims__)
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pair_pdl_enabled() ? 1 : 0;
    st = record_before(stream);
    if (st) return st;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, tm_a, tm_b, tm_b2, tm_ia, tm_ib, p);
    if (e != cudaSuccess) return cuda_fail(e, "gemm launch (pair)");
    return record_after(stream);
}

template <class CF>
int launch_cfg(const Problem& pb, const Plan& pl, const DeviceInfo& dev, void* ws, cudaStream_t stream)
{
    static bool attr_done[64] = {false};
    static std::mutex mu;
    auto kernel = mxf4_gemm_kernel<CF>;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!attr_done[dev.device])
        {
            cudaError_t e =
                cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, CF::SMEM_BYTES);
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
            attr_done[dev.device] = true;
        }
    }
    CUtensorMap tm_r, tm_c, tm_rsf, tm_csf;
    int st = make_maps(pb, pl, &tm_r, &tm_c, &tm_rsf, &tm_csf, CF::R_QUANT);
    if (st) return st;
    Params p{};
    p.M = pb.M;
    p.N = pb.N;
    p.K = pb.K;
    p.tiles_r = pl.tiles_r;
    p.tiles_c = pl.tiles_c;
    p.k_stages = pl.k_stages;
    p.num_tiles = pl.tiles_r * pl.tiles_c;
    p.sk = pl.sk ? 1 : 0;
    p.sk_units = (long long)p.num_tiles * pl.k_stages;
    p.a_factor = pb.AF;
    p.b_factor = pb.BF;
    set_outputs(p, pb);
    p.alpha = pb.alpha;
    p.bias = static_cast<const __nv_bfloat16*>(pb.bias);
    if (pl.sk)
    {
        p.flags = static_cast<unsigned*>(ws);
        p.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + kFlagBytes);
    }
    p.err = device_error_word(dev.device);
    if (p.err == nullptr) return fail(MBS_ERR_CUDA, "device error word unavailable");
    p.packed_b = pb.packed ? pb.B : nullptr;
    p.act_rows = act_box_rows(pb, pl);
    p.ksplit = pl.ksplit;
    p.withhold_release = g_withhold_release;
    if (CF::XQ != in_stage_quant(pb, pl)) return fail(MBS_ERR_CUDA, "in-stage quantiser configuration mismatch");
    if (CF::R_QUANT)
    {
        // warp 2 (and 3) quantise the bf16 rows each stage brings (tm_r maps them)
        p.qmode = 3;
    }
    else if (pb.qx != nullptr)
    {
        // the GEMM writes A and its scales itself (TMA maps above point at them)
        p.qmode = pl.ksplit > 1 ? 2 : 1;
        p.qx = static_cast<const __nv_bfloat16*>(pb.qx);
        p.qx_ld = pb.qx_ld;
        p.qa = const_cast<uint8_t*>(pb.A);
        p.qsa = const_cast<uint8_t*>(pb.AS);
        p.q_snp = pb.snp;
        p.qbar = pb.qbar;
    }
    if (pl.ksplit > 1 && !CF::SPLIT_OK) return fail(MBS_ERR_CUDA, "cluster split-K planned for a configuration without it");

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pl.G);
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = CF::SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[3];
    int na = 0;
    if (pl.ksplit > 1)
    {
        // cluster split-K: the CTAs of a cluster sum their partials in each other's shared memory
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = (unsigned)pl.ksplit;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    else
    {
        // stream-K owners wait on other CTAs, and so does the fused quantiser's grid barrier
        attr[na].id = cudaLaunchAttributeCooperative;
        attr[na].val.cooperative = (pl.sk || p.qmode == 1) ? 1 : 0;
        ++na;
    }
    // may start while the previous kernel in the stream finishes (the kernel
    // waits for it before touching global memory)
    if (pdl_enabled())
    {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    st = record_before(stream);
    if (st) return st;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, tm_r, tm_c, tm_rsf, tm_csf, p);
    if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
    return record_after(stream);
}

int dispatch(const Problem& pb, const Plan& pl, const DeviceInfo& dev, void* ws, cudaStream_t s)
{
    if (pb.packed)
    {
        // bf16 activations quantised inside each stage: 8 rows by one warp, 16 by two
        if (in_stage_quant(pb, pl) == 8) return launch_cfg<Cfg<256, false, false, 5, 32, true, 8>>(pb, pl, dev, ws, s);
        if (in_stage_quant(pb, pl) == 16) return launch_cfg<Cfg<256, false, false, 5, 32, true, 16>>(pb, pl, dev, ws, s);
        if (pl.r_rows == 32) return launch_cfg<Cfg<256, false, false, 5, 32, true>>(pb, pl, dev, ws, s);
        if (pl.r_rows == 64) return launch_cfg<Cfg<256, false, false, 5, 64, true>>(pb, pl, dev, ws, s);
        return launch_cfg<Cfg<256, false, false, 4, 128, true>>(pb, pl, dev, ws, s);
    }
    if (pl.pair)
    {
        // several output copies (other GPUs' memory among them): the staged
        // epilogue, with one pipeline stage fewer to make room for its buffers
        if (pb.n_dst > 1)
            return pl.pair_bn == 384 ? launch_pair<CfgPair<4, 384, true>>(pb, pl, dev, ws, s)
                                     : launch_pair<CfgPair<5, 256, true>>(pb, pl, dev, ws, s);
        return pl.pair_bn == 384 ? launch_pair<CfgPair<5, 384>>(pb, pl, dev, ws, s)
                                 : launch_pair<CfgPair<6, 256>>(pb, pl, dev, ws, s);
    }
    if (pl.swap)
    {
        if (pl.bn == 32)
            return pb.macro ? launch_cfg<Cfg<32, true, true, 8>>(pb, pl, dev, ws, s)
                            : launch_cfg<Cfg<32, true, false, 8>>(pb, pl, dev, ws, s);
        return pb.macro ? launch_cfg<Cfg<64, true, true, 8>>(pb, pl, dev, ws, s)
                        : launch_cfg<Cfg<64, true, false, 8>>(pb, pl, dev, ws, s);
    }
    if (in_stage_quant(pb, pl) == 8) return launch_cfg<Cfg<256, false, false, 5, 32, false, 8>>(pb, pl, dev, ws, s);
    if (pl.bn == 128)
        return pb.macro ? launch_cfg<Cfg<128, false, true, 6>>(pb, pl, dev, ws, s)
                        : launch_cfg<Cfg<128, false, false, 6>>(pb, pl, dev, ws, s);
    if (pl.r_rows == 32)
        return pb.macro ? launch_cfg<Cfg<256, false, true, 5, 32>>(pb, pl, dev, ws, s)
                        : launch_cfg<Cfg<256, false, false, 5, 32>>(pb, pl, dev, ws, s);
    if (pl.r_rows == 64)
        return pb.macro ? launch_cfg<Cfg<256, false, true, 4, 64>>(pb, pl, dev, ws, s)
                        : launch_cfg<Cfg<256, false, false, 4, 64>>(pb, pl, dev, ws, s);
    return pb.macro ? launch_cfg<Cfg<256, false, true, 4>>(pb, pl, dev, ws, s)
                    : launch_cfg<Cfg<256, false, false, 4>>(pb, pl, dev, ws, s);
}

// Library-owned stream-K scratch, one zero-filled buffer per (device, stream).
void* internal_workspace(int device, cudaStream_t stream, size_t bytes, int* status)
{
    struct Buf
    {
        void* ptr;
        size_t bytes;
        unsigned long long epoch;  // device_error_epoch() when the flags were last known zero
    };
    static std::mutex mu;
    static std::unordered_map<unsigned long long, Buf> bufs;
    std::lock_guard<std::mutex> lk(mu);
    const unsigned long long key = (reinterpret_cast<uintptr_t>(stream) << 8) ^ (unsigned)device;
    Buf& b = bufs[key];
    cudaError_t e;
    if (b.bytes >= bytes && b.ptr != nullptr)
    {
        const unsigned long long ep = device_error_epoch();
        if (b.epoch != ep)
        {
            // a launch may have stopped on a device error since: clear its flags
            e = cudaMemsetAsync(b.ptr, 0, kFlagBytes, stream);
            if (e != cudaSuccess)
            {
                *status = cuda_fail(e, "cudaMemsetAsync (gemm workspace flags)");
                return nullptr;
            }
            b.epoch = ep;
        }
        return b.ptr;
    }
    if (b.ptr != nullptr)
    {
        e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess)
        {
            *status = cuda_fail(e, "cudaStreamSynchronize (workspace growth)");
            return nullptr;
        }
        cudaFree(b.ptr);
        b.ptr = nullptr;
        b.bytes = 0;
    }
    const size_t want = bytes < (size_t)4 << 20 ? (size_t)4 << 20 : bytes;
    e = cudaMalloc(&b.ptr, want);
    if (e != cudaSuccess)
    {
        b.ptr = nullptr;
        *status = cuda_fail(e, "cudaMalloc (gemm workspace)");
        return nullptr;
    }
    e = cudaMemsetAsync(b.ptr, 0, want, stream);
    if (e != cudaSuccess)
    {
        *status = cuda_fail(e, "cudaMemsetAsync (gemm workspace)");
        return nullptr;
    }
    b.bytes = want;
    b.epoch = device_error_epoch();
    return b.ptr;
}

int run(const Problem& pb, void* ws, size_t ws_bytes, bool internal_ws, cudaStream_t stream)
{
    int st = validate(pb);
    if (st) return st;
    DeviceInfo dev;
    st = current_device(&dev);
    if (st) return st;
    const Plan pl = make_plan(pb.M, pb.N, pb.K, dev.num_sms, pb.packed);
    if (pl.ws_bytes > 0)
    {
        if (internal_ws)
        {
            ws = internal_workspace(dev.device, stream, pl.ws_bytes, &st);
            if (ws == nullptr) return st;
        }
        else
        {
            if (ws == nullptr || ws_bytes < pl.ws_bytes)
                return fail(MBS_ERR_WORKSPACE, "gemm_a4w4: workspace of %zu bytes needed, %zu given",
                            pl.ws_bytes, ws == nullptr ? (size_t)0 : ws_bytes);
            if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0)
                return fail(MBS_ERR_MISALIGNED, "gemm_a4w4: workspace must be 256-byte aligned");
        }
    }
    return dispatch(pb, pl, dev, ws, stream);
}

}  // namespace
}  // namespace gemm
}  // namespace mbs

using mbs::gemm::Problem;

#if MBS_TIMING
// Debug builds only: per-role cycle buckets summed over all CTAs (see above).
#if MBS_TIMING
// Timing builds only: per-CTA stamps of the last single-CTA GEMM launch (5 words per CTA).
extern "C" int mbs_timing_cta_read(unsigned long long* host, int ctas)
{
    if (ctas <= 0 || ctas > 1024) return MBS_ERR_INVALID_ARGUMENT;
    return cudaMemcpyFromSymbol(host, mbs::gemm::g_mbs_cta, (size_t)ctas * 5 * sizeof(unsigned long long)) ==
                   cudaSuccess
               ? MBS_OK
               : MBS_ERR_CUDA;
}
#endif

extern "C" int mbs_timing_read(unsigned long long* host, int reset)
{
    cudaError_t e = cudaMemcpyFromSymbol(host, mbs::gemm::g_mbs_timing, 16 * sizeof(unsigned long long));
    if (e == cudaSuccess && reset)
    {
        unsigned long long z[16] = {0};
        e = cudaMemcpyToSymbol(mbs::gemm::g_mbs_timing, z, sizeof(z));
    }
    return e == cudaSuccess ? MBS_OK : MBS_ERR_CUDA;
}
#endif

extern "C" int mbs_set_grid_limit(int max_ctas)
{
    mbs::clear_error();
    if (max_ctas < 0) return mbs::fail(MBS_ERR_INVALID_ARGUMENT, "mbs_set_grid_limit: max_ctas < 0");
    mbs::gemm::g_grid_limit = max_ctas;
    return MBS_OK;
}

extern "C" int mbs_set_plan_override(const mbs_plan_override* ov)
{
    mbs::clear_error();
    if (ov == nullptr)
    {
        mbs::gemm::g_ov = mbs::gemm::kAutoOverride;
        return MBS_OK;
    }
    const bool ok = (ov->schedule >= 0 && ov->schedule <= 2) && ov->grid >= 0 &&
                    (ov->pair >= -1 && ov->pair <= 1) && (ov->swap == -1 || ov->swap == 0 || ov->swap == 1) &&
                    (ov->pair_bn == 0 || ov->pair_bn == 256 || ov->pair_bn == 384) && ov->pair_wide >= 0 &&
                    (ov->ksplit == -1 || ov->ksplit == 0 || ov->ksplit == 2 || ov->ksplit == 4 || ov->ksplit == 8) &&
                    (ov->split_bn == 0 || ov->split_bn == 128 || ov->split_bn == 256);
    if (!ok)
        return mbs::fail(MBS_ERR_INVALID_ARGUMENT,
                         "mbs_set_plan_override: schedule %d grid %d pair %d swap %d pair_bn %d pair_wide %d "
                         "ksplit %d split_bn %d outside the allowed values",
                         ov->schedule, ov->grid, ov->pair, ov->swap, ov->pair_bn, ov->pair_wide, ov->ksplit,
                         ov->split_bn);
    mbs::gemm::g_ov = *ov;
    return MBS_OK;
}

extern "C" int mbs_set_withhold_release(int on)
{
    mbs::clear_error();
    mbs::gemm::g_withhold_release = on != 0 ? 1 : 0;
    return MBS_OK;
}

extern "C" int mbs_set_profile_events(void* before_main, void* after_main)
{
    mbs::clear_error();
    mbs::gemm::g_ev_before = static_cast<cudaEvent_t>(before_main);
    mbs::gemm::g_ev_after = static_cast<cudaEvent_t>(after_main);
    return MBS_OK;
}

extern "C" int gemm_a4w4_mxfp4_launch(const uint8_t* A, const uint8_t* B, const uint8_t* AScale,
                                      const uint8_t* BScale, const uint8_t* AFactor,
                                      const uint8_t* BFactor, void* out, int M, int N, int K, int Mpad,
                                      int scaleN_pad, void* stream)
{
    mbs::clear_error();
    Problem pb{A, B, AScale, BScale, AFactor, BFactor, out, M, N, K, Mpad, scaleN_pad, 0, false};
    return mbs::gemm::run(pb, nullptr, 0, true, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" size_t mbs_gemm_a4w4_workspace_size(int M, int N, int K)
{
    int num_sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess)
    {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0)
            num_sms = n;
    }
    else
    {
        cudaGetLastError();
    }
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    return mbs::gemm::make_plan(M, N, K, num_sms).ws_bytes;
}

extern "C" int mbs_gemm_a4w4_kernels_per_call(int M, int N, int K)
{
    if (M <= 0 || N <= 0 || K <= 0) return -1;
    int num_sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess)
    {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0)
            num_sms = n;
    }
    else
    {
        cudaGetLastError();
    }
    return mbs::gemm::make_plan(M, N, K, num_sms).pair ? 2 : 1;
}

extern "C" int mbs_gemm_a4w4_launch_ws(const uint8_t* A, const uint8_t* B, const uint8_t* AScale,
                                       const uint8_t* BScale, const uint8_t* AFactor,
                                       const uint8_t* BFactor, void* out, int M, int N, int K,
                                       int Mpad, int scaleN_pad, void* workspace,
                                       size_t workspace_bytes, void* stream)
{
    mbs::clear_error();
    Problem pb{A, B, AScale, BScale, AFactor, BFactor, out, M, N, K, Mpad, scaleN_pad, 0, false};
    return mbs::gemm::run(pb, workspace, workspace_bytes, false, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int mbs_gemm_a4w4_launch_ex(const uint8_t* A, const uint8_t* B, const uint8_t* AScale,
                                       const uint8_t* BScale, const uint8_t* AFactor,
                                       const uint8_t* BFactor, void* out, int M, int N, int K,
                                       int Mpad, int scaleN_pad, float alpha, const void* bias,
                                       void* workspace, size_t workspace_bytes, void* stream)
{
    mbs::clear_error();
    Problem pb{A, B, AScale, BScale, AFactor, BFactor, out, M, N, K, Mpad, scaleN_pad, 0, false};
    pb.alpha = alpha;
    pb.bias = bias;
    return mbs::gemm::run(pb, workspace, workspace_bytes, workspace == nullptr,
                          reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int mbs_gemm_a4w4_launch_multi(const uint8_t* A, const uint8_t* B, const uint8_t* AScale,
                                          const uint8_t* BScale, const uint8_t* AFactor,
                                          const uint8_t* BFactor, void* const* out_dst, int n_dst,
                                          long long ldc, int M, int N, int K, int Mpad, int scaleN_pad,
                                          float alpha, const void* bias, void* workspace,
                                          size_t workspace_bytes, void* stream)
{
    mbs::clear_error();
    if (out_dst == nullptr || n_dst < 1)
        return mbs::fail(MBS_ERR_INVALID_ARGUMENT, "mbs_gemm_a4w4_launch_multi: no output copies");
    Problem pb{A, B, AScale, BScale, AFactor, BFactor, out_dst[0], M, N, K, Mpad, scaleN_pad, 0, false};
    pb.alpha = alpha;
    pb.bias = bias;
    pb.out_dst = out_dst;
    pb.n_dst = n_dst;
    pb.ldc = ldc;
    return mbs::gemm::run(pb, workspace, workspace_bytes, workspace == nullptr,
                          reinterpret_cast<cudaStream_t>(stream));
}

namespace mbs {
namespace gemm {
namespace {

// Workspace of mbs_quant_gemm_a4w4_launch: [the GEMM's own workspace (at
// least the flag words, whose last two are the quantiser's grid barrier)]
// [quantised A: M x K/2][its flatS scales: Mpad x scaleN_pad], each part
// 256-byte aligned.
struct QuantLayout
{
    size_t gemm, a, s, total;
};

QuantLayout quant_layout(const Plan& pl, int M, int K)
{
    auto up = [](size_t x) { return (x + 255) / 256 * 256; };
    QuantLayout q;
    q.gemm = up(pl.ws_bytes > kFlagBytes ? pl.ws_bytes : kFlagBytes);
    q.a = q.gemm;
    q.s = q.a + up((size_t)M * (K / 2));
    q.total = q.s + up((size_t)round_up(M, 32) * scale_n_pad(K));
    return q;
}

int num_sms_or_default()
{
    int num_sms = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess)
    {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0) num_sms = n;
    }
    else
    {
        cudaGetLastError();
    }
    return num_sms;
}

}  // namespace
}  // namespace gemm
}  // namespace mbs

extern "C" size_t mbs_quant_gemm_a4w4_workspace_size(int M, int N, int K)
{
    using namespace mbs::gemm;
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    return quant_layout(make_plan(M, N, K, num_sms_or_default()), M, K).total;
}

extern "C" int mbs_quant_gemm_a4w4_launch(const void* x_bf16, int ld_x, const uint8_t* B, const uint8_t* BScale,
                                          const uint8_t* AFactor, const uint8_t* BFactor, void* out, int M, int N,
                                          int K, int scaleN_pad, void* workspace, size_t workspace_bytes,
                                          void* stream)
{
    using namespace mbs::gemm;
    mbs::clear_error();
    if (x_bf16 == nullptr || workspace == nullptr)
        return mbs::fail(MBS_ERR_INVALID_ARGUMENT, "mbs_quant_gemm_a4w4_launch: x and workspace must be non-NULL");
    if (M <= 0 || K <= 0 || ld_x < K || ld_x % 8 != 0 || !mbs::aligned16(x_bf16))
        return mbs::fail(MBS_ERR_INVALID_ARGUMENT,
                         "mbs_quant_gemm_a4w4_launch: x must be 16-byte aligned bf16 [M, ld_x], ld_x >= K, "
                         "ld_x %% 8 == 0 (M=%d K=%d ld_x=%d)", M, K, ld_x);
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
        return mbs::fail(MBS_ERR_MISALIGNED, "mbs_quant_gemm_a4w4_launch: workspace must be 256-byte aligned");
    mbs::DeviceInfo dev;
    int st = mbs::current_device(&dev);
    if (st) return st;
    const Plan pl = make_plan(M, N, K, dev.num_sms);
    const QuantLayout q = quant_layout(pl, M, K);
    if (workspace_bytes < q.total)
        return mbs::fail(MBS_ERR_WORKSPACE, "mbs_quant_gemm_a4w4_launch: workspace of %zu bytes needed, %zu given",
                         q.total, workspace_bytes);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    uint8_t* qa = ws + q.a;
    uint8_t* qs = ws + q.s;
    Problem pb{qa, B, qs, BScale, AFactor, BFactor, out, M, N, K, mbs::round_up(M, 32), scaleN_pad, 0, false};
    st = validate(pb);
    if (st) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (pl.pair || pl.swap)
    {
        // CTA pairs (large M: the quantiser is a small share of the call) and the
        // swapped form take A from the stand-alone quantiser, on the same stream
        st = mbs_quantize_mxfp4(x_bf16, M, K, ld_x, qa, qs, 1, stream);
        if (st) return st;
        mbs::clear_error();
        return dispatch(pb, pl, dev, ws, s);
    }
    pb.qx = x_bf16;
    pb.qx_ld = ld_x;
    pb.qbar = reinterpret_cast<unsigned*>(ws) + kQuantBarrierWord;
    return dispatch(pb, pl, dev, ws, s);
}

extern "C" size_t mbs_packed_weight_bytes(int N, int K)
{
    if (N <= 0 || K <= 0) return 0;
    return (size_t)((N + 255) / 256) * ((K + mbs::gemm::BK - 1) / mbs::gemm::BK) * mbs::gemm::PACK_STAGE_BYTES;
}

extern "C" int mbs_pack_weight(const uint8_t* B, const uint8_t* BScale, int N, int K, int scaleN_pad,
                               uint8_t* packed, void* stream)
{
    using namespace mbs::gemm;
    mbs::clear_error();
    if (!B || !BScale || !packed) return mbs::fail(MBS_ERR_INVALID_ARGUMENT, "mbs_pack_weight: null pointer");
    if (N <= 0 || K <= 0) return mbs::fail(MBS_ERR_INVALID_ARGUMENT, "mbs_pack_weight: N, K must be positive");
    if (N % 16 != 0 || K % 64 != 0)
        return mbs::fail(MBS_ERR_UNSUPPORTED_SHAPE, "mbs_pack_weight: needs N %% 16 == 0 and K %% 64 == 0");
    if (scaleN_pad % 8 != 0 || scaleN_pad < K / 32)
        return mbs::fail(MBS_ERR_INVALID_ARGUMENT, "mbs_pack_weight: bad scaleN_pad %d", scaleN_pad);
    if (!mbs::aligned16(B) || !mbs::aligned16(packed))
        return mbs::fail(MBS_ERR_MISALIGNED, "mbs_pack_weight: B and packed must be 16-byte aligned");
    mbs::DeviceInfo dev;
    int st = mbs::current_device(&dev);
    if (st) return st;
    const int ks_count = (K + BK - 1) / BK;
    const long long nblocks = (long long)((N + 255) / 256) * ks_count;
    const long long work = nblocks * ((256 * BKB) / 16 + 512);
    long long blocks = (work + 255) / 256;
    if (blocks > (long long)dev.num_sms * 16) blocks = (long long)dev.num_sms * 16;
    pack_weight_kernel<<<(int)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        B, BScale, N, K, scaleN_pad, ks_count, nblocks, packed);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? MBS_OK : mbs::cuda_fail(e, "pack_weight launch");
}

extern "C" size_t mbs_gemm_a4w4_packed_workspace_size(int M, int N, int K)
{
    int num_sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess)
    {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0)
            num_sms = n;
    }
    else
    {
        cudaGetLastError();
    }
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    return mbs::gemm::make_plan(M, N, K, num_sms, true).ws_bytes;
}

extern "C" int mbs_gemm_a4w4_packed_launch_ws(const uint8_t* A, const uint8_t* packedB, const uint8_t* AScale,
                                              const uint8_t* AFactor, const uint8_t* BFactor, void* out, int M,
                                              int N, int K, int Mpad, int scaleN_pad, void* workspace,
                                              size_t workspace_bytes, void* stream)
{
    mbs::clear_error();
    Problem pb{A, packedB, AScale, nullptr, AFactor, BFactor, out, M, N, K, Mpad, scaleN_pad, 0, false};
    pb.packed = true;
    return mbs::gemm::run(pb, workspace, workspace_bytes, false, reinterpret_cast<cudaStream_t>(stream));
}

// Workspace of mbs_quant_gemm_a4w4_packed_launch: the packed GEMM's own
// workspace followed by room for the quantised A and its scales (used when
// the rows exceed the in-stage quantiser), as for mbs_quant_gemm_a4w4_launch.
extern "C" size_t mbs_quant_gemm_a4w4_packed_workspace_size(int M, int N, int K)
{
    using namespace mbs::gemm;
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    return quant_layout(make_plan(M, N, K, num_sms_or_default(), true), M, K).total;
}

extern "C" int mbs_quant_gemm_a4w4_packed_launch(const void* x_bf16, int ld_x, const uint8_t* packedB,
                                                 const uint8_t* AFactor, const uint8_t* BFactor, void* out,
                                                 int M, int N, int K, void* workspace, size_t workspace_bytes,
                                                 void* stream)
{
    using namespace mbs::gemm;
    mbs::clear_error();
    if (x_bf16 == nullptr || workspace == nullptr)
        return mbs::fail(MBS_ERR_INVALID_ARGUMENT,
                         "mbs_quant_gemm_a4w4_packed_launch: x and workspace must be non-NULL");
    if (M <= 0 || K <= 0 || ld_x < K || ld_x % 8 != 0 || !mbs::aligned16(x_bf16))
        return mbs::fail(MBS_ERR_INVALID_ARGUMENT,
                         "mbs_quant_gemm_a4w4_packed_launch: x must be 16-byte aligned bf16 [M, ld_x], "
                         "ld_x >= K, ld_x %% 8 == 0 (M=%d K=%d ld_x=%d)", M, K, ld_x);
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
        return mbs::fail(MBS_ERR_MISALIGNED, "mbs_quant_gemm_a4w4_packed_launch: workspace must be 256-byte aligned");
    mbs::DeviceInfo dev;
    int st = mbs::current_device(&dev);
    if (st) return st;
    const Plan pl = make_plan(M, N, K, dev.num_sms, true);
    const QuantLayout q = quant_layout(pl, M, K);
    if (workspace_bytes < q.total)
        return mbs::fail(MBS_ERR_WORKSPACE,
                         "mbs_quant_gemm_a4w4_packed_launch: workspace of %zu bytes needed, %zu given", q.total,
                         workspace_bytes);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    uint8_t* qa = ws + q.a;
    uint8_t* qs = ws + q.s;
    Problem pb{qa, packedB, qs, nullptr, AFactor, BFactor, out, M, N, K, mbs::round_up(M, 32),
               mbs::scale_n_pad(K), 0, false};
    pb.packed = true;
    st = validate(pb);
    if (st) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    pb.qx = x_bf16;
    pb.qx_ld = ld_x;
    if (in_stage_quant(pb, pl) == 0)
    {
        // more rows than the in-stage quantiser takes: the stand-alone quantiser first
        pb.qx = nullptr;
        st = mbs_quantize_mxfp4(x_bf16, M, K, ld_x, qa, qs, 1, stream);
        if (st) return st;
        mbs::clear_error();
    }
    return dispatch(pb, pl, dev, ws, s);
}

extern "C" int mbs_gemm_a4w4_macro_launch_ws(const uint8_t* A, const uint8_t* B,
                                             const uint8_t* AScale, const uint8_t* BScaleMacro,
                                             const uint8_t* AFactor, const uint8_t* BFactor, void* out,
                                             int M, int N, int K, int Mpad, int scaleN_pad, int mb_ld,
                                             void* workspace, size_t workspace_bytes, void* stream)
{
    mbs::clear_error();
    Problem pb{A, B, AScale, BScaleMacro, AFactor, BFactor, out, M, N, K, Mpad, scaleN_pad, mb_ld, true};
    return mbs::gemm::run(pb, workspace, workspace_bytes, false, reinterpret_cast<cudaStream_t>(stream));
}

// ===================================================== allocation-free entry
// Some callers cannot allocate device memory: a plugin running inside a host
// framework that owns every device allocation (and its memory budget), or a
// latency-critical loop where a cudaMalloc (which can synchronise the device)
// is not allowed.  mbs_gemm_a4w4_launch_noalloc serves them with scratch that
// lives in the library image itself: a fixed-size __device__ array that every
// GPU loading the library holds until the process exits.
namespace mbs {
namespace gemm {
namespace {

constexpr size_t kNoAllocScratchBytes = (size_t)8 << 20;  // 8 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on `device` (which must be current).
// Looked up once per device; in host code the symbol itself is only a
// host-side stand-in and must never be handed to a kernel.
void* noalloc_scratch_address(int device, int* status)
{
    static std::mutex mu;
    static void* addr[64] = {nullptr};
    std::lock_guard<std::mutex> lk(mu);
    if (device < 0 || device >= 64)
    {
        *status = fail(MBS_ERR_DEVICE, "device index %d out of range", device);
        return nullptr;
    }
    if (addr[device] == nullptr)
    {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr)
        {
            *status = cuda_fail(e, "cudaGetSymbolAddress (no-alloc scratch)");
            return nullptr;
        }
        addr[device] = p;
    }
    return addr[device];
}

}  // namespace
}  // namespace gemm
}  // namespace mbs

extern "C" int mbs_gemm_a4w4_launch_noalloc(const uint8_t* A, const uint8_t* B,
                                            const uint8_t* AScale, const uint8_t* BScale,
                                            const uint8_t* AFactor, const uint8_t* BFactor, void* out,
                                            int M, int N, int K, int Mpad, int scaleN_pad,
                                            void* stream)
{
    using namespace mbs::gemm;
    mbs::clear_error();
    Problem pb{A, B, AScale, BScale, AFactor, BFactor, out, M, N, K, Mpad, scaleN_pad, 0, false};
    int st = validate(pb);
    if (st) return st;
    mbs::DeviceInfo dev;
    st = mbs::current_device(&dev);
    if (st) return st;
    const Plan pl = make_plan(M, N, K, dev.num_sms);
    if (pl.ws_bytes > kNoAllocScratchBytes)
        return mbs::fail(MBS_ERR_WORKSPACE,
                         "mbs_gemm_a4w4_launch_noalloc: this shape needs %zu bytes of scratch, more "
                         "than the %zu-byte static buffer; use mbs_gemm_a4w4_launch_ws",
                         pl.ws_bytes, kNoAllocScratchBytes);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    void* ws = nullptr;
    if (pl.ws_bytes > 0)
    {
        ws = noalloc_scratch_address(dev.device, &st);
        if (ws == nullptr) return st;
    }
    if (pl.sk)
    {
        // The stream-K flags must start at zero.  A completed launch leaves
        // them zero, but one that stopped early may not have, so clear them.
        cudaError_t e = cudaMemsetAsync(ws, 0, (size_t)pl.G * sizeof(unsigned), s);
        if (e != cudaSuccess) return mbs::cuda_fail(e, "cudaMemsetAsync (no-alloc flags)");
    }
    return dispatch(pb, pl, dev, ws, s);
}

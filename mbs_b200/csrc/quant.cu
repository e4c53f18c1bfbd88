// bf16 -> MXFP4 quantisers and the two layout kernels (weight preshuffle,
// scale shuffle).  All are HBM-bound byte work: 16-byte vector loads/stores,
// integer arithmetic for the scale, warp shuffles for the block amax, and the
// hardware e2m1 conversion for the codes (a bit-level software encoding cost
// ~20 instructions per element and made the quantiser issue-bound).
//
// Quantiser arithmetic (OCP MX per-1x32, the task's spec for aiter's
// per_1x32 quantiser called at test_gemm_a4w4.py:134-140):
//   amax   = max |x| over the 32-element block, taken on the bf16 bit
//            patterns (|x| bits = bits & 0x7FFF order like the magnitudes)
//   scale  = e8m0 byte max(E(amax) - 2, 0)   (E = biased exponent field;
//            i.e. 2^(floor(log2 amax) - 2)), 0xFF if the block holds Inf/NaN
//   code   = RNE(|x| * 2^(127 - scale)) on {0,.5,1,1.5,2,3,4,6}, saturating,
//            sign bit 3 copied from x; packed two per byte, low nibble first.
#include <cuda_bf16.h>

#include "common.h"
#include "mx_quant.cuh"

namespace mbs {
namespace {

using mx::amax_bits8;
using mx::cvt_e2m1x8;
using mx::encode8;
using mx::scale_from_amax_bits;

// As encode8 for MBS rows: the values are (x * m) * inv, both products exact
// (m = 1 + b/256 has 9 significant bits; inv is a power of two; m * inv alone
// could overflow when the block scale is 0).
__device__ __forceinline__ uint32_t encode8_mbs(const uint32_t (&w)[4], float m, float inv, bool nan_block)
{
    float f[8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        f[2 * i] = (__uint_as_float(w[i] << 16) * m) * inv;
        f[2 * i + 1] = (__uint_as_float(w[i] & 0xFFFF0000u) * m) * inv;
    }
    const uint32_t packed = cvt_e2m1x8(f);
    return nan_block ? 0u : packed;
}

// MBS factor byte of a row whose max |x| has bf16 bit pattern `amax_bits`:
// the top 8 mantissa bits of 6.0 / max (IEEE division, bits truncated;
// docs/kernel_advanced.md:122-125 of the reference); 0 for a zero, Inf or
// NaN max, and for a max so close to the top of the fp32 range that max * m
// would overflow (finite rows never become Inf blocks).  The row is then
// scaled by m = 1 + b/256, undone by the GEMM's factor 1/m.
__device__ __forceinline__ uint32_t mbs_factor_byte(uint32_t amax_bits)
{
    if (amax_bits == 0u || amax_bits >= 0x7F80u) return 0u;
    const float amax = __uint_as_float(amax_bits << 16);
    const float sc = __fdiv_rn(6.0f, amax);
    const uint32_t b = (__float_as_uint(sc) >> 15) & 0xFFu;
    const float scaled = amax * __uint_as_float(0x3F800000u | (b << 15));
    return (__float_as_uint(scaled) & 0x7F800000u) == 0x7F800000u ? 0u : b;
}

__device__ __forceinline__ int64_t flat_s(int r, int b, int snp)
{
    const int r32 = r & 31, b8 = b & 7;
    return (int64_t)(r32 >> 4) + (int64_t)(b8 >> 2) * 2 + (int64_t)(r32 & 15) * 4 +
           (int64_t)(b8 & 3) * 64 + (int64_t)(b >> 3) * 256 + (int64_t)(r >> 5) * 32 * snp;
}

// One CTA per row, one thread per 8 consecutive elements (16 bytes of bf16)
// of that row; the 4 threads of a 32-element block are 4 consecutive lanes
// and combine their amax with two xor-shuffles.  Each thread keeps
// QUANT_UNROLL independent 16-byte loads in flight before using them, and no
// index needs a division.  Lanes past the row end run the shuffles with an
// empty block.
// Both variants: 128-thread CTAs with 8 loads in flight per thread (a K =
// 8192 row in one pass) and a register budget for 8 CTAs per SM, so the rows
// in flight per SM (and for the MBS variant, which waits for a CTA-wide row
// max, most of all) are 8.  Against 256 threads x 4 loads at 6 CTAs per SM
// this took 16384x8192 from 54.5 to 53.0 us (16384x4096 33.0 -> 30.0) and
// the MBS variant from 65.5 to 60.4 us.
constexpr int QUANT_UNROLL = 8;
constexpr int QUANT_THREADS = 128;
constexpr int QUANT_MIN_CTAS = 8;
constexpr int QMBS_THREADS = 128;
constexpr int QMBS_UNROLL = 8;
constexpr int QMBS_MIN_CTAS = 8;

// MBS = true: each row is first reduced to its max |x| (one read of the row,
// kept in L2 for the second), its factor byte b is written to `factors`, and
// the row is quantised as x * (1 + b/256).
// Codes and scales of one group of UNROLL octets per thread (octet j =
// j0 + u * NT of row r), the row already multiplied by m when MBS.
template <bool MBS, int NT, int UNROLL>
__device__ __forceinline__ void quantize_group(const uint4 (&v)[UNROLL], int j0, int oct, int limit,
                                               float m, int r, int K, uint32_t* __restrict__ qr,
                                               uint8_t* __restrict__ sc, int shuffled, int snp)
{
#pragma unroll
    for (int u = 0; u < UNROLL; ++u)
    {
        const int j = j0 + u * NT;
        if (j - (int)(threadIdx.x & 31) >= limit) break;  // whole warp past the row end
        const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
        uint32_t am = amax_bits8(w);
        am = max(am, __shfl_xor_sync(0xffffffffu, am, 1));
        am = max(am, __shfl_xor_sync(0xffffffffu, am, 2));
        if (j >= oct) continue;
        uint32_t s;
        if constexpr (MBS)
        {
            // block amax of x * m is m * amax (exact): scale from its fp32 exponent
            const uint32_t e = (__float_as_uint(__uint_as_float(am << 16) * m) >> 23) & 0xFFu;
            s = am >= 0x7F80u ? 0xFFu : (e > 2u ? e - 2u : 0u);
        }
        else
        {
            s = scale_from_amax_bits(am);
        }
        const bool nan_block = s == 0xFFu;
        const float inv = __uint_as_float((254u - (nan_block ? 254u : s)) << 23);
        qr[j] = MBS ? encode8_mbs(w, m, inv, nan_block) : encode8(w, inv, nan_block);
        if ((j & 3) == 0)
        {
            const int b = j >> 2;
            if (shuffled)
                sc[flat_s(r, b, snp)] = (uint8_t)s;
            else
                sc[(int64_t)r * (K >> 5) + b] = (uint8_t)s;
        }
    }
}

template <int NT, int UNROLL>
__device__ __forceinline__ void load_group(const uint4* __restrict__ xr, int j0, int oct, uint4 (&v)[UNROLL],
                                           bool last_use)
{
#pragma unroll
    for (int u = 0; u < UNROLL; ++u)
    {
        const int j = j0 + u * NT;
        v[u] = j < oct ? (last_use ? __ldcs(xr + j) : __ldcg(xr + j)) : make_uint4(0, 0, 0, 0);
    }
}

// MBS row factor: CTA-wide max of the threads' `am`, factor byte to
// factors[r], returns the row multiplier m = 1 + b/256.
template <int NT>
__device__ __forceinline__ float mbs_row_multiplier(uint32_t am, int r, uint8_t* __restrict__ factors,
                                                    uint32_t* red)
{
    am = __reduce_max_sync(0xffffffffu, am);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = am;
    __syncthreads();
    if (threadIdx.x < 32)
    {
        uint32_t a = threadIdx.x < NT / 32 ? red[threadIdx.x] : 0u;
        a = __reduce_max_sync(0xffffffffu, a);
        if (threadIdx.x == 0)
        {
            const uint32_t b = mbs_factor_byte(a);
            factors[r] = (uint8_t)b;
            red[0] = b;
        }
    }
    __syncthreads();
    const float m = __uint_as_float(0x3F800000u | (red[0] << 15));
    __syncthreads();  // red is rewritten by the next row
    return m;
}

// MBS = true: each row is first reduced to its max |x|, its factor byte b is
// written to `factors`, and the row is quantised as x * (1 + b/256).  A row
// of up to NT * UNROLL octets (K <= 8192) stays in registers between the two
// steps; longer rows are read twice (the second read from L2).
template <bool MBS, int NT, int UNROLL, int MIN_CTAS>
__global__ void __launch_bounds__(NT, MIN_CTAS) quantize_1x32_kernel(const uint16_t* __restrict__ x,
                                                                      int rows, int K, int ld_x,
                                                                      uint8_t* __restrict__ q,
                                                                      uint8_t* __restrict__ sc, int shuffled,
                                                                      int snp, uint8_t* __restrict__ factors)
{
    __shared__ uint32_t red[NT / 32];
    const int oct = K >> 3;                 // octets in a row (multiple of 4)
    const int limit = (oct + 31) & ~31;     // whole warps
    const bool one_pass = oct <= NT * UNROLL;
    for (int r = blockIdx.x; r < rows; r += gridDim.x)
    {
        const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)r * ld_x);
        uint32_t* qr = reinterpret_cast<uint32_t*>(q + (int64_t)r * (K >> 1));
        if (MBS && one_pass)
        {
            uint4 v[UNROLL];
            load_group<NT, UNROLL>(xr, threadIdx.x, oct, v, true);
            uint32_t am = 0;
#pragma unroll
            for (int u = 0; u < UNROLL; ++u)
            {
                const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
                am = max(am, amax_bits8(w));
            }
            const float m = mbs_row_multiplier<NT>(am, r, factors, red);
            quantize_group<MBS, NT, UNROLL>(v, threadIdx.x, oct, limit, m, r, K, qr, sc, shuffled, snp);
            continue;
        }
        float m = 1.0f;
        if constexpr (MBS)
        {
            uint32_t am = 0;
            for (int j0 = threadIdx.x; j0 < oct; j0 += NT * UNROLL)
            {
                uint4 v[UNROLL];
                load_group<NT, UNROLL>(xr, j0, oct, v, false);
#pragma unroll
                for (int u = 0; u < UNROLL; ++u)
                {
                    const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
                    am = max(am, amax_bits8(w));
                }
            }
            m = mbs_row_multiplier<NT>(am, r, factors, red);
        }
        for (int j0 = threadIdx.x; j0 < limit; j0 += NT * UNROLL)
        {
            uint4 v[UNROLL];
            load_group<NT, UNROLL>(xr, j0, oct, v, true);
            quantize_group<MBS, NT, UNROLL>(v, j0, oct, limit, m, r, K, qr, sc, shuffled, snp);
        }
    }
}

// Writes 127 into the padding of a flatS buffer (rows >= rows, blocks >= K/32).
__global__ void scale_padding_kernel(uint8_t* __restrict__ sc, int rows, int nblk, int rpad,
                                     int snp)
{
    const int64_t total = (int64_t)rpad * snp;
    for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total;
         o += (int64_t)gridDim.x * blockDim.x)
    {
        const int rg = (int)(o / (32 * snp));
        const int og = (int)(o - (int64_t)rg * 32 * snp);
        const int w = og & 255;
        const int r = rg * 32 + (w & 1) * 16 + ((w & 63) >> 2);
        const int b = (og >> 8) * 8 + ((w & 3) >> 1) * 4 + (w >> 6);
        if (r >= rows || b >= nblk) sc[o] = 127;
    }
}

// One warp per 32-row x 32-K macro block: lane l owns row l of the block.
__global__ void __launch_bounds__(256) quantize_macro_kernel(const uint16_t* __restrict__ x,
                                                             int rows, int K, int ld_x,
                                                             uint8_t* __restrict__ q,
                                                             uint8_t* __restrict__ sc, int mb_ld)
{
    const int lane = threadIdx.x & 31;
    const int warps_per_block = blockDim.x >> 5;
    const int nb = (rows + 31) >> 5;
    const int64_t total = (int64_t)nb * mb_ld;
    for (int64_t wid = (int64_t)blockIdx.x * warps_per_block + (threadIdx.x >> 5); wid < total;
         wid += (int64_t)gridDim.x * warps_per_block)
    {
        const int rb = (int)(wid / mb_ld);
        const int kb = (int)(wid - (int64_t)rb * mb_ld);
        if (kb >= (K >> 5))
        {
            if (lane == 0) sc[(int64_t)rb * mb_ld + kb] = 127;
            continue;
        }
        const int r = rb * 32 + lane;
        uint32_t w[16];
        if (r < rows)
        {
            const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)r * ld_x + kb * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i)
            {
                const uint4 v = __ldcs(src + i);
                w[4 * i + 0] = v.x;
                w[4 * i + 1] = v.y;
                w[4 * i + 2] = v.z;
                w[4 * i + 3] = v.w;
            }
        }
        else
        {
#pragma unroll
            for (int i = 0; i < 16; ++i) w[i] = 0;
        }
        uint32_t am = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i)
        {
            const uint32_t wi[4] = {w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]};
            am = max(am, amax_bits8(wi));
        }
#pragma unroll
        for (int m = 1; m < 32; m <<= 1) am = max(am, __shfl_xor_sync(0xffffffffu, am, m));
        const uint32_t s = scale_from_amax_bits(am);
        const bool nan_block = s == 0xFFu;
        const float inv = __uint_as_float((254u - (nan_block ? 254u : s)) << 23);
        if (r < rows)
        {
            uint32_t out[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
            {
                const uint32_t wi[4] = {w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]};
                out[i] = encode8(wi, inv, nan_block);
            }
            *reinterpret_cast<uint4*>(q + (int64_t)r * (K >> 1) + kb * 16) =
                make_uint4(out[0], out[1], out[2], out[3]);
        }
        if (lane == 0) sc[(int64_t)rb * mb_ld + kb] = (uint8_t)s;
    }
}

// flatB preshuffle: the 16 bytes (n, kp..kp+15), kp % 16 == 0, are
// contiguous in both layouts.
__global__ void shuffle_weight_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                      int N, int K)
{
    const int chunks = K >> 5;  // 16-byte chunks per row (K/2 bytes)
    const int64_t total = (int64_t)N * chunks;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x)
    {
        const int n = (int)(t / chunks);
        const int c = (int)(t - (int64_t)n * chunks);
        const uint4 v = __ldcs(reinterpret_cast<const uint4*>(src + (int64_t)n * (K >> 1)) + c);
        const int64_t off = (int64_t)(n >> 4) * ((int64_t)K * 8) + (int64_t)c * 256 + (n & 15) * 16;
        *reinterpret_cast<uint4*>(dst + off) = v;
    }
}

// flatS shuffle, one thread per destination byte (coalesced writes), padding 127.
__global__ void shuffle_scales_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                      int rows, int nblk, int rpad, int snp)
{
    const int64_t total = (int64_t)rpad * snp;
    for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total;
         o += (int64_t)gridDim.x * blockDim.x)
    {
        const int rg = (int)(o / (32 * snp));
        const int og = (int)(o - (int64_t)rg * 32 * snp);
        const int w = og & 255;
        const int r = rg * 32 + (w & 1) * 16 + ((w & 63) >> 2);
        const int b = (og >> 8) * 8 + ((w & 3) >> 1) * 4 + (w >> 6);
        dst[o] = (r < rows && b < nblk) ? src[(int64_t)r * nblk + b] : (uint8_t)127;
    }
}

int grid_for(int64_t work, int threads, int num_sms)
{
    int64_t blocks = (work + threads - 1) / threads;
    const int64_t cap = (int64_t)num_sms * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (int)blocks;
}

}  // namespace
}  // namespace mbs

using namespace mbs;

namespace mbs {
namespace {

int quantize_1x32(const char* fn, const void* x_bf16, int rows, int K, int ld_x, uint8_t* fp4_out,
                  uint8_t* scale_out, uint8_t* factors, int shuffled, void* stream)
{
    clear_error();
    if (!x_bf16 || !fp4_out || !scale_out)
        return fail(MBS_ERR_INVALID_ARGUMENT, "%s: null pointer", fn);
    if (rows <= 0 || K <= 0) return fail(MBS_ERR_INVALID_ARGUMENT, "rows and K must be positive");
    if (K % 32 != 0) return fail(MBS_ERR_UNSUPPORTED_SHAPE, "K must be a multiple of 32, got %d", K);
    if (ld_x < K) return fail(MBS_ERR_INVALID_ARGUMENT, "ld_x (%d) < K (%d)", ld_x, K);
    if (!aligned16(x_bf16) || (ld_x % 8) != 0 || !aligned16(fp4_out) || ((K / 2) % 4) != 0)
        return fail(MBS_ERR_MISALIGNED, "x must be 16-byte aligned with ld_x %% 8 == 0");
    DeviceInfo dev;
    int st = current_device(&dev);
    if (st != MBS_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int snp = scale_n_pad(K);
    // one CTA per row (grid-stride over rows beyond the cap)
    const int qgrid = rows < dev.num_sms * 64 ? rows : dev.num_sms * 64;
    if (factors != nullptr)
        quantize_1x32_kernel<true, QMBS_THREADS, QMBS_UNROLL, QMBS_MIN_CTAS><<<qgrid, QMBS_THREADS, 0, s>>>(
            static_cast<const uint16_t*>(x_bf16), rows, K, ld_x, fp4_out, scale_out, shuffled ? 1 : 0,
            snp, factors);
    else
        quantize_1x32_kernel<false, QUANT_THREADS, QUANT_UNROLL, QUANT_MIN_CTAS><<<qgrid, QUANT_THREADS, 0, s>>>(
            static_cast<const uint16_t*>(x_bf16), rows, K, ld_x, fp4_out, scale_out, shuffled ? 1 : 0,
            snp, nullptr);
    if (shuffled && ((rows % 32) != 0 || (K / 32) != snp))
    {
        const int rpad = round_up(rows, 32);
        scale_padding_kernel<<<grid_for((int64_t)rpad * snp, 256, dev.num_sms), 256, 0, s>>>(
            scale_out, rows, K / 32, rpad, snp);
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? MBS_OK : cuda_fail(e, "quantize launch");
}

}  // namespace
}  // namespace mbs

extern "C" int mbs_quantize_mxfp4(const void* x_bf16, int rows, int K, int ld_x, uint8_t* fp4_out,
                                  uint8_t* scale_out, int shuffled, void* stream)
{
    return mbs::quantize_1x32("mbs_quantize_mxfp4", x_bf16, rows, K, ld_x, fp4_out, scale_out, nullptr,
                              shuffled, stream);
}

extern "C" int mbs_quantize_mxfp4_mbs(const void* x_bf16, int rows, int K, int ld_x, uint8_t* fp4_out,
                                      uint8_t* scale_out, uint8_t* factor_out, int shuffled, void* stream)
{
    if (factor_out == nullptr)
    {
        mbs::clear_error();
        return mbs::fail(MBS_ERR_INVALID_ARGUMENT, "mbs_quantize_mxfp4_mbs: factor_out is NULL");
    }
    return mbs::quantize_1x32("mbs_quantize_mxfp4_mbs", x_bf16, rows, K, ld_x, fp4_out, scale_out,
                              factor_out, shuffled, stream);
}

extern "C" int mbs_quantize_mxfp4_macro(const void* x_bf16, int rows, int K, int ld_x,
                                        uint8_t* fp4_out, uint8_t* scale_out, void* stream)
{
    clear_error();
    if (!x_bf16 || !fp4_out || !scale_out)
        return fail(MBS_ERR_INVALID_ARGUMENT, "mbs_quantize_mxfp4_macro: null pointer");
    if (rows <= 0 || K <= 0) return fail(MBS_ERR_INVALID_ARGUMENT, "rows and K must be positive");
    if (K % 32 != 0) return fail(MBS_ERR_UNSUPPORTED_SHAPE, "K must be a multiple of 32, got %d", K);
    if (ld_x < K) return fail(MBS_ERR_INVALID_ARGUMENT, "ld_x (%d) < K (%d)", ld_x, K);
    if (!aligned16(x_bf16) || (ld_x % 8) != 0 || !aligned16(fp4_out))
        return fail(MBS_ERR_MISALIGNED, "x must be 16-byte aligned with ld_x %% 8 == 0");
    DeviceInfo dev;
    int st = current_device(&dev);
    if (st != MBS_OK) return st;
    const int mb_ld = round_up(K / 32, 16);
    const int64_t warps = (int64_t)((rows + 31) / 32) * mb_ld;
    quantize_macro_kernel<<<grid_for(warps * 32, 256, dev.num_sms), 256, 0,
                            reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(x_bf16), rows, K, ld_x, fp4_out, scale_out, mb_ld);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? MBS_OK : cuda_fail(e, "quantize_macro launch");
}

extern "C" int mbs_shuffle_weight(const uint8_t* src, uint8_t* dst, int N, int K, void* stream)
{
    clear_error();
    if (!src || !dst) return fail(MBS_ERR_INVALID_ARGUMENT, "mbs_shuffle_weight: null pointer");
    if (N <= 0 || K <= 0) return fail(MBS_ERR_INVALID_ARGUMENT, "N and K must be positive");
    if (N % 16 != 0 || K % 64 != 0)
        return fail(MBS_ERR_UNSUPPORTED_SHAPE, "shuffle_weight needs N %% 16 == 0 and K %% 64 == 0 (N=%d K=%d)",
                    N, K);
    if (!aligned16(src) || !aligned16(dst))
        return fail(MBS_ERR_MISALIGNED, "src/dst must be 16-byte aligned");
    DeviceInfo dev;
    int st = current_device(&dev);
    if (st != MBS_OK) return st;
    shuffle_weight_kernel<<<grid_for((int64_t)N * (K / 32), 256, dev.num_sms), 256, 0,
                            reinterpret_cast<cudaStream_t>(stream)>>>(src, dst, N, K);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? MBS_OK : cuda_fail(e, "shuffle_weight launch");
}

extern "C" int mbs_shuffle_scales(const uint8_t* plain, uint8_t* shuffled, int rows, int K,
                                  void* stream)
{
    clear_error();
    if (!plain || !shuffled) return fail(MBS_ERR_INVALID_ARGUMENT, "mbs_shuffle_scales: null pointer");
    if (rows <= 0 || K <= 0) return fail(MBS_ERR_INVALID_ARGUMENT, "rows and K must be positive");
    if (K % 32 != 0) return fail(MBS_ERR_UNSUPPORTED_SHAPE, "K must be a multiple of 32, got %d", K);
    DeviceInfo dev;
    int st = current_device(&dev);
    if (st != MBS_OK) return st;
    const int snp = scale_n_pad(K);
    const int rpad = round_up(rows, 32);
    shuffle_scales_kernel<<<grid_for((int64_t)rpad * snp, 256, dev.num_sms), 256, 0,
                            reinterpret_cast<cudaStream_t>(stream)>>>(plain, shuffled, rows, K / 32,
                                                                       rpad, snp);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? MBS_OK : cuda_fail(e, "shuffle_scales launch");
}

// OCP MX per-1x32 quantiser arithmetic shared by the stand-alone quantiser
// (quant.cu) and the GEMM's fused activation quantiser (gemm.cu), so both
// produce the same bytes by construction.
//   amax   = max |x| over the 32-element block, taken on the bf16 bit
//            patterns (|x| bits = bits & 0x7FFF order like the magnitudes)
//   scale  = e8m0 byte max(E(amax) - 2, 0), 0xFF if the block holds Inf/NaN
//   code   = RNE(|x| * 2^(127 - scale)) on {0,.5,1,1.5,2,3,4,6}, saturating,
//            sign bit 3 copied from x; packed two per byte, low nibble first.
#pragma once

#include <cstdint>

namespace mbs {
namespace mx {

// Eight fp32 values -> eight e2m1 codes packed low nibble first, with the
// sm_100a conversion cvt.rn.satfinite.e2m1x2.f32: IEEE round-to-nearest-even
// onto {0,.5,1,1.5,2,3,4,6}, saturating at +-6, the sign kept (so a value
// that rounds to zero keeps its sign bit, -0 -> 0x8).  The inputs are
// x * 2^(127 - scale) for bf16 x, exact products (a power of two), so this
// is the spec's code for every finite x.  The instruction writes its first
// source to the high nibble, hence the (odd, even) operand order.
__device__ __forceinline__ uint32_t cvt_e2m1x8(const float (&f)[8])
{
    uint32_t out;
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
        "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
        : "=r"(out)
        : "f"(f[0]), "f"(f[1]), "f"(f[2]), "f"(f[3]), "f"(f[4]), "f"(f[5]), "f"(f[6]), "f"(f[7]));
    return out;
}

// max |x| bit pattern over the 8 bf16 of four 32-bit words (|x| bits =
// bits & 0x7FFF order like the magnitudes); two halfword maxes per step.
__device__ __forceinline__ uint32_t amax_bits8(const uint32_t (&w)[4])
{
    const uint32_t m = __vmaxu2(__vmaxu2(w[0] & 0x7FFF7FFFu, w[1] & 0x7FFF7FFFu),
                                __vmaxu2(w[2] & 0x7FFF7FFFu, w[3] & 0x7FFF7FFFu));
    return max(m & 0xFFFFu, m >> 16);
}

__device__ __forceinline__ uint32_t scale_from_amax_bits(uint32_t amax_bits)
{
    if (amax_bits >= 0x7F80u) return 0xFFu;  // Inf or NaN in the block
    const int e = (int)(amax_bits >> 7);      // bf16 exponent field == fp32's
    return (uint32_t)max(e - 2, 0);
}

// Encode 8 bf16 (four 32-bit words, element 0 in the low half of w[0]) with
// multiplier `inv` = 2^(127 - scale): 32 bits of packed codes.  Blocks that
// hold an Inf or NaN get all-zero codes.
__device__ __forceinline__ uint32_t encode8(const uint32_t (&w)[4], float inv, bool nan_block)
{
    float f[8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        f[2 * i] = __uint_as_float(w[i] << 16) * inv;
        f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u) * inv;
    }
    const uint32_t packed = cvt_e2m1x8(f);
    return nan_block ? 0u : packed;
}

}  // namespace mx
}  // namespace mbs

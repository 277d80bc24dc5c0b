// Per-value arithmetic of the reference's symmetric int8 quantiser, shared by
// K1 (weight preparation), K2 (activation quantisation) and the GEMM's fused
// prologue, so all produce the same bits.
//
// quantize_symmetric_into (capi/src/lib.rs:614-654, x86 scalar branch):
// scale = absmax / 127 (1.0 when the row is all zero), q = round half away
// from zero of the IEEE quotient fl(x / scale), clamped to +-127.
//
// Division-free rounding test.  With inv = RN(1 / scale) and t = RN(x * inv),
// standard error analysis of round-to-nearest binary32 (unit roundoff
// u = 2^-24) gives |t - x/scale| <= (2u + u^2) |x/scale| and
// |fl(x/scale) - x/scale| <= u |x/scale|, so t and the IEEE quotient differ
// by at most 3.000001 u |x/scale| <= 2.28e-5 for |x/scale| <= 127.0001 (every
// value of a row scaled by that row's absmax / 127).  When t is farther than
// 4e-5 from every half-integer, the quotient lies in the same interval
// between half-integers, so both round to the same integer and rint(t) is
// the answer.  Otherwise -- about 8e-5 of values, and any non-finite t --
// the exact quotient fl(x / scale) decides, as in the reference.  This is a
// rounding test in the style of Ziv's correctly-rounded evaluation: cheap
// approximation, certified error bound, exact fallback.
#pragma once

#include <cstdint>

namespace rk {

__device__ __forceinline__ float row_scale(float absmax) {
    return absmax == 0.0f ? 1.0f : __fdiv_rn(absmax, 127.0f);
}

__device__ __forceinline__ float row_inv(float scale) { return __frcp_rn(scale); }

// The reference's operation: round(fl(x / scale)), clamped.
__device__ __forceinline__ int quant_value_exact(float x, float scale) {
    float q = roundf(__fdiv_rn(x, scale));
    q = fminf(fmaxf(q, -127.0f), 127.0f);
    return static_cast<int>(q);
}

// The exact path, kept out of line: it runs for ~1e-4 of the values, and
// inlining it at every call site would bloat the unrolled quantisers' code
// (cold instruction-cache misses cost more than the arithmetic).
static __device__ __noinline__ int quant_value_slow(float x, float scale) { return quant_value_exact(x, scale); }

static __device__ __noinline__ uint32_t quant_pack4_slow(float4 v, float scale) {
    return (quant_value_exact(v.x, scale) & 0xFF) | ((quant_value_exact(v.y, scale) & 0xFF) << 8) |
           ((quant_value_exact(v.z, scale) & 0xFF) << 16) | ((quant_value_exact(v.w, scale) & 0xFF) << 24);
}

// Adding 1.5 * 2^23 to |t| < 2^22 rounds it to an integer (ties to even) in
// one FADD; the sum's low mantissa bits then hold that integer in two's
// complement, so its low byte is the int8 value without a conversion.
constexpr float kRoundMagic = 12582912.0f;

// Candidate int8 (in the low byte of the result) for t = x * inv, and whether
// the rounding test failed: |t - rint(t)| is exact (Sterbenz); NaN / inf, and
// |t| above 127.25 (outside the bound the test assumes; the exact path
// clamps), fail it too.
__device__ __forceinline__ uint32_t quant_candidate(float x, float inv, bool& doubtful) {
    const float t = __fmul_rn(x, inv);
    const float m = __fadd_rn(t, kRoundMagic);
    const float r = __fsub_rn(m, kRoundMagic);
    doubtful |= !(fabsf(__fsub_rn(t, r)) <= 0.49996f) || !(fabsf(t) <= 127.25f);
    return __float_as_uint(m);
}

// The same integer as quant_value_exact for every x of a row whose absmax
// gave `scale` (see the rounding test above); inv = row_inv(scale).
__device__ __forceinline__ int quant_value(float x, float scale, float inv) {
    bool doubtful = false;
    const uint32_t q = quant_candidate(x, inv, doubtful);
    return doubtful ? quant_value_slow(x, scale) : static_cast<int>(static_cast<int8_t>(q & 0xFFu));
}

__device__ __forceinline__ uint32_t quant_pack4(float4 v, float scale, float inv) {
    bool doubtful = false;
    const uint32_t a = quant_candidate(v.x, inv, doubtful), b = quant_candidate(v.y, inv, doubtful);
    const uint32_t c = quant_candidate(v.z, inv, doubtful), d = quant_candidate(v.w, inv, doubtful);
    const uint32_t w = __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
    return doubtful ? quant_pack4_slow(v, scale) : w;
}

// Exact float of a small non-negative integer (< 2^23) without the
// quarter-rate integer-to-float conversion: 2^23 + i has i in its mantissa.
__device__ __forceinline__ float small_uint_to_float(uint32_t i) {
    return __fsub_rn(__uint_as_float(0x4B000000u | i), 8388608.0f);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace rk

// K1 (weight preparation) and K2 (per-token activation quantisation).
//
// Both are HBM-bound byte/float streams: one CTA per row, coalesced vector
// loads, the dequantised (or loaded) row staged once in shared memory, a
// block-wide absmax, then 16-byte int8 stores.  Arithmetic follows the
// reference exactly (no contraction; the rounding of the IEEE quotient,
// half away from zero, decided by the certified test in quant_math.cuh), so
// the int8 values are bit-identical to its CPU path.
#include <cuda_fp16.h>

#include <algorithm>

#include "kernels.h"
#include "ptx.cuh"
#include "quant_math.cuh"

namespace rk {
namespace {

constexpr int kRowThreads = 256;

__device__ __forceinline__ uint32_t ld32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint32_t ld16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

__device__ __forceinline__ float half_bits_to_float(uint32_t bits) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits & 0xFFFFu)));
}

// Byte i (0..11) of the 12 scale bytes held in three little-endian words.
__device__ __forceinline__ int scale_byte(const uint32_t (&s)[3], int i) {
    const uint32_t w = i < 4 ? s[0] : (i < 8 ? s[1] : s[2]);
    return static_cast<int>((w >> (8 * (i & 3))) & 0xFFu);
}

// 6-bit scale/min pair j of a Q4_K/Q5_K superblock (ggml's K-quant scale
// packing: j < 4 in the low 6 bits of bytes j / j+4, j >= 4 split between
// the nibbles of byte j+4 and the top bits of bytes j-4 / j).
__device__ __forceinline__ void scale_min_k4(int j, const uint32_t (&s)[3], int& sc, int& m) {
    if (j < 4) {
        sc = scale_byte(s, j) & 63;
        m = scale_byte(s, j + 4) & 63;
    } else {
        sc = (scale_byte(s, j + 4) & 0x0F) | ((scale_byte(s, j - 4) >> 6) << 4);
        m = (scale_byte(s, j + 4) >> 4) | ((scale_byte(s, j) >> 6) << 4);
    }
}

// Dequantise the 8 values that thread `l` (0..31) owns in one superblock and
// hand them to `put(slot, index_in_block, value)`; slot 0..7 is a fixed
// per-lane order (Q4_K/Q5_K: slots 0-3 are 4 consecutive values at
// 64g + 4(l%8), slots 4-7 the 4 at 32 further; Q6_K: slots t and 4 + t are the
// 2 consecutive values at 128h + 2(l%16) + 32t).  Value formulas follow the
// llama-gguf dequantisers the reference calls (capi/src/lib.rs:732-733,
// 986-988): Q4_K/Q5_K (d*sc)*q - (dmin*m), Q6_K (d*sc)*(q-32), f32 each step.
template <int KIND, class Put>
__device__ __forceinline__ void dequant8(const uint8_t* blk, int l, Put&& put) {
    if constexpr (KIND == kQ4K || KIND == kQ5K) {
        const uint32_t dd = ld32(blk);
        const float d = half_bits_to_float(dd), dmin = half_bits_to_float(dd >> 16);
        const uint32_t s[3] = {ld32(blk + 4), ld32(blk + 8), ld32(blk + 12)};
        const int g = l >> 3, i4 = (l & 7) * 4;
        int sc, mn;
        scale_min_k4(2 * g, s, sc, mn);
        const float d1 = __fmul_rn(d, static_cast<float>(sc)), m1 = __fmul_rn(dmin, static_cast<float>(mn));
        scale_min_k4(2 * g + 1, s, sc, mn);
        const float d2 = __fmul_rn(d, static_cast<float>(sc)), m2 = __fmul_rn(dmin, static_cast<float>(mn));
        const uint32_t q = ld32(blk + (KIND == kQ4K ? 16 : 48) + 32 * g + i4);
        uint32_t h = 0;
        if constexpr (KIND == kQ5K) h = ld32(blk + 16 + i4);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            int lo = (q >> (8 * i)) & 0x0F, hi = (q >> (8 * i + 4)) & 0x0F;
            if constexpr (KIND == kQ5K) {
                const uint32_t hb = (h >> (8 * i)) & 0xFF;
                lo |= ((hb >> (2 * g)) & 1) << 4;
                hi |= ((hb >> (2 * g + 1)) & 1) << 4;
            }
            put(i, 64 * g + i4 + i, __fsub_rn(__fmul_rn(d1, small_uint_to_float(lo)), m1));
            put(4 + i, 64 * g + 32 + i4 + i, __fsub_rn(__fmul_rn(d2, small_uint_to_float(hi)), m2));
        }
    } else {
        const float d = half_bits_to_float(ld16(blk + 208));
        const int h = l >> 4, lp = (l & 15) * 2;
        const uint32_t qa = ld16(blk + 64 * h + lp);
        const uint32_t qb = ld16(blk + 64 * h + 32 + lp);
        const uint32_t qh = ld16(blk + 128 + 32 * h + lp);
        const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192);
        float ds[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) ds[t] = __fmul_rn(d, static_cast<float>(sc[8 * h + 2 * t + (lp >> 4)]));
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const uint32_t a = (qa >> (8 * e)) & 0xFF, b = (qb >> (8 * e)) & 0xFF, hb = (qh >> (8 * e)) & 0xFF;
            // q - 32 as an exact float: (2^23 + q) - (2^23 + 32)
            const uint32_t q0 = (a & 0x0F) | ((hb & 3) << 4);
            const uint32_t q1 = (b & 0x0F) | (((hb >> 2) & 3) << 4);
            const uint32_t q2 = (a >> 4) | (((hb >> 4) & 3) << 4);
            const uint32_t q3 = (b >> 4) | (((hb >> 6) & 3) << 4);
            const int base = 128 * h + lp + e;
            put(4 * e + 0, base, __fmul_rn(ds[0], __fsub_rn(__uint_as_float(0x4B000000u | q0), 8388640.0f)));
            put(4 * e + 1, base + 32, __fmul_rn(ds[1], __fsub_rn(__uint_as_float(0x4B000000u | q1), 8388640.0f)));
            put(4 * e + 2, base + 64, __fmul_rn(ds[2], __fsub_rn(__uint_as_float(0x4B000000u | q2), 8388640.0f)));
            put(4 * e + 3, base + 96, __fmul_rn(ds[3], __fsub_rn(__uint_as_float(0x4B000000u | q3), 8388640.0f)));
        }
    }
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        float w = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) w = fmaxf(w, __shfl_xor_sync(0xffffffffu, w, o));
        if (threadIdx.x == 0) red[32] = w;
    }
    __syncthreads();
    return red[32];
}

// Quantise a shared-memory row of k floats (k % 16 == 0) to int8 `dst`.
__device__ __forceinline__ void quantize_smem_row(const float* row, int k, float scale, int8_t* dst) {
    const float inv = row_inv(scale);
    for (int i = threadIdx.x * 16; i < k; i += blockDim.x * 16) {
        uint32_t packed[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const float4 v = *reinterpret_cast<const float4*>(row + i + 4 * w);
            packed[w] = quant_pack4(v, scale, inv);
        }
        *reinterpret_cast<uint4*>(dst + i) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    }
}

// K1: one CTA per weight row (prepare_q*_k_w8a8, capi/src/lib.rs:711-757,
// 974-994): dequantise into shared memory, absmax, int8 + scale.
template <int KIND>
__global__ void __launch_bounds__(kRowThreads) prep_w8_kernel(const uint8_t* __restrict__ blocks, int k,
                                                               int8_t* __restrict__ w, float* __restrict__ scales,
                                                               int* __restrict__ err) {
    extern __shared__ __align__(16) float srow[];
    __shared__ float red[33];
    const int row = blockIdx.x;
    const int nb = k >> 8;
    const size_t bb = KIND == kQ4K ? 144 : KIND == kQ5K ? 176 : 210;
    const uint8_t* src = blocks + static_cast<size_t>(row) * nb * bb;
    float amax = 0.0f;
    bool finite = true;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int b = warp; b < nb; b += kRowThreads / 32) {
        float* dst = srow + b * 256;
        dequant8<KIND>(src + b * bb, lane, [&](int, int idx, float v) {
            dst[idx] = v;
            finite &= isfinite(v);
            amax = fmaxf(amax, fabsf(v));
        });
    }
    if (__syncthreads_or(!finite)) {
        if (threadIdx.x == 0) atomicExch(err, kErrNonFinite);
        return;
    }
    const float scale = row_scale(block_max(amax, red));
    quantize_smem_row(srow, k, scale, w + static_cast<size_t>(row) * k);
    if (threadIdx.x == 0) scales[row] = scale;
}

// K1 for rows of up to 8 * BPW superblocks (k <= 16384): the same
// arithmetic as prep_w8_kernel with the dequantised row held in registers
// (8 values per lane per superblock) instead of shared memory, so many more
// rows are in flight per SM and every superblock's loads are issued before
// any value is used.  Stores follow dequant8's slot layout: 4-byte words
// (Q4_K/Q5_K) or 2-byte pairs (Q6_K), coalesced across the warp.
template <int KIND, int BPW>
__global__ void __launch_bounds__(kRowThreads) prep_w8_reg_kernel(const uint8_t* __restrict__ blocks, int k,
                                                                   int8_t* __restrict__ w, float* __restrict__ scales,
                                                                   int* __restrict__ err) {
    __shared__ float red[33];
    const int row = blockIdx.x;
    const int nb = k >> 8;
    const size_t bb = KIND == kQ4K ? 144 : KIND == kQ5K ? 176 : 210;
    const uint8_t* src = blocks + static_cast<size_t>(row) * nb * bb;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float v[BPW][8];
    float amax = 0.0f;
    bool finite = true;
#pragma unroll
    for (int i = 0; i < BPW; ++i) {
        const int b = warp + 8 * i;
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
        if (b < nb) {
            dequant8<KIND>(src + b * bb, lane, [&](int slot, int, float x) {
                v[i][slot] = x;
                finite &= isfinite(x);
                amax = fmaxf(amax, fabsf(x));
            });
        }
    }
    if (__syncthreads_or(!finite)) {
        if (threadIdx.x == 0) atomicExch(err, kErrNonFinite);
        return;
    }
    const float scale = row_scale(block_max(amax, red));
    const float inv = row_inv(scale);
    int8_t* dst = w + static_cast<size_t>(row) * k;
#pragma unroll
    for (int i = 0; i < BPW; ++i) {
        const int b = warp + 8 * i;
        if (b < nb) {
            int8_t* out = dst + b * 256;
            if constexpr (KIND == kQ4K || KIND == kQ5K) {
                const int off = 64 * (lane >> 3) + (lane & 7) * 4;
                *reinterpret_cast<uint32_t*>(out + off) =
                    quant_pack4(make_float4(v[i][0], v[i][1], v[i][2], v[i][3]), scale, inv);
                *reinterpret_cast<uint32_t*>(out + off + 32) =
                    quant_pack4(make_float4(v[i][4], v[i][5], v[i][6], v[i][7]), scale, inv);
            } else {
                const int off = 128 * (lane >> 4) + (lane & 15) * 2;
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const uint32_t lo = quant_value(v[i][t], scale, inv) & 0xFF;
                    const uint32_t hi = quant_value(v[i][4 + t], scale, inv) & 0xFF;
                    *reinterpret_cast<uint16_t*>(out + off + 32 * t) = static_cast<uint16_t>(lo | (hi << 8));
                }
            }
        }
    }
    if (threadIdx.x == 0) scales[row] = scale;
}

// K1 for Q4_K with one thread per 32-value sub-block (8 per superblock; the
// blocks 16-byte aligned).  A sub-block's values are v(q) = (d*sc)*q - dmin*m
// over its 4-bit codes q, each step rounded as in dequant8, so v is monotonic
// in q (rounding keeps order) and |v| over the sub-block peaks at its smallest
// or largest code: the row's absmax, and whether every value is finite, come
// from a byte-wise min / max of the codes and two values -- the same absmax as
// taking every value.  Once the row scale is known, the sub-block's 16
// possible values are quantised (quant_value: the per-value arithmetic of the
// other paths) into a 16-byte table, and every 4 codes become their 4 int8
// bytes through two byte permutes and a select on the code's top bit: the
// same bytes as quantising each value.
__device__ __forceinline__ void q4k_sub(const uint8_t* src, int t, float& d1, float& m1, uint4& c0, uint4& c1,
                                        int& shift) {
    const uint8_t* blk = src + static_cast<size_t>(t >> 3) * 144;
    const int j = t & 7;
    const uint32_t dd = ld32(blk);
    const uint32_t s[3] = {ld32(blk + 4), ld32(blk + 8), ld32(blk + 12)};
    int sc, mn;
    scale_min_k4(j, s, sc, mn);
    d1 = __fmul_rn(half_bits_to_float(dd), static_cast<float>(sc));
    m1 = __fmul_rn(half_bits_to_float(dd >> 16), static_cast<float>(mn));
    // sub-block j: the low (even j) or high (odd j) nibbles of qs[32 (j/2) ..]
    const uint4* q = reinterpret_cast<const uint4*>(blk + 16 + 32 * (j >> 1));
    c0 = q[0];
    c1 = q[1];
    shift = 4 * (j & 1);
}

__device__ __forceinline__ float q4k_value(float d1, float m1, uint32_t q) {
    return __fsub_rn(__fmul_rn(d1, small_uint_to_float(q)), m1);
}

// int8 bytes of 4 codes (one per byte, 0..15) from the 16-byte table t[0..3].
__device__ __forceinline__ uint32_t q4k_lookup4(uint32_t codes, const uint32_t (&t)[4]) {
    const uint32_t lo3 = codes & 0x07070707u;
    const uint32_t sel = __byte_perm(lo3 | (lo3 >> 4), 0u, 0x4420u);  // 4 selector nibbles
    const uint32_t a = __byte_perm(t[0], t[1], sel), b = __byte_perm(t[2], t[3], sel);
    const uint32_t hi = ((codes >> 3) & 0x01010101u) * 0xFFu;         // codes 8..15
    return (b & hi) | (a & ~hi);
}

// One warp per row (8 rows per CTA): no block-wide barrier, the row maximum
// is a warp reduction, and every warp streams its row independently.
__global__ void __launch_bounds__(kRowThreads) prep_w8_q4k_lut_kernel(const uint8_t* __restrict__ blocks, int k,
                                                                       int n, int8_t* __restrict__ w,
                                                                       float* __restrict__ scales,
                                                                       int* __restrict__ err) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (kRowThreads / 32) + (threadIdx.x >> 5);
    if (row >= n) return;  // whole warps
    const int nb = k >> 8, nsub = 8 * nb;
    const uint8_t* src = blocks + static_cast<size_t>(row) * nb * 144;
    float amax = 0.0f;
    bool finite = true;
#pragma unroll 4
    for (int t = lane; t < nsub; t += 32) {
        float d1, m1;
        uint4 c0, c1;
        int sh;
        q4k_sub(src, t, d1, m1, c0, c1, sh);
        const uint32_t m = 0x0F0F0F0Fu;
        uint32_t lo = __vminu4(__vminu4(__vminu4((c0.x >> sh) & m, (c0.y >> sh) & m), (c0.z >> sh) & m),
                               __vminu4(__vminu4((c0.w >> sh) & m, (c1.x >> sh) & m),
                                        __vminu4(__vminu4((c1.y >> sh) & m, (c1.z >> sh) & m), (c1.w >> sh) & m)));
        uint32_t hi = __vmaxu4(__vmaxu4(__vmaxu4((c0.x >> sh) & m, (c0.y >> sh) & m), (c0.z >> sh) & m),
                               __vmaxu4(__vmaxu4((c0.w >> sh) & m, (c1.x >> sh) & m),
                                        __vmaxu4(__vmaxu4((c1.y >> sh) & m, (c1.z >> sh) & m), (c1.w >> sh) & m)));
        lo = __vminu4(lo, lo >> 16);
        lo = min(lo & 0xFFu, (lo >> 8) & 0xFFu);
        hi = __vmaxu4(hi, hi >> 16);
        hi = max(hi & 0xFFu, (hi >> 8) & 0xFFu);
        const float vlo = q4k_value(d1, m1, lo), vhi = q4k_value(d1, m1, hi);
        finite &= isfinite(vlo) && isfinite(vhi);
        amax = fmaxf(amax, fmaxf(fabsf(vlo), fabsf(vhi)));
    }
    if (__any_sync(0xffffffffu, !finite)) {
        if (lane == 0) atomicExch(err, kErrNonFinite);
        return;
    }
    const float scale = row_scale(warp_max(amax));
    const float inv = row_inv(scale);
    int8_t* dst = w + static_cast<size_t>(row) * k;
#pragma unroll 2
    for (int t = lane; t < nsub; t += 32) {
        float d1, m1;
        uint4 c0, c1;
        int sh;
        q4k_sub(src, t, d1, m1, c0, c1, sh);  // this warp's own loads: L1 hits
        // the 16 possible values, quantised 4 at a time (quant_pack4: the
        // same bytes as quant_value on each)
        uint32_t tab[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            tab[i] = quant_pack4(make_float4(q4k_value(d1, m1, 4 * i), q4k_value(d1, m1, 4 * i + 1),
                                             q4k_value(d1, m1, 4 * i + 2), q4k_value(d1, m1, 4 * i + 3)),
                                 scale, inv);
        const uint32_t m = 0x0F0F0F0Fu;
        uint4 o0, o1;
        o0.x = q4k_lookup4((c0.x >> sh) & m, tab);
        o0.y = q4k_lookup4((c0.y >> sh) & m, tab);
        o0.z = q4k_lookup4((c0.z >> sh) & m, tab);
        o0.w = q4k_lookup4((c0.w >> sh) & m, tab);
        o1.x = q4k_lookup4((c1.x >> sh) & m, tab);
        o1.y = q4k_lookup4((c1.y >> sh) & m, tab);
        o1.z = q4k_lookup4((c1.z >> sh) & m, tab);
        o1.w = q4k_lookup4((c1.w >> sh) & m, tab);
        uint4* out = reinterpret_cast<uint4*>(dst + 32 * static_cast<size_t>(t));
        out[0] = o0;
        out[1] = o1;
    }
    if (lane == 0) scales[row] = scale;
}

// FP16 route (dequantize_q*_k_prefill_f16, capi/src/lib.rs:393-455):
// dequantise and round each value to f16; no finiteness check.
template <int KIND>
__global__ void __launch_bounds__(kRowThreads) dequant_f16_kernel(const uint8_t* __restrict__ blocks, int k,
                                                                   __half* __restrict__ w, long long ldw) {
    const int row = blockIdx.x;
    const int nb = k >> 8;
    const size_t bb = KIND == kQ4K ? 144 : KIND == kQ5K ? 176 : 210;
    const uint8_t* src = blocks + static_cast<size_t>(row) * nb * bb;
    __half* out = w + static_cast<size_t>(row) * ldw;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int b = warp; b < nb; b += kRowThreads / 32) {
        __half* dst = out + b * 256;
        dequant8<KIND>(src + b * bb, lane, [&](int, int idx, float v) { dst[idx] = __float2half_rn(v); });
    }
}

// K2: per-token quantisation (quantize_symmetric_into over each activation
// row, capi/src/lib.rs:1776-1791).  Rows whose length is not a multiple of 16
// are zero-padded in shared memory; the padding quantises to 0.
__global__ void __launch_bounds__(kRowThreads) quant_rows_kernel(const float* __restrict__ a, int k, long long lda,
                                                                  int8_t* __restrict__ a8, long long ld8,
                                                                  float* __restrict__ scales,
                                                                  int* __restrict__ err) {
    extern __shared__ __align__(16) float srow[];
    __shared__ float red[33];
    // let the dependent GEMM launch now: it sets up and streams weights while
    // this kernel runs, and waits (griddepcontrol.wait) before reading our
    // output.  (This kernel is an ordinary launch: a programmatic one, waiting
    // here for its own input, measured slower -- its waiting CTAs hold the
    // shared memory the next GEMM's CTAs need.)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int row = blockIdx.x;
    const float* src = a + static_cast<size_t>(row) * lda;
    const int k16 = (k + 15) & ~15;
    float amax = 0.0f;
    bool finite = true;
    const bool vec = ((reinterpret_cast<uintptr_t>(src) & 15) == 0) && (k % 4 == 0);
    if (vec) {
        for (int i = threadIdx.x * 4; i < k; i += kRowThreads * 4) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(src + i));
            *reinterpret_cast<float4*>(srow + i) = v;
            finite &= isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w);
            amax = fmaxf(fmaxf(amax, fmaxf(fabsf(v.x), fabsf(v.y))), fmaxf(fabsf(v.z), fabsf(v.w)));
        }
    } else {
        for (int i = threadIdx.x; i < k; i += kRowThreads) {
            const float v = src[i];
            srow[i] = v;
            finite &= isfinite(v);
            amax = fmaxf(amax, fabsf(v));
        }
    }
    for (int i = k + threadIdx.x; i < k16; i += kRowThreads) srow[i] = 0.0f;
    if (__syncthreads_or(!finite)) {
        if (threadIdx.x == 0) atomicExch(err, kErrNonFinite);
        return;
    }
    const float scale = row_scale(block_max(amax, red));
    int8_t* dst = a8 + static_cast<size_t>(row) * ld8;
    if ((ld8 % 16) == 0 && (reinterpret_cast<uintptr_t>(a8) & 15) == 0 && k16 <= ld8) {
        quantize_smem_row(srow, k16, scale, dst);
    } else {
        const float inv = row_inv(scale);
        for (int i = threadIdx.x; i < k; i += kRowThreads)
            dst[i] = static_cast<int8_t>(quant_value(srow[i], scale, inv));
    }
    if (threadIdx.x == 0) scales[row] = scale;
}

// K2 with the row in registers: 128 threads per row, NV float4 per thread
// (k16 <= 512 NV), the same arithmetic as quant_rows_kernel (zero padding up
// to k16 included).  It holds no row in shared memory and few registers, so
// the GEMM that this kernel launches programmatically can become resident on
// the SMs while the rows are quantised (its prologue and weight loads then
// overlap this kernel).
constexpr int kRegRowThreads = 128;

template <int NV>
__global__ void __launch_bounds__(kRegRowThreads) quant_rows_reg_kernel(const float* __restrict__ a, int k,
                                                                         long long lda, int8_t* __restrict__ a8,
                                                                         long long ld8, float* __restrict__ scales,
                                                                         int* __restrict__ err) {
    __shared__ float red[33];
    // when launched programmatically behind the previous kernel (its CTAs
    // resident before that kernel ends): the rows may be that kernel's
    // output, and a8 / scales may still be read by it; the next GEMM is let
    // go only after that
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int row = blockIdx.x;
    const float4* src = reinterpret_cast<const float4*>(a + static_cast<size_t>(row) * lda);
    const int k4 = k >> 2, k16_4 = ((k + 15) & ~15) >> 2;
    float4 v[NV];
    float amax = 0.0f;
    bool finite = true;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const int i = threadIdx.x + j * kRegRowThreads;
        v[j] = i < k4 ? __ldg(src + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        finite &= isfinite(v[j].x) && isfinite(v[j].y) && isfinite(v[j].z) && isfinite(v[j].w);
        amax = fmaxf(fmaxf(amax, fmaxf(fabsf(v[j].x), fabsf(v[j].y))), fmaxf(fabsf(v[j].z), fabsf(v[j].w)));
    }
    if (__syncthreads_or(!finite)) {
        if (threadIdx.x == 0) atomicExch(err, kErrNonFinite);
        return;
    }
    const float scale = row_scale(block_max(amax, red));
    const float inv = row_inv(scale);
    uint32_t* dst = reinterpret_cast<uint32_t*>(a8 + static_cast<size_t>(row) * ld8);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const int i = threadIdx.x + j * kRegRowThreads;
        if (i < k16_4) dst[i] = quant_pack4(v[j], scale, inv);
    }
    if (threadIdx.x == 0) scales[row] = scale;
}

// SMs running this kernel keep the largest shared-memory partition, so a
// GEMM CTA (~200 KB of shared memory) launched programmatically behind it can
// become resident beside its CTAs; with the default carveout the SM must
// drain and be reconfigured first.
template <typename F>
void prefer_max_shared(F* f) {
    static bool done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && done[dev]) return;
    if (cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared) ==
            cudaSuccess &&
        dev >= 0 && dev < 64)
        done[dev] = true;
    cudaGetLastError();
}

template <int NV>
bool launch_quant_reg(int nv, const float* a, int m, int k, long long lda, int8_t* a8, long long ld8, float* scales,
                      int* err, cudaStream_t s) {
    if constexpr (NV > 12) {
        return false;
    } else {
        if (nv > NV) return launch_quant_reg<NV + (NV < 4 ? NV : 4)>(nv, a, m, k, lda, a8, ld8, scales, err, s);
        prefer_max_shared(quant_rows_reg_kernel<NV>);
        // Up to 128 rows the launch is programmatic: the CTAs become resident
        // while the previous kernel runs and start as soon as it ends
        // (TinyLlama pp128 step on B200: 0.961 against 0.995 ms).  With more
        // rows it measured slower (pp512: 1.444 against 1.336 ms), so larger
        // calls launch normally; the kernel's griddepcontrol.wait is then a
        // no-op.
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(m);
        cfg.blockDim = dim3(kRegRowThreads);
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = m <= 128 ? 1 : 0;
        return cudaLaunchKernelEx(&cfg, quant_rows_reg_kernel<NV>, a, k, lda, a8, ld8, scales, err) == cudaSuccess;
    }
}

// HILO (hilo_stack, capi/src/lib.rs:2045-2070): residual rows of the
// two-part activation encoding, res = x - f32(q) * scale with q, scale from
// the row's own quantisation (two f32 roundings, as the reference).
__global__ void __launch_bounds__(kRowThreads) hilo_residual_kernel(const float* __restrict__ a, int k, long long lda,
                                                                     float* __restrict__ res, long long ldr,
                                                                     int* __restrict__ err) {
    __shared__ float red[33];
    const int row = blockIdx.x;
    const float* src = a + static_cast<size_t>(row) * lda;
    float amax = 0.0f;
    bool finite = true;
    for (int i = threadIdx.x; i < k; i += kRowThreads) {
        const float v = src[i];
        finite &= isfinite(v);
        amax = fmaxf(amax, fabsf(v));
    }
    if (__syncthreads_or(!finite)) {
        if (threadIdx.x == 0) atomicExch(err, kErrNonFinite);
        return;
    }
    const float scale = row_scale(block_max(amax, red));
    const float inv = row_inv(scale);
    float* dst = res + static_cast<size_t>(row) * ldr;
    for (int i = threadIdx.x; i < k; i += kRowThreads) {
        const float x = src[i];
        const float back = __fmul_rn(static_cast<float>(quant_value(x, scale, inv)), scale);
        dst[i] = __fsub_rn(x, back);
    }
}

// hilo_sum (capi/src/lib.rs:2073-2083): out = hi + lo, elementwise f32.
__global__ void add_halves_kernel(const float* __restrict__ hi, const float* __restrict__ lo, float* __restrict__ out,
                                  long long len) {
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < len; i += stride)
        out[i] = __fadd_rn(hi[i], lo[i]);
}

// Rows strided over the grid, 4 values per thread step when the rows are
// 16-byte (f32) / 8-byte (f16) aligned.
__global__ void f32_to_f16_kernel(const float* __restrict__ a, int m, int k, long long lda, __half* __restrict__ out,
                                  long long ldo, bool vec) {
    // the FP16 GEMM that follows may start its prologue and weight loads now
    // (it reads these rows only after its griddepcontrol.wait)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    for (int r = blockIdx.x; r < m; r += gridDim.x) {
        const float* src = a + static_cast<long long>(r) * lda;
        __half* dst = out + static_cast<long long>(r) * ldo;
        if (vec) {
            for (int c = threadIdx.x * 4; c < k; c += blockDim.x * 4) {
                const float4 v = __ldg(reinterpret_cast<const float4*>(src + c));
                __half2 lo = __floats2half2_rn(v.x, v.y), hi = __floats2half2_rn(v.z, v.w);
                uint2 w;
                w.x = *reinterpret_cast<uint32_t*>(&lo);
                w.y = *reinterpret_cast<uint32_t*>(&hi);
                *reinterpret_cast<uint2*>(dst + c) = w;
            }
        } else {
            for (int c = threadIdx.x; c < k; c += blockDim.x) dst[c] = __float2half_rn(src[c]);
        }
    }
}

template <class F>
void set_smem(F* f, size_t bytes) {
    // dynamic + static shared memory above 48 KB needs the opt-in
    if (bytes > 40 * 1024) cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
}

template <int KIND, int BPW>
bool launch_prep_reg(int bpw, const uint8_t* blocks, int k, int n, int8_t* w, float* scales, int* err,
                     cudaStream_t s) {
    if constexpr (BPW > 8) {
        return false;
    } else {
        if (bpw != BPW) return launch_prep_reg<KIND, BPW + 1>(bpw, blocks, k, n, w, scales, err, s);
        prep_w8_reg_kernel<KIND, BPW><<<n, kRowThreads, 0, s>>>(blocks, k, w, scales, err);
        return true;
    }
}

}  // namespace

void launch_prep_w8(int kind, const uint8_t* blocks, int k, int n, int8_t* w, float* scales, int* err,
                    cudaStream_t s) {
    // Q4_K from 16-byte aligned blocks: one thread per sub-block, a warp per row (any k)
    if (kind == kQ4K && (reinterpret_cast<uintptr_t>(blocks) & 15) == 0) {
        const int rows_per_cta = kRowThreads / 32;
        prep_w8_q4k_lut_kernel<<<(n + rows_per_cta - 1) / rows_per_cta, kRowThreads, 0, s>>>(blocks, k, n, w,
                                                                                              scales, err);
        return;
    }
    // rows of up to 64 superblocks: the register kernel
    const int bpw = ((k >> 8) + 7) / 8;
    if (bpw <= 8) {
        if (kind == kQ4K && launch_prep_reg<kQ4K, 1>(bpw, blocks, k, n, w, scales, err, s)) return;
        if (kind == kQ5K && launch_prep_reg<kQ5K, 1>(bpw, blocks, k, n, w, scales, err, s)) return;
        if (kind == kQ6K && launch_prep_reg<kQ6K, 1>(bpw, blocks, k, n, w, scales, err, s)) return;
    }
    const size_t smem = static_cast<size_t>(k) * sizeof(float);
    if (kind == kQ4K) {
        set_smem(prep_w8_kernel<kQ4K>, smem);
        prep_w8_kernel<kQ4K><<<n, kRowThreads, smem, s>>>(blocks, k, w, scales, err);
    } else if (kind == kQ5K) {
        set_smem(prep_w8_kernel<kQ5K>, smem);
        prep_w8_kernel<kQ5K><<<n, kRowThreads, smem, s>>>(blocks, k, w, scales, err);
    } else {
        set_smem(prep_w8_kernel<kQ6K>, smem);
        prep_w8_kernel<kQ6K><<<n, kRowThreads, smem, s>>>(blocks, k, w, scales, err);
    }
}

void launch_dequant_f16(int kind, const uint8_t* blocks, int k, int n, __half* w, long long ldw, int* /*err*/,
                        cudaStream_t s) {
    if (kind == kQ4K)
        dequant_f16_kernel<kQ4K><<<n, kRowThreads, 0, s>>>(blocks, k, w, ldw);
    else if (kind == kQ5K)
        dequant_f16_kernel<kQ5K><<<n, kRowThreads, 0, s>>>(blocks, k, w, ldw);
    else
        dequant_f16_kernel<kQ6K><<<n, kRowThreads, 0, s>>>(blocks, k, w, ldw);
}

void launch_quant_rows(const float* a, int m, int k, long long lda, int8_t* a8, long long ld8, float* scales,
                       int* err, cudaStream_t s) {
    const int k16 = (k + 15) & ~15;
    const int nv = (k16 / 4 + kRegRowThreads - 1) / kRegRowThreads;
    if (k % 4 == 0 && lda % 4 == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0 && ld8 % 4 == 0 &&
        (reinterpret_cast<uintptr_t>(a8) & 3) == 0 && k16 <= ld8 && nv <= 12 &&
        launch_quant_reg<1>(nv, a, m, k, lda, a8, ld8, scales, err, s))
        return;
    const size_t smem = static_cast<size_t>(k16) * sizeof(float);
    set_smem(quant_rows_kernel, smem);
    quant_rows_kernel<<<m, kRowThreads, smem, s>>>(a, k, lda, a8, ld8, scales, err);
}

void launch_f32_to_f16(const float* a, int m, int k, long long lda, __half* out, long long ldo, cudaStream_t s) {
    const bool vec = k % 4 == 0 && lda % 4 == 0 && ldo % 4 == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(out) & 7) == 0;
    const int blocks = std::max(1, std::min(m, 148 * 8));
    prefer_max_shared(f32_to_f16_kernel);
    f32_to_f16_kernel<<<blocks, 256, 0, s>>>(a, m, k, lda, out, ldo, vec);
}

void launch_hilo_residual(const float* a, int m, int k, long long lda, float* res, long long ldr, int* err,
                          cudaStream_t s) {
    hilo_residual_kernel<<<m, kRowThreads, 0, s>>>(a, k, lda, res, ldr, err);
}

void launch_add_halves(const float* hi, const float* lo, float* out, long long len, cudaStream_t s) {
    const int blocks = static_cast<int>(std::min<long long>((len + 255) / 256, 148LL * 16));
    add_halves_kernel<<<std::max(blocks, 1), 256, 0, s>>>(hi, lo, out, len);
}

}  // namespace rk

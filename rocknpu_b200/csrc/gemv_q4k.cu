// K5b for Q4_K: the M=1 decode GEMV y[n] = W[n, k] . x[k] over Q4_K blocks
// split into two planes, streamed from HBM through a shared-memory ring.
//
// Decode layout (prepared once per resident weight, the same 144 bytes per
// 256 weights as ggml's blocks):
//   codes  [n][nb][128]  each block's qs bytes, unchanged;
//   heads  [n][nb][16]   each block's d, dmin, and its 8 scales and 8 mins
//                        regrouped per sub-block pair (q4k_head below).
// The code plane of a row is a run of 16-byte chunks: chunk j (0..7) of
// block b holds bytes 16j..16j+15 of qs, i.e. weights 64g + 16h + [0,16) of
// sub-block 2g in the low nibbles and weights 64g + 32 + 16h + [0,16) of
// sub-block 2g + 1 in the high nibbles (g = j / 2, h = j % 2; ggml's
// dequantize_row_q4_K order).
//
// Work split: a stage is `sr` consecutive rows -- two contiguous ranges, one
// in each plane -- brought in by bulk copies from a producer warp.  Eight
// consumer warps split the stage into units of one 32-chunk step (4 blocks)
// of R rows: lane l always owns chunk l % 8 of block 4 step + l / 8, so it
// reads consecutive 16-byte words (no bank conflicts), its sub-block pair
// (and which header bits to unpack) never changes, and its 32 x values are
// read from shared memory once for the R rows.
//
// Numerics: x is 16-bit fixed point per 64 values, one sub-block pair (X =
// rint(x * 32767 / max|x|), x ~ X * s); per chunk and row the two 16-weight
// code sums against X are exact int32 dp2a sums S_a (low nibbles) and S_b
// (high nibbles, used in place as 16 * code, so the sum is 16 S_b exactly);
// the 6-bit sub-block scales and mins apply in int32 and d, dmin, s in f32:
//   y += s * (d * (sc_a * S_a + sc_b * S_b) - dmin * (m_a * X_a + m_b * X_b))
// with X_a, X_b the sums of X over the chunk's two halves.
//
// x in shared memory ("lane order"): chunk c = 8b + j gets 64 bytes, the 16
// X of its low half then the 16 of its high half, as four 16-byte pieces
// stored at slots rotated by (c / 2) % 4, so the 8 lanes of a quarter-warp
// read 8 different bank groups; then per chunk the constants {s, X_a, X_b}.
//
// Measured on B200 (cfg5 Q4_K 28672 x 8192, 132 MB, back-to-back calls):
// 30.9 us, 0.66 of the measured copy bandwidth; the same pipeline without
// the arithmetic 28.9 us.  Not kept: per-warp 16-byte cp.async rings of 4 x
// 512-byte row pieces (35 us: the scattered 512-byte pieces stream at ~3.7
// TB/s even without arithmetic); loads straight into registers (47 us: too
// few bytes in flight at the register budget); a CTA-wide barrier per stage
// instead of the producer warp (41 us); units of 4 rows instead of 8 (39 us).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdlib>

#include "kernels.h"
#include "ptx.cuh"

namespace rk {
namespace {

constexpr int kQ4Warps = 8;                    // consumer warps
constexpr int kQ4Threads = (kQ4Warps + 1) * 32;  // + one producer warp

struct Q4Params {
    const uint4* codes;  // [n][nb * 8] 16-byte chunks
    const uint4* heads;  // [n][nb]
    const float* x;
    float* y;
    int* err;
    int k, n, nb;
    int steps;  // ceil(nb / 4): 32-chunk steps per row
    int sr;     // rows per stage (a multiple of the rows per unit)
};

// The header of a block in the decode layout: bytes 0..3 as in ggml (f16 d,
// f16 dmin); bytes 4..15 the 8 scales and 8 mins (6 bits each) regrouped per
// sub-block pair: pair g (sub-blocks 2g, 2g + 1) is the 24-bit value
// sc[2g] | sc[2g+1] << 6 | m[2g] << 12 | m[2g+1] << 18 at bytes 4 + 3g.
// ggml's packing (get_scale_min_k4): j < 4: sc = s[j] & 63, m = s[j+4] & 63;
// j >= 4: sc = (s[j+4] & 15) | (s[j-4] >> 6) << 4, m = (s[j+4] >> 4) |
// (s[j] >> 6) << 4, over the 12 scale bytes s.
__device__ __forceinline__ uint4 q4k_head(uint4 h) {
    uint8_t sb[12];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        sb[i] = static_cast<uint8_t>(h.y >> (8 * i));
        sb[4 + i] = static_cast<uint8_t>(h.z >> (8 * i));
        sb[8 + i] = static_cast<uint8_t>(h.w >> (8 * i));
    }
    uint32_t sc[8], mn[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        sc[j] = sb[j] & 63u;
        mn[j] = sb[j + 4] & 63u;
        sc[j + 4] = (sb[j + 8] & 15u) | ((sb[j] >> 6) << 4);
        mn[j + 4] = (sb[j + 8] >> 4) | ((sb[j + 4] >> 6) << 4);
    }
    uint8_t out[12];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        const uint32_t v = sc[2 * g] | (sc[2 * g + 1] << 6) | (mn[2 * g] << 12) | (mn[2 * g + 1] << 18);
        out[3 * g] = static_cast<uint8_t>(v);
        out[3 * g + 1] = static_cast<uint8_t>(v >> 8);
        out[3 * g + 2] = static_cast<uint8_t>(v >> 16);
    }
    uint4 r;
    r.x = h.x;
    r.y = out[0] | (out[1] << 8) | (out[2] << 16) | (static_cast<uint32_t>(out[3]) << 24);
    r.z = out[4] | (out[5] << 8) | (out[6] << 16) | (static_cast<uint32_t>(out[7]) << 24);
    r.w = out[8] | (out[9] << 8) | (out[10] << 16) | (static_cast<uint32_t>(out[11]) << 24);
    return r;
}

// Q4_K ggml blocks (144 bytes, 9 x 16, so 16-byte aligned when the base is)
// -> the two planes.  One 16-byte piece per thread.
__global__ void q4k_planes_kernel(const uint4* __restrict__ src, long long nblocks, uint4* __restrict__ codes,
                                  uint4* __restrict__ heads) {
    const long long total = nblocks * 9;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long b = i / 9;
        const int part = static_cast<int>(i - b * 9);
        const uint4 v = src[i];
        if (part == 0)
            heads[b] = q4k_head(v);
        else
            codes[b * 8 + part - 1] = v;
    }
}

// acc + X0 * b0 + X1 * b1 + X2 * b2 + X3 * b3: the 4 unsigned byte codes of
// `codes` against the signed 16-bit X packed two per word in x01, x23.
__device__ __forceinline__ int dot4(uint32_t codes, uint32_t x01, uint32_t x23, int acc) {
    asm("dp2a.lo.s32.u32 %0, %1, %2, %0;" : "+r"(acc) : "r"(x01), "r"(codes));
    asm("dp2a.hi.s32.u32 %0, %1, %2, %0;" : "+r"(acc) : "r"(x23), "r"(codes));
    return acc;
}

// 16 codes of one half-chunk (byte mask 0x0F0F0F0F: low nibbles; 0xF0F0F0F0:
// 16 * high nibbles) against its 16 X (two 16-byte pieces).
__device__ __forceinline__ int dot16(const uint4& q, uint32_t mask, const uint4& x0, const uint4& x1) {
    int s = dot4(q.x & mask, x0.x, x0.y, 0);
    s = dot4(q.y & mask, x0.z, x0.w, s);
    s = dot4(q.z & mask, x1.x, x1.y, s);
    return dot4(q.w & mask, x1.z, x1.w, s);
}

// Byte `sel & 3` of v as a float, exact: the byte under exponent 2^23, minus
// 2^23.  `sel` is a byte_perm selector 0x7540 | byte.
__device__ __forceinline__ float byte_at(uint32_t v, uint32_t sel) {
    return __uint_as_float(__byte_perm(v, 0x4B000000u, sel)) - 8388608.f;
}

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// x as 16-bit fixed point per 64 values -- one sub-block pair, i.e. the two
// halves of the chunks 8b + 2g and 8b + 2g + 1 -- into lane order (see the
// file comment): one pair per thread per pass.  A chunk's constants are
// {s, X_a, X_b, 0}: the pair's x scale and the sums of X over the chunk's low
// and high half, as int32 bits.
__device__ void q4k_prepare_x(const Q4Params& p, uint4* xq, int4* cst) {
    for (int s = threadIdx.x; s < p.k / 64; s += kQ4Threads) {
        const float4* src = reinterpret_cast<const float4*>(p.x) + 16 * s;
        float4 v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = __ldg(src + i);
        float m = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i)
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
        const bool finite = isfinite(m);
        if (!finite) atomicCAS(p.err, 0, kErrNonFinite);
        const float inv = (finite && m > 0.f) ? 32767.f / m : 0.f;
        const float scale = (finite && m > 0.f) ? m / 32767.f : 0.f;
        // values 0..31: sub-block 2g (low nibbles), 32..63: 2g + 1 (high);
        // quarter qd = 16 values = one half of one sub-block
        uint32_t packed[32];
        int qsum[4] = {0, 0, 0, 0};
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int q0 = max(-32767, min(32767, __float2int_rn(v[i].x * inv)));
            const int q1 = max(-32767, min(32767, __float2int_rn(v[i].y * inv)));
            const int q2 = max(-32767, min(32767, __float2int_rn(v[i].z * inv)));
            const int q3 = max(-32767, min(32767, __float2int_rn(v[i].w * inv)));
            packed[2 * i] = (static_cast<uint32_t>(q0) & 0xFFFFu) | (static_cast<uint32_t>(q1) << 16);
            packed[2 * i + 1] = (static_cast<uint32_t>(q2) & 0xFFFFu) | (static_cast<uint32_t>(q3) << 16);
            qsum[i >> 2] += q0 + q1 + q2 + q3;
        }
        const int b = s >> 2, g = s & 3;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int c = 8 * b + 2 * g + h;  // low half: values 16h.., high half: 32 + 16h..
            const int rot = (c >> 1) & 3;
#pragma unroll
            for (int piece = 0; piece < 4; ++piece) {
                const uint32_t* w = packed + 16 * (piece >> 1) + 8 * h + 4 * (piece & 1);
                xq[4 * c + ((piece + rot) & 3)] = make_uint4(w[0], w[1], w[2], w[3]);
            }
            cst[c] = make_int4(__float_as_int(scale), qsum[h], qsum[2 + h], 0);
        }
    }
}

// Bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned)
// global -> this CTA's shared memory, completing on `bar` (no multicast).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}


// Sum each of R per-lane values over the warp with a transposing butterfly
// (each level sends half of the values still held): row r's total ends in
// lane r * 32 / R (R = 8: 9 shuffles instead of 40; R = 4: 6 instead of 20).
template <int R>
__device__ __forceinline__ float warp_rows(const float (&v)[R], int lane) {
    if constexpr (R == 8) {
        const bool up = lane & 16;
        float r[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            r[i] = (up ? v[4 + i] : v[i]) + __shfl_xor_sync(0xffffffffu, up ? v[i] : v[4 + i], 16);
        const bool b8 = lane & 8;
        float q[2];
#pragma unroll
        for (int i = 0; i < 2; ++i)
            q[i] = (b8 ? r[2 + i] : r[i]) + __shfl_xor_sync(0xffffffffu, b8 ? r[i] : r[2 + i], 8);
        const bool b4 = lane & 4;
        float t = (b4 ? q[1] : q[0]) + __shfl_xor_sync(0xffffffffu, b4 ? q[0] : q[1], 4);
        t += __shfl_xor_sync(0xffffffffu, t, 2);
        t += __shfl_xor_sync(0xffffffffu, t, 1);
        return t;
    } else if constexpr (R == 4) {
        const bool up = lane & 16;
        const float r0 = (up ? v[2] : v[0]) + __shfl_xor_sync(0xffffffffu, up ? v[0] : v[2], 16);
        const float r1 = (up ? v[3] : v[1]) + __shfl_xor_sync(0xffffffffu, up ? v[1] : v[3], 16);
        const bool b8 = lane & 8;
        float t = (b8 ? r1 : r0) + __shfl_xor_sync(0xffffffffu, b8 ? r0 : r1, 8);
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        return t;
    } else if constexpr (R == 2) {
        const bool up = lane & 16;
        float t = (up ? v[1] : v[0]) + __shfl_xor_sync(0xffffffffu, up ? v[0] : v[1], 16);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        return t;
    } else {
        float t = v[0];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        return t;
    }
}

// Lane constants of the unit computation: the lane's sub-block pair
// g = (lane % 8) / 2 sits at header bytes 4 + 3g .. 6 + 3g, i.e. in words
// (y, z) for g < 2 and (z, w) otherwise, gathered by one byte permute; and
// the rotated slots of the lane's four x pieces.
struct Q4Lane {
    bool zw;        // the pair's bytes lie in words z, w (else y, z)
    uint32_t psel;  // byte_perm selector gathering them into bits 0..23
    int s0, s1, s2, s3;
};

// One unit: step `step` (chunk c = 32 step + lane of block 4 step + lane / 8)
// of stage rows r0 .. r0 + R - 1; rows past the stage's end (a partial last
// stage) repeat its last row, and their sums are never read.  Per-lane
// partials in acc.
template <int R>
__device__ __forceinline__ void q4k_unit(const Q4Params& p, const Q4Lane& ln, const uint4* codes, const uint4* heads,
                                         const uint4* xq, const int4* cst, int step, int r0, int rows, int lane,
                                         float (&acc)[R]) {
    const int c = 32 * step + lane, b = 4 * step + (lane >> 3);
    if (b >= p.nb) {
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = 0.f;
        return;
    }
    const uint4 xa0 = xq[4 * c + ln.s0], xa1 = xq[4 * c + ln.s1];
    const uint4 xb0 = xq[4 * c + ln.s2], xb1 = xq[4 * c + ln.s3];
    const int4 k4 = cst[c];  // {x scale bits, X_a, X_b, 0}
    const float xs = __int_as_float(k4.x);
    const uint4* cq = codes + c;
    const uint4* hq = heads + b;
    const int row_u4 = 8 * p.nb;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int rr = min(r0 + r, rows - 1);
        const uint4 q = cq[rr * row_u4];
        const uint4 hw = hq[rr * p.nb];
        const int sa = dot16(q, 0x0F0F0F0Fu, xa0, xa1);
        // high nibbles used in place: every product is 16 x (code x X)
        const int sb = dot16(q, 0xF0F0F0F0u, xb0, xb1) >> 4;
        const uint32_t v = __byte_perm(ln.zw ? hw.z : hw.y, ln.zw ? hw.w : hw.z, ln.psel);
        // both halves share the pair's x scale: scales and mins apply in
        // int32 (|sc * S| < 2^29 each, |m * X| < 2^25 each)
        const int qs = static_cast<int>(v & 63u) * sa + static_cast<int>((v >> 6) & 63u) * sb;
        const int ms = static_cast<int>((v >> 12) & 63u) * k4.y + static_cast<int>((v >> 18) & 63u) * k4.z;
        const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&hw.x));
        acc[r] = xs * fmaf(dm.x, static_cast<float>(qs), -dm.y * static_cast<float>(ms));
    }
}

__device__ __forceinline__ void q4_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Persistent CTAs of 8 consumer warps and one producer warp.  A stage is `sr`
// consecutive rows: their code bytes (one contiguous range of the code plane)
// and their headers (one range of the header plane), brought into ring slot
// k % kQ4Stages by two bulk copies.  The stage's work is split into units
// (32-chunk step along the row) x (R-row group); consumer warp w takes units
// w, w + 8, ...  A unit's lane reads its chunk of each of the R rows
// (consecutive 16-byte words across the warp: conflict-free) and its block's
// header (8 lanes, one address), with the x pieces and constants of its chunk
// read once for the R rows; the unit's warp-reduced row partials go to
// red[slot][row][step], and the warp arrives on the slot's `empty` barrier.
// The producer warp waits for all 8 arrivals, adds each row's steps in order
// (deterministic) into y and refills the slot.  No CTA-wide barrier after the
// prologue; every wait is bounded.
template <int R, int kQ4Stages>
__global__ void __launch_bounds__(kQ4Threads, 2) gemv_q4k_kernel(const Q4Params p) {
    extern __shared__ __align__(128) uint4 smem4[];
    __shared__ uint64_t full[kQ4Stages], empty[kQ4Stages];
    __shared__ volatile int abort_all;
    const int code_u4 = p.sr * p.nb * 8, stage_u4 = code_u4 + p.sr * p.nb;
    uint4* ring = smem4;
    uint4* xq = ring + kQ4Stages * stage_u4;                   // [nb * 8][4]
    int4* cst = reinterpret_cast<int4*>(xq + 32 * p.nb);      // [nb * 8]
    float* red = reinterpret_cast<float*>(cst + 8 * p.nb);    // [kQ4Stages][sr][steps]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nstage = (p.n + p.sr - 1) / p.sr;
    const int my = static_cast<int>(blockIdx.x) < nstage ? (nstage - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    auto stage_row0 = [&](int k) { return (static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x)) * p.sr; };

    if (threadIdx.x == 0) {
        for (int i = 0; i < kQ4Stages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kQ4Warps);
        }
        fence_mbar_init();
        abort_all = 0;
    }
    __syncthreads();
    auto issue = [&](int k) {  // one thread: this CTA's k-th stage into slot k % kQ4Stages
        const int row0 = stage_row0(k);
        const int rows = min(p.sr, p.n - row0);
        uint4* dst = ring + (k % kQ4Stages) * stage_u4;
        const uint32_t cb = static_cast<uint32_t>(rows * p.nb) * 128u, hb = static_cast<uint32_t>(rows * p.nb) * 16u;
        uint64_t* bar = &full[k % kQ4Stages];
        mbar_arrive_expect_tx(bar, cb + hb);
        bulk_g2s(dst, p.codes + static_cast<size_t>(row0) * p.nb * 8, cb, bar);
        bulk_g2s(dst + code_u4, p.heads + static_cast<size_t>(row0) * p.nb, hb, bar);
    };
    // the weight stream starts before x is prepared
    int issued = 0;
    if (warp == kQ4Warps && lane == 0)
        for (; issued < kQ4Stages && issued < my; ++issued) issue(issued);
    q4k_prepare_x(p, xq, cst);
    __syncthreads();

    if (warp == kQ4Warps) {
        // ---- producer: finalise stage k once the consumers are done, refill its slot ----
        int k = 0;
        for (; k < my; ++k) {
            const int sl = k % kQ4Stages;
            int ok = lane == 0 ? (mbar_wait(&empty[sl], (k / kQ4Stages) & 1) ? 1 : 0) : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok || abort_all) {
                if (lane == 0 && !abort_all) {
                    atomicCAS(p.err, 0, kErrTimeoutEmpty);
                    abort_all = 1;
                }
                break;
            }
            const int row0 = stage_row0(k), rows = min(p.sr, p.n - row0);
            const float* rd = red + sl * p.sr * p.steps;
            if (lane < rows) {
                float v = 0.f;
                for (int st = 0; st < p.steps; ++st) v += rd[lane * p.steps + st];
                p.y[row0 + lane] = v;
            }
            __syncwarp();
            if (lane == 0 && issued < my) issue(issued++);
        }
        // copies still in flight (after an abort) land before the CTA leaves
        if (lane == 0)
            for (int i = k; i < issued; ++i)
                if (!mbar_wait(&full[i % kQ4Stages], (i / kQ4Stages) & 1)) break;
    } else {
        // ---- consumers ----
        const int g = (lane & 7) >> 1;
        Q4Lane ln;
        ln.zw = g >= 2;
        ln.psel = g == 0 ? 0x0210u : g == 1 ? 0x0543u : g == 2 ? 0x0432u : 0x0765u;
        const int rot = (lane >> 1) & 3;
        ln.s0 = rot;
        ln.s1 = (1 + rot) & 3;
        ln.s2 = (2 + rot) & 3;
        ln.s3 = (3 + rot) & 3;
        const int units = p.steps * (p.sr / R);
        // this warp's units w, w + 8, ... as (step, first row), advanced
        // without divisions: +8 units = +(8 % steps) steps, +(8 / steps) groups
        const int step0 = warp % p.steps, row0w = (warp / p.steps) * R;
        const int dstep = kQ4Warps % p.steps, drow = (kQ4Warps / p.steps) * R;
        for (int k = 0; k < my; ++k) {
            const int sl = k % kQ4Stages;
            if (!mbar_wait(&full[sl], (k / kQ4Stages) & 1)) {
                if (!abort_all) {
                    atomicCAS(p.err, 0, kErrTimeoutFull);
                    abort_all = 1;
                }
                break;
            }
            if (abort_all) break;
            const uint4* codes = ring + sl * stage_u4;
            const uint4* heads = codes + code_u4;
            const int rows = min(p.sr, p.n - stage_row0(k));
            float* rd = red + sl * p.sr * p.steps;
            int step = step0, r0 = row0w;
            for (int u = warp; u < units; u += kQ4Warps) {
                float acc[R];
                q4k_unit<R>(p, ln, codes, heads, xq, cst, step, r0, rows, lane, acc);
                const float t = warp_rows<R>(acc, lane);
                if ((lane & (32 / R - 1)) == 0) rd[(r0 + lane / (32 / R)) * p.steps + step] = t;
                step += dstep;
                r0 += drow;
                if (step >= p.steps) {
                    step -= p.steps;
                    r0 += R;
                }
            }
            __syncwarp();  // the warp's partials are written before its arrival
            if (lane == 0) q4_arrive(&empty[sl]);
        }
    }
}
}  // namespace

int launch_q4k_layout(const uint8_t* blocks, int k, int n, uint8_t* layout, cudaStream_t s) {
    if (k <= 0 || k % 256 != 0 || n <= 0 || !blocks || !layout) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(blocks) % 16) || (reinterpret_cast<uintptr_t>(layout) % 16))
        return cudaErrorInvalidValue;
    const long long nblocks = static_cast<long long>(n) * (k / 256);
    uint4* codes = reinterpret_cast<uint4*>(layout);
    uint4* heads = codes + nblocks * 8;
    const long long pieces = nblocks * 9;
    const int grid = static_cast<int>(std::min<long long>((pieces + 255) / 256, 148LL * 32));
    q4k_planes_kernel<<<std::max(grid, 1), 256, 0, s>>>(reinterpret_cast<const uint4*>(blocks), nblocks, codes, heads);
    return cudaGetLastError();
}

// Stage rows: as many whole rows as fit ~40 KB (at most 32), rounded down to
// a multiple of the rows per unit (8 when there are 8, else 4, 2 or 1); three
// ring slots when they and x fit ~100 KB (two CTAs per SM), else two.
// ROCKNPU_B200_Q4K_STAGE_KB (8..64) overrides the ~40 KB for tuning; the
// results do not depend on it.
int launch_gemv_q4k(const uint8_t* layout, int k, int n, const float* x, float* y, int* err, cudaStream_t s) {
    if (k <= 0 || k % 256 != 0 || n <= 0 || !layout || !x || !y || !err) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(layout) % 16) || (reinterpret_cast<uintptr_t>(x) % 16))
        return cudaErrorInvalidValue;
    Q4Params p{};
    p.k = k;
    p.n = n;
    p.nb = k / 256;
    p.steps = (p.nb + 3) / 4;
    p.codes = reinterpret_cast<const uint4*>(layout);
    p.heads = p.codes + static_cast<size_t>(n) * p.nb * 8;
    p.x = x;
    p.y = y;
    p.err = err;
    int stage_kb = 40;
    if (const char* v = std::getenv("ROCKNPU_B200_Q4K_STAGE_KB")) {
        const int want = std::atoi(v);
        if (want >= 8 && want <= 64) stage_kb = want;
    }
    const size_t row_bytes = 144u * static_cast<size_t>(p.nb);
    const size_t x_bytes = static_cast<size_t>(p.nb) * 8 * (64 + 16);
    int sr = static_cast<int>(std::max<size_t>(1, std::min<size_t>(32, (stage_kb * 1024u) / row_bytes)));
    sr = std::min(sr, n);
    const int rows = sr >= 8 ? 8 : sr >= 4 ? 4 : sr >= 2 ? 2 : 1;
    sr -= sr % rows;
    p.sr = sr;
    const int stages = 3 * sr * row_bytes + x_bytes <= 100u * 1024u ? 3 : 2;
    const size_t smem = static_cast<size_t>(stages) * sr * row_bytes + x_bytes +
                        static_cast<size_t>(stages) * sr * p.steps * 4;
    if (smem > 200u * 1024u) return cudaErrorInvalidValue;
    const int ri = rows == 8 ? 3 : rows == 4 ? 2 : rows == 2 ? 1 : 0, si = stages - 2;
    static const void* const fns[4][2] = {
        {reinterpret_cast<const void*>(gemv_q4k_kernel<1, 2>), reinterpret_cast<const void*>(gemv_q4k_kernel<1, 3>)},
        {reinterpret_cast<const void*>(gemv_q4k_kernel<2, 2>), reinterpret_cast<const void*>(gemv_q4k_kernel<2, 3>)},
        {reinterpret_cast<const void*>(gemv_q4k_kernel<4, 2>), reinterpret_cast<const void*>(gemv_q4k_kernel<4, 3>)},
        {reinterpret_cast<const void*>(gemv_q4k_kernel<8, 2>), reinterpret_cast<const void*>(gemv_q4k_kernel<8, 3>)}};
    const void* fn = fns[ri][si];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    static bool attr_done[64][4][2] = {};
    if (!attr_done[dev][ri][si]) {
        const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        attr_done[dev][ri][si] = true;
    }
    // CTAs per SM for this shared-memory size (cached per device and variant)
    static int occ[64][4][2] = {};
    static size_t occ_smem[64][4][2] = {};
    int& per_sm = occ[dev][ri][si];
    if (per_sm == 0 || occ_smem[dev][ri][si] != smem) {
        int b = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, fn, kQ4Threads, smem) != cudaSuccess) b = 1;
        per_sm = std::max(b, 1);
        occ_smem[dev][ri][si] = smem;
    }
    const int nstage = (n + sr - 1) / sr;
    const int grid = std::max(1, std::min(nstage, sm_count() * per_sm));
    void* args[] = {&p};
    return cudaLaunchKernel(fn, dim3(grid), dim3(kQ4Threads), args, smem, s);
}

}  // namespace rk

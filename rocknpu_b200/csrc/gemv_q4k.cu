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
// Work split: the shared stage pipeline (gemv_stage.cuh) with a step of 32
// chunks (4 blocks): lane l always owns chunk l % 8 of block 4 step + l / 8,
// so it reads consecutive 16-byte words of a staged row (no bank conflicts),
// its sub-block pair (and which header bits to unpack) never changes, and its
// 32 x values are read from shared memory once for the R rows of a unit.
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

#include "gemv_stage.cuh"

namespace rk {
namespace {

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

// The Q4_K format of the stage pipeline.
struct Q4Fmt {
    static constexpr int kCodeBytes = 128;    // qs
    static constexpr int kHeadBytes = 16;     // d, dmin, regrouped scales and mins
    static constexpr int kBlocksPerStep = 4;  // 8 lanes per block
    static int sr_align(int) { return 1; }    // plane 2 is 16 bytes per block
    // lane-order x (64 bytes per chunk) and per chunk {s, X_a, X_b, 0}
    __host__ __device__ static size_t x_bytes(int nb) { return static_cast<size_t>(nb) * 8 * (64 + 16); }

    // x as 16-bit fixed point per 64 values -- one sub-block pair, i.e. the
    // two halves of the chunks 8b + 2g and 8b + 2g + 1 -- into lane order:
    // one pair per thread per pass.
    __device__ static void prepare_x(const kq::StageParams& p, uint8_t* xsm) {
        uint4* xq = reinterpret_cast<uint4*>(xsm);
        int4* cst = reinterpret_cast<int4*>(xq + 32 * p.nb);
        for (int s = threadIdx.x; s < p.k / 64; s += kq::kThreads) {
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
                const uint2 w = kq::x16_pack(v[i], inv, &qsum[i >> 2]);
                packed[2 * i] = w.x;
                packed[2 * i + 1] = w.y;
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

    // The lane's sub-block pair g = (lane % 8) / 2 sits at header bytes
    // 4 + 3g .. 6 + 3g, i.e. in words (y, z) for g < 2 and (z, w) otherwise,
    // gathered by one byte permute; and the rotated slots of its x pieces.
    struct Lane {
        bool zw;
        uint32_t psel;
        int s0, s1, s2, s3;
    };
    __device__ static Lane lane_consts(int lane) {
        const int g = (lane & 7) >> 1;
        Lane ln;
        ln.zw = g >= 2;
        ln.psel = g == 0 ? 0x0210u : g == 1 ? 0x0543u : g == 2 ? 0x0432u : 0x0765u;
        const int rot = (lane >> 1) & 3;
        ln.s0 = rot;
        ln.s1 = (1 + rot) & 3;
        ln.s2 = (2 + rot) & 3;
        ln.s3 = (3 + rot) & 3;
        return ln;
    }

    // One unit: step `step` (chunk c = 32 step + lane of block 4 step + lane
    // / 8) of stage rows r0 .. r0 + R - 1; rows past the stage's end (a
    // partial last stage) repeat its last row, and their sums are never read.
    template <int R>
    __device__ static void unit(const kq::StageParams& p, const Lane& ln, const uint8_t* codes, const uint8_t* heads,
                                const uint8_t* xsm, int step, int r0, int rows, int lane, float (&acc)[R]) {
        const int c = 32 * step + lane, b = 4 * step + (lane >> 3);
        if (b >= p.nb) {
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r] = 0.f;
            return;
        }
        const uint4* xq = reinterpret_cast<const uint4*>(xsm);
        const int4* cst = reinterpret_cast<const int4*>(xq + 32 * p.nb);
        const uint4 xa0 = xq[4 * c + ln.s0], xa1 = xq[4 * c + ln.s1];
        const uint4 xb0 = xq[4 * c + ln.s2], xb1 = xq[4 * c + ln.s3];
        const int4 k4 = cst[c];  // {x scale bits, X_a, X_b, 0}
        const float xs = __int_as_float(k4.x);
        const uint4* cq = reinterpret_cast<const uint4*>(codes) + c;
        const uint4* hq = reinterpret_cast<const uint4*>(heads) + b;
        const int row_u4 = 8 * p.nb;
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int rr = min(r0 + r, rows - 1);
            const uint4 q = cq[rr * row_u4];
            const uint4 hw = hq[rr * p.nb];
            const int sa = kq::dot16(q, 0x0F0F0F0Fu, xa0, xa1);
            // high nibbles used in place: every product is 16 x (code x X)
            const int sb = kq::dot16(q, 0xF0F0F0F0u, xb0, xb1) >> 4;
            const uint32_t v = __byte_perm(ln.zw ? hw.z : hw.y, ln.zw ? hw.w : hw.z, ln.psel);
            // both halves share the pair's x scale: scales and mins apply in
            // int32 (|sc * S| < 2^29 each, |m * X| < 2^25 each)
            const int qs = static_cast<int>(v & 63u) * sa + static_cast<int>((v >> 6) & 63u) * sb;
            const int ms = static_cast<int>((v >> 12) & 63u) * k4.y + static_cast<int>((v >> 18) & 63u) * k4.z;
            const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&hw.x));
            acc[r] = xs * fmaf(dm.x, static_cast<float>(qs), -dm.y * static_cast<float>(ms));
        }
    }
};

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

int launch_gemv_q4k(const uint8_t* layout, int k, int n, const float* x, float* y, int* err, cudaStream_t s) {
    if (k <= 0 || k % 256 != 0 || n <= 0 || !layout || !x || !y || !err) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(layout) % 16) || (reinterpret_cast<uintptr_t>(x) % 16))
        return cudaErrorInvalidValue;
    const size_t nb = static_cast<size_t>(k / 256);
    return kq::launch_stage<Q4Fmt>(layout, layout + static_cast<size_t>(n) * nb * 128, k, n, x, y, err, s);
}

}  // namespace rk

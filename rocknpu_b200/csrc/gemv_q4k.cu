// K5b for Q4_K: the M=1 decode GEMV y[n] = W[n, k] . x[k] over Q4_K blocks
// split into two planes, streamed from HBM through a shared-memory ring.
//
// Decode layout (prepared once per resident weight, the same 144 bytes per
// 256 weights as ggml's blocks):
//   codes  [n][nb][128]  each row's qs bytes, regrouped per step of 8 blocks
//                        (q4k_planes_kernel);
//   heads  [n][nb][16]   each block's d, dmin, and its 8 scales and 8 mins
//                        regrouped per sub-block pair (q4k_head below).
// Chunk j (qs bytes 16j .. 16j + 15) of a block holds weights 64g + 16h +
// [0,16) of sub-block 2g in the low nibbles and 64g + 32 + 16h + [0,16) of
// sub-block 2g + 1 in the high nibbles (g = j / 2, h = j % 2; ggml's
// dequantize_row_q4_K order).  Within a step the first halves (h = 0) of
// every pair come first, lane-ordered (block i, pair g -> slot 4 i + g), then
// the second halves.
//
// Work split: the shared stage pipeline (gemv_stage.cuh) with a step of 8
// blocks: lane l owns pair g = l % 4 of block 8 step + l / 4, so it reads its
// two chunks at 16-byte slots l and 4 nbs + l of a staged row (consecutive
// lanes, consecutive words: no bank conflicts), decodes the pair's header
// field once per row for 64 weights, and reads its 64 x values from shared
// memory once for the R rows of a unit.
//
// Numerics: x is 16-bit fixed point per 64 values, one sub-block pair (X =
// rint(x * 32767 / max|x|), x ~ X * s); per row the 32-weight code sums
// against X are exact int32 dp2a sums S_a (low nibbles) and S_b (high
// nibbles, used in place as 16 * code, so the sum is 16 S_b exactly); the
// 6-bit sub-block scales and mins apply in int32 and d, dmin, s in f32:
//   y += s * (d * (sc_a * S_a + sc_b * S_b) - dmin * (m_a * X_a + m_b * X_b))
// with X_a, X_b the sums of X over the pair's two sub-blocks.
//
// Measured on B200 (cfg5 Q4_K 28672 x 8192, 132 MB, back-to-back calls):
// the earlier split of one 16-byte chunk per lane (4 blocks per step, the
// header field and scale math per 32 weights) 30.9 us, 0.66 of the measured
// copy bandwidth.  Not kept: per-warp 16-byte cp.async rings of 4 x 512-byte
// row pieces (35 us: the scattered 512-byte pieces stream at ~3.7 TB/s even
// without arithmetic); loads straight into registers (47 us: too few bytes
// in flight at the register budget); a CTA-wide barrier per stage instead of
// the producer warp (41 us); units of 4 rows instead of 8 (39 us); a
// contiguous range of rows per CTA instead of interleaved stages (33 us).
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
// -> the two planes.  One 16-byte piece per thread.  Code chunk j (bytes
// 16j .. 16j + 15 of qs) of block b = 8 t + i of a row goes to 16-byte slot
// (j % 2) * 4 nbs + 4 i + j / 2 of the row's step t (nbs = the step's
// blocks, 8 except in a short last step): the first halves of every
// sub-block pair of the step, then the second halves.
__global__ void q4k_planes_kernel(const uint4* __restrict__ src, long long nblocks, int nb, uint4* __restrict__ codes,
                                  uint4* __restrict__ heads) {
    const long long total = nblocks * 9;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long bi = i / 9;
        const int part = static_cast<int>(i - bi * 9);
        const uint4 v = src[i];
        if (part == 0) {
            heads[bi] = q4k_head(v);
        } else {
            const long long row = bi / nb;
            const int b = static_cast<int>(bi - row * nb), j = part - 1;
            const int t = b >> 3, nbs = min(8, nb - 8 * t);
            codes[row * nb * 8 + 64 * t + (j & 1) * 4 * nbs + 4 * (b & 7) + (j >> 1)] = v;
        }
    }
}

// The Q4_K format of the stage pipeline: a step is 8 blocks (1 KB of codes
// per row) and lane l owns sub-block pair g = l % 4 of block 8 step + l / 4:
// both 16-byte code chunks of the pair, its 64 x values and its header field.
struct Q4Fmt {
    static constexpr int kCodeBytes = 128;    // qs
    static constexpr int kHeadBytes = 16;     // d, dmin, regrouped scales and mins
    static constexpr bool kSplitFull = true;
    static constexpr int kBlocksPerStep = 8;  // 4 lanes per block
    static int sr_align(int) { return 1; }    // plane 2 is 16 bytes per block
    // lane-order x: per step 9 pieces x 32 lanes x 16 bytes
    __host__ __device__ static size_t x_bytes(int nb) { return static_cast<size_t>((nb + 7) / 8) * 9 * 32 * 16; }

    // x as 16-bit fixed point per 64 values -- one sub-block pair -- into
    // lane order: pair t (values 64t .. 64t + 63) is lane t % 32 of step
    // t / 32; its pieces 0..7 hold X[8j .. 8j + 7] and piece 8 the constants
    // {s, X_a = sum X[0..31], X_b = sum X[32..63], 0}; piece j of a step's
    // lane l sits at 16-byte slot 32 (9 step + j) + l.
    __device__ static void prepare_x(const kq::StageParams& p, uint8_t* xsm) {
        uint4* xq = reinterpret_cast<uint4*>(xsm);
        for (int t = threadIdx.x; t < p.k / 64; t += kq::kThreads) {
            const float4* src = reinterpret_cast<const float4*>(p.x) + 16 * t;
            float4 v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = __ldg(src + i);
            float m = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i)
                m = fmaxf(m, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
            const bool finite = isfinite(m);
            if (!finite) kq::set_err(p, kErrNonFinite);
            const float inv = (finite && m > 0.f) ? 32767.f / m : 0.f;
            const float scale = (finite && m > 0.f) ? m / 32767.f : 0.f;
            uint32_t packed[32];
            int qsum[4] = {0, 0, 0, 0};
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint2 w = kq::x16_pack(v[i], inv, &qsum[i >> 2]);
                packed[2 * i] = w.x;
                packed[2 * i + 1] = w.y;
            }
            uint4* dst = xq + 9 * 32 * (t >> 5) + (t & 31);
#pragma unroll
            for (int j = 0; j < 8; ++j)
                dst[32 * j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
            dst[32 * 8] = make_uint4(__float_as_uint(scale), static_cast<uint32_t>(qsum[0] + qsum[1]),
                                     static_cast<uint32_t>(qsum[2] + qsum[3]), 0u);
        }
    }

    // The lane's pair g = lane % 4 sits at header bytes 4 + 3g .. 6 + 3g,
    // i.e. in words (y, z) for g < 2 and (z, w) otherwise, gathered by one
    // byte permute.
    struct Lane {
        bool zw;
        uint32_t psel;
    };
    __device__ static Lane lane_consts(int lane) {
        const int g = lane & 3;
        Lane ln;
        ln.zw = g >= 2;
        ln.psel = g == 0 ? 0x0210u : g == 1 ? 0x0543u : g == 2 ? 0x0432u : 0x0765u;
        return ln;
    }

    // One unit: step `step` of stage rows r0 .. r0 + R - 1.  Per row the
    // lane's two chunks give S_a (low nibbles: sub-block 2g, X[0..31]) and
    // S_b (high nibbles in place, 16 x code: sub-block 2g + 1, X[32..63]) as
    // exact int32 dp2a sums (|S_a| < 2^24, |16 S_b| < 2^28); then
    //   acc = s * (d * (sc_a S_a + sc_b S_b) - dmin * (m_a X_a + m_b X_b))
    // with |sc_a S_a + sc_b S_b| <= 2 * 63 * 15 * 32767 * 32 < 2^31.
    template <int R, bool Full>
    __device__ static void unit(const kq::StageParams& p, const Lane& ln, const uint8_t* codes, const uint8_t* heads,
                                const uint8_t* xsm, int step, int r0, int rows, int lane, float (&acc)[R]) {
        const int b = 8 * step + (lane >> 2);
        if (b >= p.nb) {
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r] = 0.f;
            return;
        }
        const int second = 4 * min(8, p.nb - 8 * step);  // slot of the second halves
        const uint4* xq = reinterpret_cast<const uint4*>(xsm) + 9 * 32 * step + lane;
        const uint4 x0 = xq[0], x1 = xq[32], x2 = xq[64], x3 = xq[96];
        const uint4 x4 = xq[128], x5 = xq[160], x6 = xq[192], x7 = xq[224];
        const uint4 k4 = xq[256];  // {x scale bits, X_a, X_b, 0}
        const float xs = __uint_as_float(k4.x);
        const int xa = static_cast<int>(k4.y), xb = static_cast<int>(k4.z);
        const uint4* cq = reinterpret_cast<const uint4*>(codes) + 64 * step + lane;
        const uint4* hq = reinterpret_cast<const uint4*>(heads) + b;
        const int row_u4 = 8 * p.nb;
#pragma unroll
        for (int r = 0; r < R; ++r) {
            // a full stage has all R rows; a short one skips the missing rows
            if (!Full && r0 + r >= rows) {
                acc[r] = 0.f;
                continue;
            }
            const int rr = r0 + r;
            const uint4 qa = cq[rr * row_u4], qb = cq[rr * row_u4 + second];
            const uint4 hw = hq[rr * p.nb];
            const int sa = kq::dot16(qb, 0x0F0F0F0Fu, x2, x3, kq::dot16(qa, 0x0F0F0F0Fu, x0, x1, 0));
            const int sb = kq::dot16(qb, 0xF0F0F0F0u, x6, x7, kq::dot16(qa, 0xF0F0F0F0u, x4, x5, 0)) >> 4;
            const uint32_t v = __byte_perm(ln.zw ? hw.z : hw.y, ln.zw ? hw.w : hw.z, ln.psel);
            const int qs = static_cast<int>(v & 63u) * sa + static_cast<int>((v >> 6) & 63u) * sb;
            const int ms = static_cast<int>((v >> 12) & 63u) * xa + static_cast<int>((v >> 18) & 63u) * xb;
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
    q4k_planes_kernel<<<std::max(grid, 1), 256, 0, s>>>(reinterpret_cast<const uint4*>(blocks), nblocks, k / 256,
                                                         codes, heads);
    return cudaGetLastError();
}

int launch_gemv_q4k(const uint8_t* layout, int k, int n, const float* x, float* y, int* err, cudaStream_t s,
                    bool host_out) {
    if (k <= 0 || k % 256 != 0 || n <= 0 || !layout || !x || !y || !err) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(layout) % 16) || (reinterpret_cast<uintptr_t>(x) % 16))
        return cudaErrorInvalidValue;
    const size_t nb = static_cast<size_t>(k / 256);
    return kq::launch_stage<Q4Fmt>(layout, layout + static_cast<size_t>(n) * nb * 128, k, n, x, y, err, s, host_out);
}

}  // namespace rk

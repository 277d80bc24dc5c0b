// K5b for Q6_K: the M=1 decode GEMV y[n] = W[n, k] . x[k] over Q6_K blocks in
// a two-plane decode layout, on the shared stage pipeline (gemv_stage.cuh).
//
// ggml's Q6_K block (210 bytes, 256 weights): ql[128], qh[64], scales[16]
// (int8), d (f16).  Weight 128h + 32t + l (h < 2, t < 4, l < 32) has the 6-bit
// code formed by nibble t / 2 of ql[64h + 32 (t % 2) + l] under bits
// 2t..2t+1 of qh[32h + l], sub-block 8h + 2t + l / 16 (16 weights each), and
// value d * sc * (q - 32) (dequantize_row_q6_K).
//
// Decode layout (prepared once per resident weight, the same 210 bytes per
// block plus 16 bytes of padding at the end):
//   plane 1  [n][nb][208]: per block four 48-byte groups G = 2h + c (c < 2),
//            ql[64h + 16c ..+16], ql[64h + 32 + 16c ..+16], qh[32h + 16c ..+16]
//            -- the 64 weights 128h + 32t + 16c + [0,16), t < 4 -- then the 16
//            scales regrouped so that word G holds sc[8h + c + 2t] in byte t;
//   plane 2  [n][nb] the f16 d values.
// Work split: a step is 8 blocks; lane l owns group l % 4 of block
// 8 step + l / 4, so a row's step is 32 x 48 consecutive bytes of the staged
// row, the lane's four sub-blocks never change, and its 64 x values are read
// once for the R rows of a unit.
//
// Numerics as in gemv_kq.cu: x is 16-bit fixed point per block of 32 values
// (X = rint(x * 32767 / max|x|), x ~ X * s); per group, row and t the 16-code
// sum S_t = sum q X is an exact int32 dp2a sum and the offset is applied
// exactly, S_t - 32 sum X; then y += d * sum_t sc_t * s_t * (S_t - 32 sum X)
// in f32.
//
// x in shared memory ("lane order"): chunk cc = 4b + G gets 128 bytes, the X
// of its four 16-value runs t as eight 16-byte pieces 2t, 2t + 1 stored at
// slots rotated by cc % 8 (the 8 lanes of a quarter-warp read 8 different
// bank groups); then per chunk {s_t} (float4) and {32 sum X over run t}
// (int4), the two stored at slots rotated by (cc / 4) % 2.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "gemv_stage.cuh"

namespace rk {
namespace {

// ggml Q6_K blocks (210 bytes, 2-byte aligned) -> the planes: one 16-byte
// piece of plane 1 (13 per block) or one d value per thread.
__global__ void q6k_planes_kernel(const uint8_t* __restrict__ src, long long nblocks, uint8_t* __restrict__ codes,
                                  __half* __restrict__ dvals) {
    const long long total = nblocks * 14;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long b = i / 14;
        const int piece = static_cast<int>(i - b * 14);
        const uint8_t* s = src + b * 210;
        if (piece == 13) {
            dvals[b] = __ushort_as_half(static_cast<unsigned short>(s[208] | (s[209] << 8)));
            continue;
        }
        uint8_t out[16];
        if (piece < 12) {
            const int G = piece / 3, part = piece % 3, h = G >> 1, c = G & 1;
            const int off = part == 0 ? 64 * h + 16 * c : part == 1 ? 64 * h + 32 + 16 * c : 128 + 32 * h + 16 * c;
#pragma unroll
            for (int j = 0; j < 16; ++j) out[j] = s[off + j];
        } else {
#pragma unroll
            for (int G = 0; G < 4; ++G)
#pragma unroll
                for (int t = 0; t < 4; ++t) out[4 * G + t] = s[192 + 8 * (G >> 1) + (G & 1) + 2 * t];
        }
        uint4 v;
        v.x = out[0] | (out[1] << 8) | (out[2] << 16) | (static_cast<uint32_t>(out[3]) << 24);
        v.y = out[4] | (out[5] << 8) | (out[6] << 16) | (static_cast<uint32_t>(out[7]) << 24);
        v.z = out[8] | (out[9] << 8) | (out[10] << 16) | (static_cast<uint32_t>(out[11]) << 24);
        v.w = out[12] | (out[13] << 8) | (out[14] << 16) | (static_cast<uint32_t>(out[15]) << 24);
        reinterpret_cast<uint4*>(codes + b * 208)[piece] = v;
    }
}

// The Q6_K format of the stage pipeline.
struct Q6Fmt {
    static constexpr int kCodeBytes = 208;    // four 48-byte groups + regrouped scales
    static constexpr int kHeadBytes = 2;      // d
    static constexpr bool kSplitFull = false;
    static constexpr int kBlocksPerStep = 8;  // 4 lanes per block
    // plane 2 holds 2 bytes per block: a stage's d range starts 16-byte
    // aligned when sr * nb is a multiple of 8
    static int sr_align(int nb) {
        int g = 8;
        while (nb % g) g >>= 1;
        return 8 / g;
    }
    // lane-order x (128 bytes per chunk) and per chunk {s_t}, {32 sum X}
    __host__ __device__ static size_t x_bytes(int nb) { return static_cast<size_t>(nb) * 4 * (128 + 32); }

    // x as 16-bit fixed point per block of 32 values: block s = 8b + 4h + t
    // holds run t of the chunks 4b + 2h and 4b + 2h + 1 (its halves).
    __device__ static void prepare_x(const kq::StageParams& p, uint8_t* xsm) {
        uint4* xq = reinterpret_cast<uint4*>(xsm);
        uint4* cst = xq + 32 * p.nb;
        for (int s = threadIdx.x; s < p.k / 32; s += kq::kThreads) {
            const float4* src = reinterpret_cast<const float4*>(p.x) + 8 * s;
            float4 v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = __ldg(src + i);
            float m = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                m = fmaxf(m, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
            const bool finite = isfinite(m);
            if (!finite) kq::set_err(p, kErrNonFinite);
            const float inv = (finite && m > 0.f) ? 32767.f / m : 0.f;
            const float scale = (finite && m > 0.f) ? m / 32767.f : 0.f;
            uint32_t packed[16];
            int half_sum[2] = {0, 0};
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint2 w = kq::x16_pack(v[i], inv, &half_sum[i >> 2]);
                packed[2 * i] = w.x;
                packed[2 * i + 1] = w.y;
            }
            const int b = s >> 3, h = (s >> 2) & 1, t = s & 3;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int cc = 4 * b + 2 * h + c;
                const int rot8 = cc & 7, rot2 = (cc >> 2) & 1;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const uint32_t* w = packed + 8 * c + 4 * half;
                    xq[8 * cc + ((2 * t + half + rot8) & 7)] = make_uint4(w[0], w[1], w[2], w[3]);
                }
                reinterpret_cast<float*>(cst + 2 * cc + (rot2 & 1))[t] = scale;
                reinterpret_cast<int*>(cst + 2 * cc + ((1 + rot2) & 1))[t] = 32 * half_sum[c];
            }
        }
    }

    struct Lane {
        int G;     // group within the block
        int rot8;  // rotation of the x pieces
        int rot2;  // rotation of the constants
    };
    __device__ static Lane lane_consts(int lane) {
        Lane ln;
        ln.G = lane & 3;
        ln.rot8 = lane & 7;
        ln.rot2 = (lane >> 2) & 1;
        return ln;
    }

    // One unit: step `step` (group G of block 8 step + lane / 4) of stage
    // rows r0 .. r0 + R - 1; rows past the stage's end repeat its last row
    // (their sums are never read).
    template <int R, bool Full>
    __device__ static void unit(const kq::StageParams& p, const Lane& ln, const uint8_t* codes, const uint8_t* heads,
                                const uint8_t* xsm, int step, int r0, int rows, int lane, float (&acc)[R]) {
        const int cc = 32 * step + lane, b = 8 * step + (lane >> 2);
        if (b >= p.nb) {
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r] = 0.f;
            return;
        }
        const uint4* xq = reinterpret_cast<const uint4*>(xsm);
        uint4 X[8];
#pragma unroll
        for (int pc = 0; pc < 8; ++pc) X[pc] = xq[8 * cc + ((pc + ln.rot8) & 7)];
        const uint4* cst = xq + 32 * p.nb;
        const float4 xs = *reinterpret_cast<const float4*>(cst + 2 * cc + (ln.rot2 & 1));
        const int4 x32 = *reinterpret_cast<const int4*>(cst + 2 * cc + ((1 + ln.rot2) & 1));
        const float xsv[4] = {xs.x, xs.y, xs.z, xs.w};
        const int x32v[4] = {x32.x, x32.y, x32.z, x32.w};
        const __half* dv = reinterpret_cast<const __half*>(heads);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            // rows past a short stage's end repeat its last row (their sums
            // are never read); measured faster here than skipping them
            const int rr = min(r0 + r, rows - 1);
            const uint8_t* blk = codes + (static_cast<size_t>(rr) * p.nb + b) * 208;
            const uint4 A = *reinterpret_cast<const uint4*>(blk + 48 * ln.G);
            const uint4 B = *reinterpret_cast<const uint4*>(blk + 48 * ln.G + 16);
            const uint4 C = *reinterpret_cast<const uint4*>(blk + 48 * ln.G + 32);
            const uint32_t scw = *reinterpret_cast<const uint32_t*>(blk + 192 + 4 * ln.G);
            const uint32_t Aw[4] = {A.x, A.y, A.z, A.w}, Bw[4] = {B.x, B.y, B.z, B.w}, Cw[4] = {C.x, C.y, C.z, C.w};
            int S[4] = {0, 0, 0, 0};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint32_t q[4] = {(Aw[u] & 0x0F0F0F0Fu) | ((Cw[u] << 4) & 0x30303030u),
                                       (Bw[u] & 0x0F0F0F0Fu) | ((Cw[u] << 2) & 0x30303030u),
                                       ((Aw[u] >> 4) & 0x0F0F0F0Fu) | (Cw[u] & 0x30303030u),
                                       ((Bw[u] >> 4) & 0x0F0F0F0Fu) | ((Cw[u] >> 2) & 0x30303030u)};
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const uint4& xp = X[2 * t + (u >> 1)];
                    S[t] = (u & 1) ? kq::dot4(q[t], xp.z, xp.w, S[t]) : kq::dot4(q[t], xp.x, xp.y, S[t]);
                }
            }
            float sum = 0.f;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float sc = static_cast<float>(static_cast<int8_t>((scw >> (8 * t)) & 0xFFu));
                sum = fmaf(sc * xsv[t], static_cast<float>(S[t] - x32v[t]), sum);
            }
            acc[r] = __half2float(dv[static_cast<size_t>(rr) * p.nb + b]) * sum;
        }
    }
};

}  // namespace

int launch_q6k_layout(const uint8_t* blocks, int k, int n, uint8_t* layout, cudaStream_t s) {
    if (k <= 0 || k % 256 != 0 || n <= 0 || !blocks || !layout) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(blocks) % 2) || (reinterpret_cast<uintptr_t>(layout) % 16))
        return cudaErrorInvalidValue;
    const long long nblocks = static_cast<long long>(n) * (k / 256);
    const long long items = nblocks * 14;
    const int grid = static_cast<int>(std::min<long long>((items + 255) / 256, 148LL * 32));
    q6k_planes_kernel<<<std::max(grid, 1), 256, 0, s>>>(blocks, nblocks, layout,
                                                         reinterpret_cast<__half*>(layout + nblocks * 208));
    // the 16 bytes of padding after the d plane (read by rounded-up stage copies)
    const cudaError_t e = cudaMemsetAsync(layout + nblocks * 210, 0, 16, s);
    return e != cudaSuccess ? e : cudaGetLastError();
}

int launch_gemv_q6k(const uint8_t* layout, int k, int n, const float* x, float* y, int* err, cudaStream_t s,
                    bool host_out) {
    if (k <= 0 || k % 256 != 0 || n <= 0 || !layout || !x || !y || !err) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(layout) % 16) || (reinterpret_cast<uintptr_t>(x) % 16))
        return cudaErrorInvalidValue;
    const size_t nb = static_cast<size_t>(k / 256);
    return kq::launch_stage<Q6Fmt>(layout, layout + static_cast<size_t>(n) * nb * 208, k, n, x, y, err, s, host_out);
}

}  // namespace rk

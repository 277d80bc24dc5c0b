// K5b: M=1 decode GEMV straight from K-quant superblocks, y[n] = W[n, k] . x[k]
// with W dequantised in registers (no tensor cores, no int8 copy): the Q6_K
// kernel and the layout / launch entry points for both kinds (the Q4_K
// kernel is in gemv_q4k.cu).
//
// Why: a decode step streams every weight once, so its time is the weight
// bytes over HBM bandwidth.  Q4_K is 0.5625 bytes per weight, Q6_K 0.8203,
// the prepared int8 rows of the W8A8 path 1 + 4/k -- the reference keeps
// M=1 on llama.cpp's K-quant kernels for exactly that reason
// (ggml-rocknpu.cpp:305-312).
//
// Numerics: every weight is ggml's f32 dequantisation (Q6_K: d * sc * (q -
// 32) over 16-weight sub-blocks), applied per sub-block rather than per
// weight: sum_i w_i x_i = d sc (sum_i q_i x_i - 32 sum_i x_i).  x is held as
// 16-bit fixed point per block of 32 (X = rint(x * 32767 / max|x|), x ~ X *
// s), so sum_i q_i X_i is an exact int32 dp2a sum.  Representing x that way
// moves each x by at most 1/65534 of its block's largest magnitude; the
// outputs land within ~1e-6 of sum |w x| of the exact dot product of the f32
// weights (the tests assert the north_star's 1e-3 relative bound with that
// cancellation term).
//
// Q6_K decode layout: each 210-byte block without its trailing f16 d: 208
// bytes = 13 x 16 (ql[128], qh[64], scales[16]), rows of 208 * k/256 bytes,
// followed by the d values [n][k/256] as f16 -- the same 210 bytes per
// block, laid out so that 128-bit copies stay aligned.
//
// Kernel: persistent CTAs of 8 warps (two per SM).  Each warp walks its own
// sequence of row sets (32 / seg consecutive rows, seg = the power of two at
// or above k / 256, at most 32) and streams them into its own shared-memory
// ring with 16-byte cp.async copies issued by all 32 lanes -- coalesced, 512
// bytes per instruction, one set ahead.  A lane then takes whole
// superblocks (256 weights) of one row from shared memory, so a block's 16
// scales are read once per 256 weights, and the row's partial sums are
// reduced with shuffles inside its segment of seg lanes.  No block-wide
// barrier after the prologue and no spin: a warp waits only for its own
// copies.  x is quantised once per CTA into shared memory as int16 with 16
// bytes of padding per 256 values, so lanes on neighbouring blocks read
// different banks.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdlib>

#include "kernels.h"
#include "ptx.cuh"

namespace rk {
namespace {

constexpr int kKqWarps = 8;
constexpr int kKqThreads = kKqWarps * 32;
constexpr int kQ6Body = 208;  // Q6_K decode-layout block (ql, qh, scales)

struct KqParams {
    const uint8_t* w;   // decode-layout rows
    const __half* d6;   // Q6_K: d [n][nb]; unused for Q4_K
    const float* x;
    float* y;
    int* err;
    int k, n, nb;
    int row_bytes;        // bytes of one decode-layout row
    int seg, rows_per_warp;  // seg lanes per row, 32 / seg rows per warp
    int slot_bytes;          // rows_per_warp rows, rounded up to 16
};

// Shared-memory byte offset of the 16-bit x value at position i: 16 bytes of
// padding after every 256 values (512 bytes), so lanes reading different
// superblocks hit different banks.
__device__ __forceinline__ int xq_off(int i) { return 2 * i + 16 * (i >> 8); }

// acc + X0 * b0 + X1 * b1 + X2 * b2 + X3 * b3 for the 4 unsigned byte codes of
// `codes` and the signed 16-bit x values packed two per word in x01, x23.
__device__ __forceinline__ int dot4(uint32_t codes, uint32_t x01, uint32_t x23, int acc) {
    asm("dp2a.lo.s32.u32 %0, %1, %2, %0;" : "+r"(acc) : "r"(x01), "r"(codes));
    asm("dp2a.hi.s32.u32 %0, %1, %2, %0;" : "+r"(acc) : "r"(x23), "r"(codes));
    return acc;
}

// Byte J of v as a float: the byte under exponent 2^23, minus 2^23 (exact).
template <int J>
__device__ __forceinline__ float byte_f(uint32_t v) {
    return __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7540u | J)) - 8388608.f;
}

// Byte J of v as a signed integer, as a float.
template <int J>
__device__ __forceinline__ float sbyte_f(uint32_t v) {
    return static_cast<float>(static_cast<int8_t>((v >> (8 * J)) & 0xFFu));
}

// One Q6_K superblock (decode layout: ql[128], qh[64], scales[16]) of one
// row.  Weight 128h + 32t + l (h < 2, t < 4, l < 32) has the 6-bit code
// formed by nibble (t >> 1) of ql[64h + 32(t & 1) + l] and bits 2t..2t+1 of
// qh[32h + l] above it, sub-block 8h + 2t + l/16, and value d * sc * (q - 32).
// xs: the block's 8 x scales (per 32 values); xsum: its 16 sums of X (per 16).
__device__ __forceinline__ float q6k_block(const uint4* __restrict__ blk, float d, const uint8_t* __restrict__ xb,
                                           const float* __restrict__ xs, const int* __restrict__ xsum) {
    const uint4 scw = blk[12];
    float r = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint4 l0 = blk[4 * h], l1 = blk[4 * h + 1], l2 = blk[4 * h + 2], l3 = blk[4 * h + 3];
        const uint4 h0 = blk[8 + 2 * h], h1 = blk[9 + 2 * h];
        const uint32_t a[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};  // ql[64h + l]
        const uint32_t b[8] = {l2.x, l2.y, l2.z, l2.w, l3.x, l3.y, l3.z, l3.w};  // ql[64h + 32 + l]
        const uint32_t c[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};  // qh[32h + l]
        int sm[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // [2t + l/16]
#pragma unroll
        for (int i = 0; i < 8; ++i) {  // columns l = 4i .. 4i+3
            const uint32_t q0 = (a[i] & 0x0F0F0F0Fu) | ((c[i] << 4) & 0x30303030u);
            const uint32_t q1 = (b[i] & 0x0F0F0F0Fu) | ((c[i] << 2) & 0x30303030u);
            const uint32_t q2 = ((a[i] >> 4) & 0x0F0F0F0Fu) | (c[i] & 0x30303030u);
            const uint32_t q3 = ((b[i] >> 4) & 0x0F0F0F0Fu) | ((c[i] >> 2) & 0x30303030u);
            const int hb = i >> 2;
            const uint2 x0 = *reinterpret_cast<const uint2*>(xb + 2 * (128 * h + 4 * i));
            const uint2 x1 = *reinterpret_cast<const uint2*>(xb + 2 * (128 * h + 32 + 4 * i));
            const uint2 x2 = *reinterpret_cast<const uint2*>(xb + 2 * (128 * h + 64 + 4 * i));
            const uint2 x3 = *reinterpret_cast<const uint2*>(xb + 2 * (128 * h + 96 + 4 * i));
            sm[hb] = dot4(q0, x0.x, x0.y, sm[hb]);
            sm[2 + hb] = dot4(q1, x1.x, x1.y, sm[2 + hb]);
            sm[4 + hb] = dot4(q2, x2.x, x2.y, sm[4 + hb]);
            sm[6 + hb] = dot4(q3, x3.x, x3.y, sm[6 + hb]);
        }
        // scales of sub-blocks 8h .. 8h + 7: bytes of scw.x, scw.y (h = 0) or scw.z, scw.w
        const uint32_t s0 = h ? scw.z : scw.x, s1 = h ? scw.w : scw.y;
        const float f[8] = {sbyte_f<0>(s0), sbyte_f<1>(s0), sbyte_f<2>(s0), sbyte_f<3>(s0),
                            sbyte_f<0>(s1), sbyte_f<1>(s1), sbyte_f<2>(s1), sbyte_f<3>(s1)};
#pragma unroll
        for (int j = 0; j < 8; ++j)  // sub-block 8h + j: t = j / 2, x block 4h + j / 2
            r = fmaf(f[j] * xs[4 * h + (j >> 1)], static_cast<float>(sm[j] - 32 * xsum[8 * h + j]), r);
    }
    return d * r;
}

// 16-byte asynchronous copy global -> shared (L2 only), and its group
// bookkeeping: a lane's copies since the last commit form one group.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Ring slots per warp (copies run kSlots - 1 row sets ahead).  Two slots
// leave room for two CTAs per SM, which measured fastest on B200 (cfg5 Q4_K
// 28672 x 8192: 41 us with 2 slots x 2 CTAs, 47-51 us with 3-4 slots x 1 CTA,
// 43 us with 1 slot x 3 CTAs).
constexpr int kSlots = 2;

// Shared memory: [warps][kSlots][slot_bytes] row-set ring | x as int16,
// padded | x scale per 32 | sum of X per 16 | sum of x as held per 32.
template <int SLOTS>
__global__ void __launch_bounds__(kKqThreads, 2) gemv_kq_kernel(const KqParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* ring = smem + static_cast<size_t>(warp) * SLOTS * p.slot_bytes;
    uint8_t* xq = smem + static_cast<size_t>(kKqWarps) * SLOTS * p.slot_bytes;
    float* xscale = reinterpret_cast<float*>(xq + xq_off(p.k));
    int* xsum16 = reinterpret_cast<int*>(xscale + p.k / 32);

    // This warp's row sets: first, first + stride, ...  A set is the
    // rows_per_warp consecutive rows the warp works on at once.
    const int sets = (p.n + p.rows_per_warp - 1) / p.rows_per_warp;
    const int first = blockIdx.x * kKqWarps + warp, stride = gridDim.x * kKqWarps;
    auto issue = [&](int set, int slot) {
        const int rows = min(p.rows_per_warp, p.n - set * p.rows_per_warp);
        const int chunks = rows * p.row_bytes / 16;
        const uint4* src = reinterpret_cast<const uint4*>(p.w + static_cast<size_t>(set) * p.rows_per_warp * p.row_bytes);
        uint4* dst = reinterpret_cast<uint4*>(ring + static_cast<size_t>(slot) * p.slot_bytes);
        for (int c = lane; c < chunks; c += 32) cp_async16(dst + c, src + c);  // coalesced: 512 B per step
    };
    // the weight stream starts before x is quantised
#pragma unroll
    for (int i = 0; i < SLOTS - 1; ++i) {
        const int set = first + i * stride;
        if (set < sets) issue(set, i);
        cp_async_commit();
    }

    // x as 16-bit fixed point per block of 32 values, X = rint(x * 32767 /
    // max|x|): one block per thread, all its loads in flight at once
    for (int blk = threadIdx.x; blk < p.k / 32; blk += kKqThreads) {
        const float4* src = reinterpret_cast<const float4*>(p.x) + 8 * blk;
        float4 v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __ldg(src + i);
        float m = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i)
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
        const bool finite = isfinite(m);
        if (!finite) atomicCAS(p.err, 0, kErrNonFinite);
        const float inv = (finite && m > 0.f) ? 32767.f / m : 0.f;
        uint32_t packed[16];
        int s0 = 0, s1 = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int q0 = max(-32767, min(32767, __float2int_rn(v[i].x * inv)));
            const int q1 = max(-32767, min(32767, __float2int_rn(v[i].y * inv)));
            const int q2 = max(-32767, min(32767, __float2int_rn(v[i].z * inv)));
            const int q3 = max(-32767, min(32767, __float2int_rn(v[i].w * inv)));
            packed[2 * i] = (static_cast<uint32_t>(q0) & 0xFFFFu) | (static_cast<uint32_t>(q1) << 16);
            packed[2 * i + 1] = (static_cast<uint32_t>(q2) & 0xFFFFu) | (static_cast<uint32_t>(q3) << 16);
            if (i < 4)
                s0 += q0 + q1 + q2 + q3;
            else
                s1 += q0 + q1 + q2 + q3;
        }
        uint4* dst = reinterpret_cast<uint4*>(xq + xq_off(32 * blk));
#pragma unroll
        for (int i = 0; i < 4; ++i)
            dst[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
        xsum16[2 * blk] = s0;
        xsum16[2 * blk + 1] = s1;
        const float scale = (finite && m > 0.f) ? m / 32767.f : 0.f;
        xscale[blk] = scale;
    }
    __syncthreads();

    // each lane: superblocks b0, b0 + seg, ... of row `rw` of the set
    const int rw = lane / p.seg, b0 = lane - rw * p.seg;
    int it = 0;
    for (int set = first; set < sets; set += stride, ++it) {
        // refill the slot the previous set used, SLOTS - 1 sets ahead
        const int ahead = set + (SLOTS - 1) * stride;
        if (ahead < sets) issue(ahead, (it + SLOTS - 1) % SLOTS);
        cp_async_commit();
        cp_async_wait<SLOTS - 1>();  // this set's group has landed (for this lane)
        __syncwarp();                // ... and for every lane of the warp
        const int row = set * p.rows_per_warp + rw;
        float acc = 0.f;
        if (row < p.n) {
            const uint8_t* rowp = ring + static_cast<size_t>(it % SLOTS) * p.slot_bytes + static_cast<size_t>(rw) * p.row_bytes;
            for (int b = b0; b < p.nb; b += p.seg) {
                const uint8_t* xb = xq + xq_off(256 * b);
                const float dv = __half2float(p.d6[static_cast<size_t>(row) * p.nb + b]);
                acc += q6k_block(reinterpret_cast<const uint4*>(rowp + kQ6Body * b), dv, xb, xscale + 8 * b,
                                 xsum16 + 16 * b);
            }
        }
        for (int o = p.seg >> 1; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (b0 == 0 && row < p.n) p.y[row] = acc;
        __syncwarp();  // the slot is read by every lane before it is refilled
    }
    cp_async_wait<0>();
}

// Q6_K ggml blocks (210 bytes) -> decode layout: 208-byte bodies [n][nb] then
// the f16 d values [n][nb].  One warp per block; 2-byte loads (the 210-byte
// blocks are only 2-byte aligned).
__global__ void q6k_layout_kernel(const uint8_t* __restrict__ src, long long nblocks, uint8_t* __restrict__ body,
                                  __half* __restrict__ dvals) {
    const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
    const int lane = threadIdx.x & 31;
    for (long long b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < nblocks; b += warps) {
        const uint16_t* s = reinterpret_cast<const uint16_t*>(src + b * 210);
        uint16_t* o = reinterpret_cast<uint16_t*>(body + b * kQ6Body);
        for (int i = lane; i < kQ6Body / 2; i += 32) o[i] = s[i];
        if (lane == 0) dvals[b] = __ushort_as_half(s[kQ6Body / 2]);
    }
}

}  // namespace

size_t kq_layout_bytes(int kind, size_t k, size_t n) {
    const size_t nb = k / 256;
    if (kind == kQ4K) return n * nb * 144;
    if (kind == kQ6K) return n * nb * (kQ6Body + 2);
    return 0;
}

int launch_kq_layout(int kind, const uint8_t* blocks, int k, int n, uint8_t* layout, cudaStream_t s) {
    const long long nb = k / 256;
    if (kind == kQ4K) return launch_q4k_layout(blocks, k, n, layout, s);
    if (kind != kQ6K) return cudaErrorInvalidValue;
    const long long nblocks = static_cast<long long>(n) * nb;
    const int grid = static_cast<int>(std::min<long long>((nblocks + 7) / 8, 148LL * 16));
    q6k_layout_kernel<<<std::max(grid, 1), 256, 0, s>>>(blocks, nblocks, layout,
                                                         reinterpret_cast<__half*>(layout + nblocks * kQ6Body));
    return cudaGetLastError();
}

// Geometry: a row takes `seg` lanes (the power of two at or above k / 256,
// at most 32), a warp 32 / seg rows at a time; CTAs of 8 warps, each warp
// with a ring of kSlots row-set slots beside x, as many CTAs per SM as fit.
// Rows too long for one slot per warp in ~220 KB are rejected.
int launch_gemv_kq(int kind, const uint8_t* layout, int k, int n, const float* x, float* y, int* err,
                   cudaStream_t s) {
    if (kind == kQ4K) return launch_gemv_q4k(layout, k, n, x, y, err, s);
    if (kind != kQ6K || k <= 0 || k % 256 != 0 || n <= 0 || !layout || !x || !y || !err)
        return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(layout) % 16) || (reinterpret_cast<uintptr_t>(x) % 16))
        return cudaErrorInvalidValue;
    KqParams p{};
    p.k = k;
    p.n = n;
    p.nb = k / 256;
    p.row_bytes = p.nb * kQ6Body;
    p.seg = 1;
    while (p.seg < p.nb && p.seg < 32) p.seg <<= 1;
    p.rows_per_warp = 32 / p.seg;
    p.slot_bytes = p.rows_per_warp * p.row_bytes;
    p.w = layout;
    p.d6 = reinterpret_cast<const __half*>(layout + static_cast<size_t>(n) * p.nb * kQ6Body);
    p.x = x;
    p.y = y;
    p.err = err;
    const size_t xbytes = static_cast<size_t>(2 * k + 16 * (k / 256)) + 4 * static_cast<size_t>(k / 32) +
                          4 * static_cast<size_t>(k / 16);
    constexpr size_t kBudget = 220u * 1024u;
    int slots = 0;
    for (int sl = kSlots; sl >= 1 && slots == 0; --sl)
        if (static_cast<size_t>(kKqWarps) * sl * p.slot_bytes + xbytes <= kBudget) slots = sl;
    if (const char* v = std::getenv("ROCKNPU_B200_KQ_SLOTS")) {  // tuning override (same results)
        const int want = std::atoi(v);
        if (want >= 1 && want < slots) slots = want;
    }
    if (slots == 0) return cudaErrorInvalidValue;
    const size_t smem = static_cast<size_t>(kKqWarps) * slots * p.slot_bytes + xbytes;
    // the shared-memory limit is raised once per device and depth
    static bool attr_done[64][4] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    const void* fn = slots == 4   ? reinterpret_cast<const void*>(gemv_kq_kernel<4>)
                     : slots == 3 ? reinterpret_cast<const void*>(gemv_kq_kernel<3>)
                     : slots == 2 ? reinterpret_cast<const void*>(gemv_kq_kernel<2>)
                                  : reinterpret_cast<const void*>(gemv_kq_kernel<1>);
    if (!attr_done[dev][slots - 1]) {
        const cudaError_t e =
            cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kBudget));
        if (e != cudaSuccess) return e;
        attr_done[dev][slots - 1] = true;
    }
    // CTAs per SM for this shared-memory size (cached per device and depth)
    static int occ[64][4] = {};
    static size_t occ_smem[64][4] = {};
    int& per_sm = occ[dev][slots - 1];
    if (per_sm == 0 || occ_smem[dev][slots - 1] != smem) {
        int b = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, fn, kKqThreads, smem) != cudaSuccess) b = 1;
        per_sm = std::max(b, 1);
        occ_smem[dev][slots - 1] = smem;
    }
    const int sets = (n + p.rows_per_warp - 1) / p.rows_per_warp;
    const int grid = std::max(1, std::min((sets + kKqWarps - 1) / kKqWarps, sm_count() * per_sm));
    void* args[] = {&p};
    return cudaLaunchKernel(fn, dim3(grid), dim3(kKqThreads), args, smem, s);
}

}  // namespace rk

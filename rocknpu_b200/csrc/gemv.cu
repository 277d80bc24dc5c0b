// K5: M=1 W8A8 GEMV for decode (execute_cached_w8a8_m1,
// capi/src/lib.rs:1567-1701), HBM-bound on the resident int8 weights.
//
// One warp per output row: the quantised activation (K bytes) is staged once
// per CTA in shared memory; each lane streams 16-byte weight chunks with
// no-L1-allocate loads, four dp4a per chunk, an exact int32 warp sum, and
// lane 0 applies the reference's rescale (f32(acc) * a_scale) * w_scale.
#include "kernels.h"
#include "ptx.cuh"
#include "quant_math.cuh"

namespace rk {
namespace {

constexpr int kGemvThreads = 256;
constexpr int kRowsPerCta = kGemvThreads / 32;

__device__ __forceinline__ int4 ld_stream(const int4* p) {
    int4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// The first chunks a lane reads of its warp's row (16-byte chunks lane,
// lane + 32, lane + 64, lane + 96; zero past the row or for a row past n),
// issued before the activation is ready so that their DRAM latency overlaps
// its staging; at k <= 2048 they are the whole row.
__device__ __forceinline__ void row_head(const int8_t* __restrict__ w, int k, int n, int4 (&pre)[4]) {
    const int chunks = k >> 4;
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * kRowsPerCta + (threadIdx.x >> 5);
    const int4* wr = reinterpret_cast<const int4*>(w + static_cast<size_t>(row) * k);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int idx = lane + 32 * u;
        pre[u] = (row < n && idx < chunks) ? ld_stream(wr + idx) : make_int4(0, 0, 0, 0);
    }
}

__device__ __forceinline__ int dot_chunk(const int4& w, const int4& a, int acc) {
    acc = __dp4a(w.x, a.x, acc);
    acc = __dp4a(w.y, a.y, acc);
    acc = __dp4a(w.z, a.z, acc);
    return __dp4a(w.w, a.w, acc);
}

// The warp's row of this CTA against the quantised activation staged in
// shared memory, starting from its row_head: the rescaled result, in every
// lane (0 for a row past n).  The int32 sum is exact, so the order in which
// chunks are added does not change it.
__device__ __forceinline__ float gemv_row(const int4* sa, const int8_t* __restrict__ w,
                                          const float* __restrict__ w_scale, float a_scale, int k, int n,
                                          const int4 (&pre)[4]) {
    const int chunks = k >> 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * kRowsPerCta + warp;
    if (row >= n) return 0.0f;
    const int4* wr = reinterpret_cast<const int4*>(w + static_cast<size_t>(row) * k);
    int acc = 0;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int idx = lane + 32 * u;
        if (idx < chunks) acc = dot_chunk(pre[u], sa[idx], acc);
    }
    int i = lane + 128;
    for (; i + 96 < chunks; i += 128) {
        const int4 w0 = ld_stream(wr + i), w1 = ld_stream(wr + i + 32), w2 = ld_stream(wr + i + 64),
                   w3 = ld_stream(wr + i + 96);
        acc = dot_chunk(w0, sa[i], acc);
        acc = dot_chunk(w1, sa[i + 32], acc);
        acc = dot_chunk(w2, sa[i + 64], acc);
        acc = dot_chunk(w3, sa[i + 96], acc);
    }
    for (; i < chunks; i += 32) acc = dot_chunk(ld_stream(wr + i), sa[i], acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    return __fmul_rn(__fmul_rn(__int2float_rn(acc), a_scale), w_scale[row]);
}

__global__ void __launch_bounds__(kGemvThreads) gemv_w8a8_kernel(const int8_t* __restrict__ w,
                                                                  const float* __restrict__ w_scale,
                                                                  const int8_t* __restrict__ a8,
                                                                  const float* __restrict__ a_scale, int k, int n,
                                                                  float* __restrict__ out) {
    extern __shared__ int4 sa[];
    int4 pre[4];
    row_head(w, k, n, pre);
    const int chunks = k >> 4;
    for (int i = threadIdx.x; i < chunks; i += kGemvThreads) sa[i] = reinterpret_cast<const int4*>(a8)[i];
    __syncthreads();
    const float v = gemv_row(sa, w, w_scale, *a_scale, k, n, pre);
    const int row = blockIdx.x * kRowsPerCta + (threadIdx.x >> 5);
    if ((threadIdx.x & 31) == 0 && row < n) out[row] = v;
}

// K2 + K5 in one launch for M=1: every CTA quantises the f32 activation x
// (16-byte aligned, k % 16 == 0) into shared memory with the row quantiser's
// arithmetic -- the same absmax (a max is order-independent), scale and
// per-value rounding, so the same bits -- then runs the rows above.  The
// repeated work per CTA is one 4k-byte read of x (L2-resident after the
// first CTAs) and a block reduction.  A non-finite x sets kErrNonFinite and
// no output is written.  HostOut: `out` and `err` are page-locked host memory
// mapped into the device: a CTA's 8 results leave as one 32-byte store, and
// the error is a plain store (every writer stores the same value; atomics to
// host memory need PCIe atomics).
template <bool HostOut>
__global__ void __launch_bounds__(kGemvThreads) gemv_w8a8_x_kernel(const int8_t* __restrict__ w,
                                                                    const float* __restrict__ w_scale,
                                                                    const float* __restrict__ x, int k, int n,
                                                                    float* __restrict__ out, int* err) {
    extern __shared__ int4 sa[];
    __shared__ float red[kGemvThreads / 32];
    int4 pre[4];
    row_head(w, k, n, pre);
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const int k4 = k >> 2;
    float amax = 0.0f;
    bool finite = true;
    for (int i = threadIdx.x; i < k4; i += kGemvThreads) {
        const float4 v = __ldg(x4 + i);
        finite &= isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w);
        amax = fmaxf(fmaxf(amax, fmaxf(fabsf(v.x), fabsf(v.y))), fmaxf(fabsf(v.z), fabsf(v.w)));
    }
    if (__syncthreads_or(!finite)) {
        if (threadIdx.x == 0) {
            if constexpr (HostOut)
                *reinterpret_cast<volatile int*>(err) = kErrNonFinite;
            else
                atomicExch(err, kErrNonFinite);
        }
        return;
    }
    amax = warp_max(amax);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    float m = red[0];
#pragma unroll
    for (int i = 1; i < kGemvThreads / 32; ++i) m = fmaxf(m, red[i]);
    const float scale = row_scale(m), inv = row_inv(scale);
    uint32_t* sa32 = reinterpret_cast<uint32_t*>(sa);
    for (int i = threadIdx.x; i < k4; i += kGemvThreads) sa32[i] = quant_pack4(__ldg(x4 + i), scale, inv);
    __syncthreads();
    const float v = gemv_row(sa, w, w_scale, scale, k, n, pre);
    if constexpr (HostOut) {
        __shared__ float res[kRowsPerCta];
        if ((threadIdx.x & 31) == 0) res[threadIdx.x >> 5] = v;
        __syncthreads();
        const int r = blockIdx.x * kRowsPerCta + threadIdx.x;
        if (threadIdx.x < kRowsPerCta && r < n) out[r] = res[threadIdx.x];
    } else {
        const int row = blockIdx.x * kRowsPerCta + (threadIdx.x >> 5);
        if ((threadIdx.x & 31) == 0 && row < n) out[row] = v;
    }
}

}  // namespace

void launch_gemv_w8a8(const int8_t* w, const float* w_scale, const int8_t* a8, const float* a_scale, int k, int n,
                      float* out, cudaStream_t s) {
    const size_t smem = static_cast<size_t>(k);
    if (smem > 48 * 1024)
        cudaFuncSetAttribute(gemv_w8a8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    gemv_w8a8_kernel<<<(n + kRowsPerCta - 1) / kRowsPerCta, kGemvThreads, smem, s>>>(w, w_scale, a8, a_scale, k, n,
                                                                                     out);
}

void launch_gemv_w8a8_x(const int8_t* w, const float* w_scale, const float* x, int k, int n, float* out, int* err,
                        cudaStream_t s, bool host_out) {
    const size_t smem = static_cast<size_t>(k);
    auto kern = host_out ? gemv_w8a8_x_kernel<true> : gemv_w8a8_x_kernel<false>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    kern<<<(n + kRowsPerCta - 1) / kRowsPerCta, kGemvThreads, smem, s>>>(w, w_scale, x, k, n, out, err);
}

}  // namespace rk

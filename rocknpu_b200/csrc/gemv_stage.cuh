// The K5b decode-GEMV pipeline shared by the K-quant formats (gemv_q4k.cu,
// gemv_q6k.cu): y[n] = W[n, k] . x[k] with W in a two-plane decode layout,
// streamed from HBM in stages of whole rows.
//
// A stage is `sr` consecutive rows: their bytes in plane 1 (codes, one
// contiguous range) and in plane 2 (per-block header bytes, one contiguous
// range), brought into ring slot k % S of the CTA's shared memory by two bulk
// copies from a producer warp.  Eight consumer warps split the stage into
// units of one step along the row (the blocks that 32 lanes cover) x R rows;
// consumer warp w takes units w, w + 8, ...  A format's unit routine reads
// each lane's piece of every row from the slot and the lane's x values once
// for the R rows; the unit's warp-reduced row partials go to
// red[slot][row][step], and the warp arrives on the slot's `empty` barrier.
// The producer waits for all 8 arrivals, adds each row's steps in order
// (deterministic) into y and refills the slot.  No CTA-wide barrier after the
// prologue; every wait is bounded (ptx.cuh), and a wait that runs out sets
// the status word and a CTA-wide abort flag.
//
// A format F provides:
//   kCodeBytes, kHeadBytes      plane-1 and plane-2 bytes per block;
//   kBlocksPerStep              blocks per step (32 lanes);
//   x_bytes(nb)                 shared-memory bytes of its x representation;
//   prepare_x(p, xsm)           x into shared memory (all threads, once per CTA);
//   Lane, lane_consts(lane)     per-lane constants;
//   kSplitFull                  whether full stages get their own unit<R, true>
//                               (measured on B200, cfg5 weight: Q4_K 27.3
//                               against 28.9 us; Q6_K 41.8 against 40.6 us,
//                               its larger unit body twice in the loop);
//   unit<R, Full>(p, ln, codes, heads, xsm, step, r0, rows, lane, acc)
//                               per-lane partials of rows r0 .. r0 + R - 1
//                               (Full: all R rows exist; else rows >= `rows`
//                               give 0 and are not read).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdlib>

#include "kernels.h"
#include "ptx.cuh"

namespace rk {
namespace kq {

constexpr int kWarps = 8;                    // consumer warps
constexpr int kThreads = (kWarps + 1) * 32;  // + one producer warp

struct StageParams {
    const uint8_t* codes;  // plane 1: [n][nb][F::kCodeBytes]
    const uint8_t* heads;  // plane 2: [n][nb][F::kHeadBytes]
    const float* x;
    float* y;
    int* err;
    int k, n, nb;
    int steps;  // steps per row: ceil(nb / F::kBlocksPerStep)
    int sr;     // rows per stage (a multiple of the rows per unit)
    int err_plain;  // err (and y) are mapped host memory: errors by plain store
};

// Record an error code: in device memory the first error wins (atomic); a
// status word in mapped host memory takes a plain store (atomics to host
// memory need PCIe atomic operations), so there a later error code may
// replace an earlier one -- either way the word is non-zero.
__device__ __forceinline__ void set_err(const StageParams& p, int code) {
    if (p.err_plain)
        *reinterpret_cast<volatile int*>(p.err) = code;
    else
        atomicCAS(p.err, 0, code);
}

// acc + X0 * b0 + X1 * b1 + X2 * b2 + X3 * b3: the 4 unsigned byte codes of
// `codes` against the signed 16-bit X packed two per word in x01, x23.
__device__ __forceinline__ int dot4(uint32_t codes, uint32_t x01, uint32_t x23, int acc) {
    asm("dp2a.lo.s32.u32 %0, %1, %2, %0;" : "+r"(acc) : "r"(x01), "r"(codes));
    asm("dp2a.hi.s32.u32 %0, %1, %2, %0;" : "+r"(acc) : "r"(x23), "r"(codes));
    return acc;
}

// acc + 16 byte codes (one uint4, each byte masked with `mask`) against 16 X
// (two 16-byte pieces of 8 int16 each).
__device__ __forceinline__ int dot16(const uint4& q, uint32_t mask, const uint4& x0, const uint4& x1, int acc) {
    int s = dot4(q.x & mask, x0.x, x0.y, acc);
    s = dot4(q.y & mask, x0.z, x0.w, s);
    s = dot4(q.z & mask, x1.x, x1.y, s);
    return dot4(q.w & mask, x1.z, x1.w, s);
}

// 16-bit fixed point of 4 floats: rint(v * inv) clamped to +-32767, packed
// two per word; adds the four values to *sum.
__device__ __forceinline__ uint2 x16_pack(const float4& v, float inv, int* sum) {
    const int q0 = max(-32767, min(32767, __float2int_rn(v.x * inv)));
    const int q1 = max(-32767, min(32767, __float2int_rn(v.y * inv)));
    const int q2 = max(-32767, min(32767, __float2int_rn(v.z * inv)));
    const int q3 = max(-32767, min(32767, __float2int_rn(v.w * inv)));
    *sum += q0 + q1 + q2 + q3;
    return make_uint2((static_cast<uint32_t>(q0) & 0xFFFFu) | (static_cast<uint32_t>(q1) << 16),
                      (static_cast<uint32_t>(q2) & 0xFFFFu) | (static_cast<uint32_t>(q3) << 16));
}

// Bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned)
// global -> this CTA's shared memory, completing on `bar` (no multicast).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void stage_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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

__host__ __device__ constexpr size_t round16(size_t b) { return (b + 15) & ~static_cast<size_t>(15); }

// Persistent CTAs of 8 consumer warps and one producer warp (see the top of
// this file).  Shared memory: S ring slots of one stage each (plane 1, then
// plane 2 at a 16-byte boundary) | the format's x | red[S][sr][steps].
template <class F, int R, int S>
__global__ void __launch_bounds__(kThreads, 2) stage_kernel(const StageParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[S], empty[S];
    __shared__ volatile int abort_all;
    const size_t code_bytes = static_cast<size_t>(p.sr) * p.nb * F::kCodeBytes;
    const size_t stage_bytes = round16(code_bytes) + round16(static_cast<size_t>(p.sr) * p.nb * F::kHeadBytes);
    uint8_t* ring = smem;
    uint8_t* xsm = smem + S * stage_bytes;
    float* red = reinterpret_cast<float*>(xsm + F::x_bytes(p.nb));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // CTA b's k-th stage starts at row (b + k * grid) * sr: neighbouring CTAs
    // stream neighbouring rows (measured faster on B200 than a contiguous
    // range per CTA, 30.9 against 33.0 us on the cfg5 Q4_K weight)
    const int nstage = (p.n + p.sr - 1) / p.sr;
    const int my = static_cast<int>(blockIdx.x) < nstage ? (nstage - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    auto stage_row0 = [&](int k) { return (static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x)) * p.sr; };
    auto stage_rows = [&](int k) { return min(p.sr, p.n - stage_row0(k)); };

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kWarps);
        }
        fence_mbar_init();
        abort_all = 0;
    }
    __syncthreads();
    // one thread: this CTA's k-th stage into slot k % S.  Plane 2's range is
    // rounded up to 16 bytes (the host keeps its start 16-byte aligned and the
    // layout ends in 16 bytes of padding)
    auto issue = [&](int k) {
        const int row0 = stage_row0(k);
        const int rows = stage_rows(k);
        uint8_t* dst = ring + (k % S) * stage_bytes;
        const uint32_t cb = static_cast<uint32_t>(rows * p.nb) * F::kCodeBytes;
        const uint32_t hb = static_cast<uint32_t>(round16(static_cast<size_t>(rows) * p.nb * F::kHeadBytes));
        uint64_t* bar = &full[k % S];
        mbar_arrive_expect_tx(bar, cb + hb);
        bulk_g2s(dst, p.codes + static_cast<size_t>(row0) * p.nb * F::kCodeBytes, cb, bar);
        bulk_g2s(dst + round16(code_bytes), p.heads + static_cast<size_t>(row0) * p.nb * F::kHeadBytes, hb, bar);
    };
    // the weight stream starts before x is prepared
    int issued = 0;
    if (warp == kWarps && lane == 0)
        for (; issued < S && issued < my; ++issued) issue(issued);
    F::prepare_x(p, xsm);
    __syncthreads();

    if (warp == kWarps) {
        // ---- producer: finalise stage k once the consumers are done, refill its slot ----
        int k = 0;
        for (; k < my; ++k) {
            const int sl = k % S;
            int ok = lane == 0 ? (mbar_wait(&empty[sl], (k / S) & 1) ? 1 : 0) : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok || abort_all) {
                if (lane == 0 && !abort_all) {
                    set_err(p, kErrTimeoutEmpty);
                    abort_all = 1;
                }
                break;
            }
            const int row0 = stage_row0(k), rows = stage_rows(k);
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
                if (!mbar_wait(&full[i % S], (i / S) & 1)) break;
    } else {
        // ---- consumers ----
        const typename F::Lane ln = F::lane_consts(lane);
        const int units = p.steps * (p.sr / R);
        // this warp's units w, w + 8, ... as (step, first row), advanced
        // without divisions: +8 units = +(8 % steps) steps, +(8 / steps) groups
        const int step0 = warp % p.steps, row0w = (warp / p.steps) * R;
        const int dstep = kWarps % p.steps, drow = (kWarps / p.steps) * R;
        for (int k = 0; k < my; ++k) {
            const int sl = k % S;
            if (!mbar_wait(&full[sl], (k / S) & 1)) {
                if (!abort_all) {
                    set_err(p, kErrTimeoutFull);
                    abort_all = 1;
                }
                break;
            }
            if (abort_all) break;
            const uint8_t* codes = ring + sl * stage_bytes;
            const uint8_t* heads = codes + round16(code_bytes);
            const int rows = stage_rows(k);
            float* rd = red + sl * p.sr * p.steps;
            int step = step0, r0 = row0w;
            for (int u = warp; u < units; u += kWarps) {
                if constexpr (F::kSplitFull) {
                    if (r0 < rows) {  // a short last stage skips its empty units
                        float acc[R];
                        if (rows == p.sr)
                            F::template unit<R, true>(p, ln, codes, heads, xsm, step, r0, rows, lane, acc);
                        else
                            F::template unit<R, false>(p, ln, codes, heads, xsm, step, r0, rows, lane, acc);
                        const float t = warp_rows<R>(acc, lane);
                        if ((lane & (32 / R - 1)) == 0) rd[(r0 + lane / (32 / R)) * p.steps + step] = t;
                    }
                } else {
                    float acc[R];
                    F::template unit<R, false>(p, ln, codes, heads, xsm, step, r0, rows, lane, acc);
                    const float t = warp_rows<R>(acc, lane);
                    if ((lane & (32 / R - 1)) == 0) rd[(r0 + lane / (32 / R)) * p.steps + step] = t;
                }
                step += dstep;
                r0 += drow;
                if (step >= p.steps) {
                    step -= p.steps;
                    r0 += R;
                }
            }
            __syncwarp();  // the warp's partials are written before its arrival
            if (lane == 0) stage_arrive(&empty[sl]);
        }
    }
}

// Host side.  Stage rows: as many whole rows as fit ~40 KB (at most 32),
// rounded down to a multiple of the rows per unit (8 when there are 8, else
// 4, 2 or 1) and of F::sr_align(nb) (plane-2 copies start 16-byte aligned);
// three ring slots when they and x fit ~100 KB (two CTAs per SM), else two.
// ROCKNPU_B200_KQ_STAGE_KB (8..64) overrides the ~40 KB for tuning; results
// do not depend on it.  F::x_bytes and the ring must fit 200 KB.
template <class F>
int launch_stage(const uint8_t* codes, const uint8_t* heads, int k, int n, const float* x, float* y, int* err,
                 cudaStream_t s, bool host_out = false) {
    StageParams p{};
    p.err_plain = host_out ? 1 : 0;
    p.k = k;
    p.n = n;
    p.nb = k / 256;
    p.steps = (p.nb + F::kBlocksPerStep - 1) / F::kBlocksPerStep;
    p.codes = codes;
    p.heads = heads;
    p.x = x;
    p.y = y;
    p.err = err;
    int stage_kb = 40;
    if (const char* v = std::getenv("ROCKNPU_B200_KQ_STAGE_KB")) {
        const int want = std::atoi(v);
        if (want >= 8 && want <= 64) stage_kb = want;
    }
    const size_t row_bytes = static_cast<size_t>(p.nb) * (F::kCodeBytes + F::kHeadBytes);
    int sr = static_cast<int>(std::max<size_t>(1, std::min<size_t>(32, (stage_kb * 1024u) / row_bytes)));
    sr = std::min(sr, n);
    int rows = sr >= 8 ? 8 : sr >= 4 ? 4 : sr >= 2 ? 2 : 1;
    const int step_rows = std::max(rows, F::sr_align(p.nb));  // both are powers of two
    if (sr >= step_rows) {
        sr -= sr % step_rows;
    } else if (n >= step_rows) {
        sr = step_rows;
    } else {
        sr = n;  // one stage from row 0: plane 2 starts aligned
        rows = 1;
    }
    p.sr = sr;
    const size_t stage_bytes = round16(static_cast<size_t>(sr) * p.nb * F::kCodeBytes) +
                               round16(static_cast<size_t>(sr) * p.nb * F::kHeadBytes);
    const size_t x_bytes = F::x_bytes(p.nb);
    const int stages = 3 * stage_bytes + x_bytes <= 100u * 1024u ? 3 : 2;
    const size_t smem = stages * stage_bytes + x_bytes + static_cast<size_t>(stages) * sr * p.steps * 4;
    if (smem > 200u * 1024u) return cudaErrorInvalidValue;
    const int ri = rows == 8 ? 3 : rows == 4 ? 2 : rows == 2 ? 1 : 0, si = stages - 2;
    static const void* const fns[4][2] = {
        {reinterpret_cast<const void*>(stage_kernel<F, 1, 2>), reinterpret_cast<const void*>(stage_kernel<F, 1, 3>)},
        {reinterpret_cast<const void*>(stage_kernel<F, 2, 2>), reinterpret_cast<const void*>(stage_kernel<F, 2, 3>)},
        {reinterpret_cast<const void*>(stage_kernel<F, 4, 2>), reinterpret_cast<const void*>(stage_kernel<F, 4, 3>)},
        {reinterpret_cast<const void*>(stage_kernel<F, 8, 2>), reinterpret_cast<const void*>(stage_kernel<F, 8, 3>)}};
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
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, fn, kThreads, smem) != cudaSuccess) b = 1;
        per_sm = std::max(b, 1);
        occ_smem[dev][ri][si] = smem;
    }
    const int nstage = (n + sr - 1) / sr;
    const int grid = std::max(1, std::min(nstage, sm_count() * per_sm));
    void* args[] = {&p};
    return cudaLaunchKernel(fn, dim3(grid), dim3(kThreads), args, smem, s);
}

}  // namespace kq
}  // namespace rk

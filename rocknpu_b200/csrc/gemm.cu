// K3 (W8A8 prefill GEMM) and K4 (FP16 executor GEMM) on the 5th-generation
// tensor cores.
//
// Orientation ("swap AB"): the MMA's M side is 128 weight rows (output
// columns) and its N side is a tile of BT tokens, so one tcgen05.mma
// instruction covers 128 x BT x 32 bytes of K, and short prompts (BT = 16..64)
// waste no tensor-core rows.  The int32 / f32 accumulator lives in TMEM:
// lane = weight row, column = token.  The epilogue reads one lane per thread,
// so a warp's 32 threads own 32 consecutive output columns and every store of
// the f32 result row is a coalesced 128-byte line.
//
// Pipeline: warp 0 issues TMA tile loads (128-byte swizzle, no multicast) into
// a STAGES-deep shared-memory ring; warp 1 owns TMEM and issues the MMAs
// (one elected thread); warps 2..5 run the epilogue
//   kind 0:  out[m, n] = (f32(acc) * a_scale[m]) * w_scale[n]
//            (rescale_i32_row's order, capi/src/lib.rs:692-709), optional
//            raw int32 dump;
//   kind 1:  out[m, n] = acc (f32).
// Every barrier wait is bounded; a wait that runs out records an error code
// in *err, drains what is in flight (bounded), frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <mutex>

#include "kernels.h"
#include "ptx.cuh"

namespace rk {
namespace {

constexpr int kWRows = 128;          // weight rows per tile (MMA M)
constexpr int kKBytes = 128;         // K bytes per pipeline stage (one swizzle row)
constexpr int kThreads = 192;        // 6 warps

struct GemmParams {
    CUtensorMap tmap_w;  // [n rows][k] K-major
    CUtensorMap tmap_a;  // [m rows][k] K-major
    const float* w_scale;
    const float* a_scale;
    int m, n, num_kb, kb_elems;
    int tiles_n, tiles_m, group_m;
    int nmembers;
    int n_start[5];
    float* out[4];
    long long ldo[4];
    int32_t* acc_out;
    long long acc_ld;
    int* err;
};

template <int BT, int STAGES>
struct Smem {
    static constexpr int kWBytes = kWRows * kKBytes;
    static constexpr int kABytes = BT * kKBytes;
    static constexpr int kStage = kWBytes + kABytes;
    static constexpr int kBarOffset = STAGES * kStage;
    static constexpr int kBytes = kBarOffset + (2 * STAGES + 1) * 8 + 16 + 1024;  // + alignment slack
    static constexpr uint32_t kTmemCols = BT < 32 ? 32 : BT;
};

__device__ __forceinline__ void record_error(int* err, int code) { atomicCAS(err, 0, code); }

template <int KIND, int BT, int STAGES>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ GemmParams p) {
    using S = Smem<BT, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOffset);
    uint64_t* empty = full + STAGES;
    uint64_t* accum = empty + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // Grouped rasterisation: group_m token tiles advance together so that a
    // wave's weight and activation tiles stay L2-resident.
    const int t = blockIdx.x;
    const int per_group = p.group_m * p.tiles_n;
    const int g = t / per_group;
    const int first_m = g * p.group_m;
    const int gsz = min(p.group_m, p.tiles_m - first_m);
    const int local = t - g * per_group;
    const int tm = first_m + local % gsz;
    const int tn = local / gsz;
    const int n0 = tn * kWRows;
    const int m0 = tm * BT;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        fence_mbar_init();
        prefetch_tmap(&p.tmap_w);
        prefetch_tmap(&p.tmap_a);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, S::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer ----
            int issued = 0;
            for (int kb = 0; kb < p.num_kb; ++kb) {
                const int s = kb % STAGES;
                const uint32_t ph = (kb / STAGES) & 1;
                if (kb >= STAGES && !mbar_wait(&empty[s], ph ^ 1)) {
                    record_error(p.err, kErrTimeoutEmpty);
                    break;
                }
                uint8_t* st = smem + s * S::kStage;
                mbar_arrive_expect_tx(&full[s], S::kStage);
                tma_load_2d(st, &p.tmap_w, &full[s], kb * p.kb_elems, n0);
                tma_load_2d(st + S::kWBytes, &p.tmap_a, &full[s], kb * p.kb_elems, m0);
                issued = kb + 1;
            }
            // Drain: every issued stage's data must have landed before exit.
            for (int kb = max(0, issued - STAGES); kb < issued; ++kb) {
                if (!mbar_wait(&full[kb % STAGES], (kb / STAGES) & 1)) {
                    record_error(p.err, kErrTimeoutDrain);
                    break;
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer ----
            constexpr uint32_t idesc = make_idesc<KIND>(kWRows, BT);
            for (int kb = 0; kb < p.num_kb; ++kb) {
                const int s = kb % STAGES;
                const uint32_t ph = (kb / STAGES) & 1;
                if (!mbar_wait(&full[s], ph)) {
                    record_error(p.err, kErrTimeoutFull);
                    break;
                }
                tc_fence_after();
                const uint32_t wa = smem_u32(smem + s * S::kStage);
                const uint32_t aa = wa + S::kWBytes;
#pragma unroll
                for (int ks = 0; ks < kKBytes / 32; ++ks) {
                    tc_mma<KIND>(tmem_base, smem_desc_k128(wa + ks * 32), smem_desc_k128(aa + ks * 32), idesc,
                                 (kb | ks) != 0);
                }
                tc_commit(&empty[s]);
            }
            tc_commit(accum);
            // Wait for our own MMAs before TMEM can be released.
            if (!mbar_wait(accum, 0)) record_error(p.err, kErrTimeoutDrain);
        }
        __syncwarp();
    } else {
        // ---- epilogue warps 2..5: TMEM lane quarter q = warp % 4 ----
        const int q = warp & 3;
        int ready = 0;
        if (lane == 0) ready = mbar_wait(accum, 0) ? 1 : 0;
        ready = __shfl_sync(0xffffffffu, ready, 0);
        if (!ready) {
            if (lane == 0) record_error(p.err, kErrTimeoutAccum);
        } else {
            tc_fence_after();
            const int col = n0 + q * 32 + lane;  // output column owned by this thread
            const bool col_ok = col < p.n;
            int mi = 0;
#pragma unroll
            for (int i = 1; i < 4; ++i)
                if (i < p.nmembers && col >= p.n_start[i]) mi = i;
            float* out = p.out[mi];
            const long long ldo = p.ldo[mi];
            const int ocol = col - p.n_start[mi];
            float ws = 0.0f;
            if constexpr (KIND == 0) ws = col_ok ? p.w_scale[col] : 0.0f;
#pragma unroll 1
            for (int c = 0; c < BT; c += 16) {
                uint32_t r[16];
                tmem_ld16(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + c, r);
                tmem_ld_wait();
                if (col_ok) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int m = m0 + c + j;
                        if (m < p.m) {
                            float v;
                            if constexpr (KIND == 0) {
                                const int acc = static_cast<int>(r[j]);
                                v = __fmul_rn(__fmul_rn(__int2float_rn(acc), p.a_scale[m]), ws);
                                if (p.acc_out) p.acc_out[static_cast<long long>(m) * p.acc_ld + col] = acc;
                            } else {
                                v = __uint_as_float(r[j]);
                            }
                            out[static_cast<long long>(m) * ldo + ocol] = v;
                        }
                    }
                }
            }
        }
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, S::kTmemCols);
    }
}

// ---- host side -----------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D K-major tile map: rows x k elements, row pitch `ld_bytes`, box of
// (128 bytes of K) x box_rows, 128-byte swizzle, zero fill out of bounds.
bool make_map(CUtensorMap* map, const void* base, int elem_bytes, int k, int rows, long long ld_bytes,
              int box_rows) {
    auto encode = get_encode();
    if (!encode) return false;
    const CUtensorMapDataType dt = elem_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld_bytes)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(kKBytes / elem_bytes), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int KIND, int BT, int STAGES>
int launch_cfg(GemmParams& p, cudaStream_t s) {
    using S = Smem<BT, STAGES>;
    auto kern = gemm_tc_kernel<KIND, BT, STAGES>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes);
    if (e != cudaSuccess) return e;
    p.tiles_m = (p.m + BT - 1) / BT;
    p.group_m = std::min(p.tiles_m, 8);
    const int tiles = p.tiles_m * p.tiles_n;
    kern<<<tiles, kThreads, S::kBytes, s>>>(p);
    return cudaGetLastError();
}

}  // namespace

int sm_count() {
    static int count = 0;
    if (count == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev);
        if (count <= 0) count = 148;
    }
    return count;
}

int launch_gemm_tc(int kind, const void* w, long long ldw_bytes, const void* a, long long lda_bytes, int m, int n,
                   int k, const float* w_scale, const float* a_scale, const OutMembers& outs, int32_t* acc_out,
                   long long acc_ld, int* err, cudaStream_t s) {
    if (m <= 0 || n <= 0 || k <= 0) return cudaErrorInvalidValue;
    if ((ldw_bytes % 16) || (lda_bytes % 16) || (reinterpret_cast<uintptr_t>(w) % 16) ||
        (reinterpret_cast<uintptr_t>(a) % 16))
        return cudaErrorInvalidValue;
    const int eb = kind == 0 ? 1 : 2;
    GemmParams p{};
    p.w_scale = w_scale;
    p.a_scale = a_scale;
    p.m = m;
    p.n = n;
    p.kb_elems = kKBytes / eb;
    p.num_kb = (k + p.kb_elems - 1) / p.kb_elems;
    p.tiles_n = (n + kWRows - 1) / kWRows;
    p.nmembers = outs.count;
    for (int i = 0; i < 5; ++i) p.n_start[i] = outs.n_start[i];
    for (int i = 0; i < 4; ++i) {
        p.out[i] = outs.out[i];
        p.ldo[i] = outs.ldo[i];
    }
    p.acc_out = acc_out;
    p.acc_ld = acc_ld;
    p.err = err;
    const int bt = m <= 16 ? 16 : m <= 32 ? 32 : m <= 64 ? 64 : m <= 128 ? 128 : 256;
    if (!make_map(&p.tmap_w, w, eb, k, n, ldw_bytes, kWRows)) return cudaErrorInvalidValue;
    if (!make_map(&p.tmap_a, a, eb, k, m, lda_bytes, bt)) return cudaErrorInvalidValue;
    if (kind == 0) {
        switch (bt) {
            case 16: return launch_cfg<0, 16, 8>(p, s);
            case 32: return launch_cfg<0, 32, 8>(p, s);
            case 64: return launch_cfg<0, 64, 8>(p, s);
            case 128: return launch_cfg<0, 128, 6>(p, s);
            default: return launch_cfg<0, 256, 4>(p, s);
        }
    }
    switch (bt) {
        case 16: return launch_cfg<1, 16, 8>(p, s);
        case 32: return launch_cfg<1, 32, 8>(p, s);
        case 64: return launch_cfg<1, 64, 8>(p, s);
        case 128: return launch_cfg<1, 128, 6>(p, s);
        default: return launch_cfg<1, 256, 4>(p, s);
    }
}

}  // namespace rk

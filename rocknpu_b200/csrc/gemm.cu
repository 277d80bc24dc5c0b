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
//
// Short prompts leave few output tiles, so the K range can be split over
// `ksplit` CTAs per tile (kind 0 only): each adds its int32 partial into an
// int32 workspace with red.global.add (exact and order-independent, like the
// reference's wrapping K-partial sum, capi/src/lib.rs:1906-1914), and the CTA
// that arrives last on the tile's counter applies the epilogue and returns
// the workspace and counter to zero for the next launch.
//
// Launch: programmatic dependent launch -- the CTA initialises barriers,
// allocates TMEM and streams its first weight stages while the preceding
// kernel (the activation quantiser) finishes; activation loads, scale reads
// and output writes wait on griddepcontrol.wait.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
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
    int ksplit, kb_per_split;
    int nmembers;
    int n_start[5];
    float* out[4];
    long long ldo[4];
    int32_t* acc_out;
    long long acc_ld;
    int32_t* ws;          // split-K partial sums [m][n], all zero between launches
    unsigned* counters;   // split-K arrivals per tile, all zero between launches
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

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void epilogue_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <int KIND>
__device__ __forceinline__ float rescale(uint32_t raw, float a_s, float w_s) {
    if constexpr (KIND == 0)
        return __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(raw)), a_s), w_s);
    else
        return __uint_as_float(raw);
}

__device__ __forceinline__ int member_of(const GemmParams& p, int col) {
    int mi = 0;
#pragma unroll
    for (int i = 1; i < 4; ++i)
        if (i < p.nmembers && col >= p.n_start[i]) mi = i;
    return mi;
}

// Last CTA of a split-K tile: read the summed int32 tile from the workspace
// (vector loads, 8 rows in flight per thread), apply the rescale, write the
// outputs and return the workspace cells and the tile counter to zero.
// `tid` is 0..127 over the four epilogue warps.
template <int BT>
__device__ __forceinline__ void finalize_split(const GemmParams& p, int tile, int m0, int n0, int tid, bool leader) {
    const long long wld = p.n;
    const int mend = min(p.m, m0 + BT);
    const int c0 = n0 + (tid & 31) * 4;  // four consecutive columns
    const int r_first = m0 + (tid >> 5);
    if ((p.n & 3) == 0) {
        if (c0 < p.n) {
            float wsc[4];
            float* optr[4];
            long long oldo[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int col = c0 + j;
                wsc[j] = p.w_scale[col];
                const int mi = member_of(p, col);
                optr[j] = p.out[mi] + (col - p.n_start[mi]);
                oldo[j] = p.ldo[mi];
            }
            for (int rb = r_first; rb < mend; rb += 32) {
                int4 v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int m = rb + 4 * u;
                    if (m < mend) v[u] = __ldcg(reinterpret_cast<const int4*>(p.ws + m * wld + c0));
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int m = rb + 4 * u;
                    if (m < mend) {
                        *reinterpret_cast<int4*>(p.ws + m * wld + c0) = make_int4(0, 0, 0, 0);
                        const float a_s = p.a_scale[m];
                        const int acc[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            optr[j][m * oldo[j]] = __fmul_rn(__fmul_rn(__int2float_rn(acc[j]), a_s), wsc[j]);
                            if (p.acc_out) p.acc_out[m * p.acc_ld + c0 + j] = acc[j];
                        }
                    }
                }
            }
        }
    } else {
        // odd widths: one column per thread, all rows
        const int col = n0 + (tid & 127);
        if (col < p.n && tid < 128) {
            const int mi = member_of(p, col);
            float* o = p.out[mi] + (col - p.n_start[mi]);
            const float wsc = p.w_scale[col];
            for (int m = m0; m < mend; ++m) {
                int32_t* cell = p.ws + m * wld + col;
                const int acc = __ldcg(cell);
                *cell = 0;
                o[m * p.ldo[mi]] = __fmul_rn(__fmul_rn(__int2float_rn(acc), p.a_scale[m]), wsc);
                if (p.acc_out) p.acc_out[m * p.acc_ld + col] = acc;
            }
        }
    }
    if (leader) p.counters[tile] = 0u;
}

template <int KIND, int BT, int STAGES, int MINB>
__global__ void __launch_bounds__(kThreads, MINB) gemm_tc_kernel(const __grid_constant__ GemmParams p) {
    using S = Smem<BT, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOffset);
    uint64_t* empty = full + STAGES;
    uint64_t* accum = empty + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
    uint32_t* last_flag = tmem_slot + 1;

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
    const int kb0 = blockIdx.y * p.kb_per_split;
    const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
    const int nkb = kb1 - kb0;  // >= 1 (the host never launches an empty split)

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
            // Weights do not depend on the preceding kernel: stream the first
            // stages' weight tiles before waiting for it.
            const int pre = min(STAGES, nkb);
            for (int i = 0; i < pre; ++i) {
                mbar_arrive_expect_tx(&full[i], S::kStage);
                tma_load_2d(smem + i * S::kStage, &p.tmap_w, &full[i], (kb0 + i) * p.kb_elems, n0);
            }
            griddep_wait();
            for (int i = 0; i < pre; ++i)
                tma_load_2d(smem + i * S::kStage + S::kWBytes, &p.tmap_a, &full[i], (kb0 + i) * p.kb_elems, m0);
            int issued = pre;
            for (int i = pre; i < nkb; ++i) {
                const int s = i % STAGES;
                const uint32_t ph = (i / STAGES) & 1;
                if (!mbar_wait(&empty[s], ph ^ 1)) {
                    record_error(p.err, kErrTimeoutEmpty);
                    break;
                }
                uint8_t* st = smem + s * S::kStage;
                mbar_arrive_expect_tx(&full[s], S::kStage);
                tma_load_2d(st, &p.tmap_w, &full[s], (kb0 + i) * p.kb_elems, n0);
                tma_load_2d(st + S::kWBytes, &p.tmap_a, &full[s], (kb0 + i) * p.kb_elems, m0);
                issued = i + 1;
            }
            // Drain: every issued stage's data must have landed before exit.
            for (int i = max(0, issued - STAGES); i < issued; ++i) {
                if (!mbar_wait(&full[i % STAGES], (i / STAGES) & 1)) {
                    record_error(p.err, kErrTimeoutDrain);
                    break;
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer ----
            constexpr uint32_t idesc = make_idesc<KIND>(kWRows, BT);
            for (int i = 0; i < nkb; ++i) {
                const int s = i % STAGES;
                const uint32_t ph = (i / STAGES) & 1;
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
                                 (i | ks) != 0);
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
        griddep_wait();
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
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
        if (!ready) {
            if (lane == 0) record_error(p.err, kErrTimeoutAccum);
        } else if (p.ksplit == 1) {
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < BT; c += 16) {
                uint32_t r[16];
                tmem_ld16(lane_base + c, r);
                tmem_ld_wait();
                if (col_ok) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int m = m0 + c + j;
                        if (m < p.m) {
                            float a_s = 0.0f;
                            if constexpr (KIND == 0) a_s = p.a_scale[m];
                            out[static_cast<long long>(m) * ldo + ocol] = rescale<KIND>(r[j], a_s, ws);
                            if constexpr (KIND == 0)
                                if (p.acc_out) p.acc_out[static_cast<long long>(m) * p.acc_ld + col] = r[j];
                        }
                    }
                }
            }
        }
        if (KIND == 0 && p.ksplit > 1) {
            // split-K: add this CTA's partial into the workspace.  Every
            // epilogue warp reaches both named barriers, timed out or not.
            const long long wld = p.n;
            if (ready) {
                tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < BT; c += 16) {
                    uint32_t r[16];
                    tmem_ld16(lane_base + c, r);
                    tmem_ld_wait();
                    if (col_ok) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int m = m0 + c + j;
                            if (m < p.m)
                                atomicAdd(p.ws + static_cast<long long>(m) * wld + col, static_cast<int>(r[j]));
                        }
                    }
                }
            }
            __threadfence();
            epilogue_bar();
            if (warp == 2 && lane == 0) {
                const unsigned prev = atomicAdd(p.counters + t, 1u);
                *last_flag = (prev == static_cast<unsigned>(p.ksplit - 1)) ? 1u : 0u;
            }
            epilogue_bar();
            if (*last_flag) {
                __threadfence();
                finalize_split<BT>(p, t, m0, n0, threadIdx.x - 64, warp == 2 && lane == 0);
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

int current_device() {
    int d = 0;
    cudaGetDevice(&d);
    return d;
}

template <int KIND, int BT, int STAGES, int MINB>
int launch_cfg(GemmParams& p, cudaStream_t s) {
    using S = Smem<BT, STAGES>;
    auto kern = gemm_tc_kernel<KIND, BT, STAGES, MINB>;
    static bool attr_done[64] = {};
    const int dev = current_device();
    if (dev < 0 || dev >= 64 || !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_done[dev] = true;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(p.tiles_m * p.tiles_n), static_cast<unsigned>(p.ksplit), 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = S::kBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

}  // namespace

int sm_count() {
    static int count[64] = {};
    const int dev = current_device();
    if (dev < 0 || dev >= 64) return 148;
    if (count[dev] == 0) {
        int c = 0;
        cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
        count[dev] = c > 0 ? c : 148;
    }
    return count[dev];
}

GemmPlan plan_gemm(int kind, int m, int n, int k) {
    GemmPlan pl;
    const int eb = kind == 0 ? 1 : 2;
    const int num_kb = (k * eb + kKBytes - 1) / kKBytes;
    const int tiles_n = (n + kWRows - 1) / kWRows;
    const int sms = sm_count();
    auto tiles_for = [&](int b) { return tiles_n * ((m + b - 1) / b); };
    // Token tile: the largest of 128/64/32 that still gives every SM a tile
    // (two 96 KB CTAs fit an SM); 256 once tiles are plentiful (large M).
    // Measured on the TinyLlama pp128/pp512 shapes: filling the SMs beats
    // re-reading fewer activation tiles at these sizes.
    int bt = m <= 16 ? 16 : 32;
    for (int b : {128, 64}) {
        if (m > 16 && b < 2 * m && tiles_for(b) >= sms) {
            bt = b;
            break;
        }
    }
    if (bt == 128 && tiles_for(256) >= 4 * sms) bt = 256;
    int tiles = tiles_for(bt);
    // K splits only for long-K shapes that still leave SMs idle: the
    // workspace round trip costs more than it saves on short K.
    int ksplit = 1;
    if (kind == 0 && tiles < sms && k * eb >= 4096) {
        ksplit = (2 * sms + tiles / 2) / tiles;
        ksplit = std::min(ksplit, std::min(8, num_kb / 8));
        ksplit = std::max(ksplit, 1);
    }
    // tuning overrides: ROCKNPU_B200_GEMM_BT (16/32/64/128/256) and
    // ROCKNPU_B200_GEMM_KSPLIT (>= 1); both keep the result bit-identical
    if (const char* v = std::getenv("ROCKNPU_B200_GEMM_BT")) {
        const int b = std::atoi(v);
        if (b == 16 || b == 32 || b == 64 || b == 128 || b == 256) {
            bt = b;
            tiles = tiles_n * ((m + bt - 1) / bt);
        }
    }
    if (const char* v = std::getenv("ROCKNPU_B200_GEMM_KSPLIT")) {
        const int ks = std::atoi(v);
        if (ks >= 1 && kind == 0) ksplit = std::min(ks, std::max(1, num_kb));
    }
    const int per = (num_kb + ksplit - 1) / ksplit;
    ksplit = (num_kb + per - 1) / per;  // no empty split
    pl.bt = bt;
    pl.ksplit = ksplit;
    pl.kb_per_split = per;
    pl.tiles = tiles;
    pl.ws_elems = ksplit > 1 ? static_cast<size_t>(m) * n : 0;
    pl.counter_elems = ksplit > 1 ? static_cast<size_t>(tiles) : 0;
    return pl;
}

int launch_gemm_tc(int kind, const void* w, long long ldw_bytes, const void* a, long long lda_bytes, int m, int n,
                   int k, const float* w_scale, const float* a_scale, const OutMembers& outs, int32_t* acc_out,
                   long long acc_ld, int* err, cudaStream_t s, const GemmWorkspace* ws) {
    if (m <= 0 || n <= 0 || k <= 0) return cudaErrorInvalidValue;
    if ((ldw_bytes % 16) || (lda_bytes % 16) || (reinterpret_cast<uintptr_t>(w) % 16) ||
        (reinterpret_cast<uintptr_t>(a) % 16))
        return cudaErrorInvalidValue;
    const int eb = kind == 0 ? 1 : 2;
    GemmPlan pl = plan_gemm(kind, m, n, k);
    if (pl.ksplit > 1 && (ws == nullptr || ws->ws == nullptr || ws->counters == nullptr ||
                          ws->ws_elems < pl.ws_elems || ws->counter_elems < pl.counter_elems)) {
        // no (large enough) workspace: one CTA per tile over the whole K
        pl.ksplit = 1;
        pl.kb_per_split = (k * eb + kKBytes - 1) / kKBytes;
    }
    GemmParams p{};
    p.w_scale = w_scale;
    p.a_scale = a_scale;
    p.m = m;
    p.n = n;
    p.kb_elems = kKBytes / eb;
    p.num_kb = (k + p.kb_elems - 1) / p.kb_elems;
    p.tiles_n = (n + kWRows - 1) / kWRows;
    p.tiles_m = (m + pl.bt - 1) / pl.bt;
    p.group_m = std::min(p.tiles_m, 8);
    p.ksplit = pl.ksplit;
    p.kb_per_split = pl.kb_per_split;
    p.nmembers = outs.count;
    for (int i = 0; i < 5; ++i) p.n_start[i] = outs.n_start[i];
    for (int i = 0; i < 4; ++i) {
        p.out[i] = outs.out[i];
        p.ldo[i] = outs.ldo[i];
    }
    p.acc_out = acc_out;
    p.acc_ld = acc_ld;
    p.ws = pl.ksplit > 1 ? ws->ws : nullptr;
    p.counters = pl.ksplit > 1 ? ws->counters : nullptr;
    p.err = err;
    if (!make_map(&p.tmap_w, w, eb, k, n, ldw_bytes, kWRows)) return cudaErrorInvalidValue;
    if (!make_map(&p.tmap_a, a, eb, k, m, lda_bytes, pl.bt)) return cudaErrorInvalidValue;
    if (kind == 0) {
        switch (pl.bt) {
            case 16: return launch_cfg<0, 16, 6, 2>(p, s);
            case 32: return launch_cfg<0, 32, 5, 2>(p, s);
            case 64: return launch_cfg<0, 64, 4, 2>(p, s);
            case 128: return launch_cfg<0, 128, 3, 2>(p, s);
            default: return launch_cfg<0, 256, 4, 1>(p, s);
        }
    }
    switch (pl.bt) {
        case 16: return launch_cfg<1, 16, 6, 2>(p, s);
        case 32: return launch_cfg<1, 32, 5, 2>(p, s);
        case 64: return launch_cfg<1, 64, 4, 2>(p, s);
        case 128: return launch_cfg<1, 128, 3, 2>(p, s);
        default: return launch_cfg<1, 256, 4, 1>(p, s);
    }
}

}  // namespace rk

// K3 (W8A8 prefill GEMM) and K4 (FP16 executor GEMM) on the 5th-generation
// tensor cores.
//
// Orientation ("swap AB"): the MMA's M side is weight rows (output columns),
// its N side a tile of BT tokens, so short prompts (BT = 16..64) waste no
// tensor-core rows.  A tile is WT = 128 or 256 weight rows: 256-row tiles
// issue two M=128 MMAs per K step into two TMEM accumulators.  A pipeline
// stage holds KA = 1 or 2 K atoms of 128 bytes, so every barrier wait of the
// MMA thread feeds about 500 tensor-core cycles (one tcgen05.mma with M=128
// costs at least ~55 cycles whatever N is; the thread's wait, commit and loop
// cost ~150 more per stage).  Accumulators are int32 (kind::i8) or f32 (kind::f16); lane =
// weight row, column = token, so each epilogue warp stores 32 consecutive
// output columns (a coalesced 128-byte line) per token.
//
// Persistent: one CTA per SM walks a static list of (tile, K split) units.
// Warp roles:
//   warp 0      weight producer: one TMA box (WT x 128 B, 128-byte swizzle,
//               no multicast) per stage;
//   warp 1      activation producer: one TMA box (BT x 128 B) per stage;
//   warp 2      owns TMEM (double-buffered accumulators) and issues the
//               tcgen05.mma instructions from one thread;
//   warps 3-10  epilogue: TMEM -> registers -> global, overlapped with the
//               next unit's main loop.
//
// Epilogue: kind 0  out[m, n] = (f32(acc) * a_scale[m]) * w_scale[n]
//           (rescale_i32_row's order, capi/src/lib.rs:692-709), optional raw
//           int32 dump; kind 1  out[m, n] = acc.
//
// Split K (kind 0): units of one tile add their int32 partials into a
// workspace with red.global.add -- exact and order-independent, like the
// reference's wrapping K-partial sum (capi/src/lib.rs:1906-1914) -- and the
// unit arriving last on the tile's counter applies the epilogue and returns
// the workspace cells and the counter to zero.
//
// Launch: programmatic dependent launch.  The weight producer streams from
// the start; the activation producer and the epilogue wait on
// griddepcontrol.wait for the preceding kernel (the activation quantiser).
//
// Every wait is bounded (2 s).  A wait that runs out records an error code
// in *err and raises a CTA-wide abort flag; the other roles then stop
// waiting, the producers wait (bounded) for their own copies in flight, the
// MMA thread for its own MMAs, and TMEM is freed before the CTA exits.
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

constexpr int kKBytes = 128;  // K bytes per stage (one swizzle row)
constexpr int kEpiWarps = 8;
constexpr int kThreads = (3 + kEpiWarps) * 32;

struct GemmParams {
    CUtensorMap tmap_w;  // [n rows][k] K-major, box WT rows
    CUtensorMap tmap_a;  // [m rows][k] K-major, box BT rows
    const float* w_scale;
    const float* a_scale;
    int m, n, num_kb, kb_elems;
    int tiles_n, tiles_m, group_m;
    int units, ksplit, kb_per_split;
    int nmembers;
    int n_start[5];
    float* out[4];
    long long ldo[4];
    int copies;                   // > 1: elements go to every copy_out[c] instead
    float* copy_out[kMaxCopies];  // at out[0]'s offsets (peer all-gather)
    int32_t* acc_out;
    long long acc_ld;
    int32_t* ws;         // split-K partial sums [m][n], all zero between launches
    unsigned* counters;  // split-K arrivals per tile, all zero between launches
    int* err;
};

template <int WT, int BT, int KA, int STAGES>
struct Cfg {
    static constexpr int kAcc = WT / 128;  // accumulators per tile
    static constexpr int kWBox = WT * kKBytes;  // one K atom of the weight tile
    static constexpr int kABox = BT * kKBytes;  // one K atom of the token tile
    static constexpr int kWBytes = KA * kWBox;
    static constexpr int kABytes = KA * kABox;
    static constexpr int kStage = kWBytes + kABytes;
    static constexpr int kBarOffset = STAGES * kStage;
    static constexpr int kNumBars = 2 * STAGES + 5;
    static constexpr int kBytes = kBarOffset + kNumBars * 8 + 32 + 1024;  // + alignment slack
    static constexpr uint32_t kTmemCols = 2 * kAcc * BT < 32 ? 32 : 2 * kAcc * BT;
    static_assert((kTmemCols & (kTmemCols - 1)) == 0 && kTmemCols <= 512, "TMEM allocation");
    static_assert(kBytes <= 232448, "shared memory");
};

struct Shared {
    uint64_t* full;  // two arrivals per phase: weight and activation producer
    uint64_t* empty;
    uint64_t* tfull;   // [2]
    uint64_t* tempty;  // [2]
    uint64_t* drain;
    uint32_t* tmem_slot;
    uint32_t* last_flag;
    volatile uint32_t* abort;
};

__device__ __forceinline__ void fail(const GemmParams& p, const Shared& sh, int code) {
    atomicCAS(p.err, 0, code);
    *sh.abort = 1u;
}

// Bounded wait that also gives up once another role has aborted.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile uint32_t* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
#pragma unroll 1
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void epilogue_bar() {
    asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
}

__device__ __forceinline__ int member_of(const GemmParams& p, int col) {
    int mi = 0;
#pragma unroll
    for (int i = 1; i < 4; ++i)
        if (i < p.nmembers && col >= p.n_start[i]) mi = i;
    return mi;
}

// Unit u -> tile coordinates and K range.  Grouped rasterisation: group_m
// token tiles advance together so a wave's weight and activation tiles stay
// L2-resident.
struct Unit {
    int tile, n0, m0, kb0, kb1;
};

template <int WT, int BT>
__device__ __forceinline__ Unit unit_coords(const GemmParams& p, int u) {
    Unit r;
    r.tile = u / p.ksplit;
    const int split = u - r.tile * p.ksplit;
    const int per_group = p.group_m * p.tiles_n;
    const int g = r.tile / per_group;
    const int first_m = g * p.group_m;
    const int gsz = min(p.group_m, p.tiles_m - first_m);
    const int local = r.tile - g * per_group;
    r.m0 = (first_m + local % gsz) * BT;
    r.n0 = (local / gsz) * WT;
    r.kb0 = split * p.kb_per_split;
    r.kb1 = min(p.num_kb, r.kb0 + p.kb_per_split);
    return r;
}

// Last unit of a split-K tile: read the summed int32 tile from the
// workspace (vector loads, several rows in flight per thread), rescale,
// write the outputs, and return the cells and the tile counter to zero.
template <int WT, int BT>
__device__ __forceinline__ void finalize_split(const GemmParams& p, const Unit& u, int tid, bool leader) {
    constexpr int kGroups = WT / 4;                       // 4-column groups per tile
    constexpr int kRowStep = (kEpiWarps * 32) / kGroups;  // rows handled in parallel
    const long long wld = p.n;
    const int mend = min(p.m, u.m0 + BT);
    const int c0 = u.n0 + (tid % kGroups) * 4;
    const int r0 = u.m0 + tid / kGroups;
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
            for (int rb = r0; rb < mend; rb += 4 * kRowStep) {
                int4 v[4];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const int m = rb + t * kRowStep;
                    if (m < mend) v[t] = __ldcg(reinterpret_cast<const int4*>(p.ws + m * wld + c0));
                }
                float a_sv[4];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const int m = rb + t * kRowStep;
                    a_sv[t] = m < mend ? __ldg(p.a_scale + m) : 0.0f;
                }
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const int m = rb + t * kRowStep;
                    if (m < mend) {
                        *reinterpret_cast<int4*>(p.ws + m * wld + c0) = make_int4(0, 0, 0, 0);
                        const float a_s = a_sv[t];
                        const int acc[4] = {v[t].x, v[t].y, v[t].z, v[t].w};
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
        // odd widths: one cell per thread per step
        for (int idx = tid; idx < WT * BT; idx += kEpiWarps * 32) {
            const int col = u.n0 + idx % WT;
            const int m = u.m0 + idx / WT;
            if (col < p.n && m < mend) {
                const int mi = member_of(p, col);
                int32_t* cell = p.ws + m * wld + col;
                const int acc = __ldcg(cell);
                *cell = 0;
                p.out[mi][m * p.ldo[mi] + (col - p.n_start[mi])] =
                    __fmul_rn(__fmul_rn(__int2float_rn(acc), p.a_scale[m]), p.w_scale[col]);
                if (p.acc_out) p.acc_out[m * p.acc_ld + col] = acc;
            }
        }
    }
    if (leader) p.counters[u.tile] = 0u;
}

template <int KIND, int WT, int BT, int KA, int STAGES>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ GemmParams p) {
    using C = Cfg<WT, BT, KA, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
    Shared sh;
    sh.full = bars;
    sh.empty = bars + STAGES;
    sh.tfull = bars + 2 * STAGES;
    sh.tempty = sh.tfull + 2;
    sh.drain = sh.tempty + 2;
    sh.tmem_slot = reinterpret_cast<uint32_t*>(sh.drain + 1);
    sh.last_flag = sh.tmem_slot + 1;
    sh.abort = sh.tmem_slot + 2;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&sh.full[s], 2);
            mbar_init(&sh.empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&sh.tfull[b], 1);
            mbar_init(&sh.tempty[b], kEpiWarps);
        }
        mbar_init(sh.drain, 1);
        *sh.abort = 0u;
        fence_mbar_init();
        prefetch_tmap(&p.tmap_w);
        prefetch_tmap(&p.tmap_a);
    }
    if (warp == 2) {
        tmem_alloc(sh.tmem_slot, C::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *sh.tmem_slot;

    if (warp == 0 || warp == 1) {
        if (lane == 0) {
            // ---- producers: warp 0 weights, warp 1 activations ----
            const bool is_w = warp == 0;
            const CUtensorMap* map = is_w ? &p.tmap_w : &p.tmap_a;
            const uint32_t box = is_w ? C::kWBox : C::kABox;
            const int off = is_w ? 0 : C::kWBytes;
            if (!is_w) griddep_wait();
            int g = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
                const Unit t = unit_coords<WT, BT>(p, u);
                const int row = is_w ? t.n0 : t.m0;
                for (int kb = t.kb0; kb < t.kb1; kb += KA, ++g) {
                    const int s = g % STAGES;
                    const uint32_t ph = (g / STAGES) & 1;
                    if (g >= STAGES && !wait_or_abort(&sh.empty[s], ph ^ 1, sh.abort)) {
                        if (!*sh.abort) fail(p, sh, kErrTimeoutEmpty);
                        ok = false;
                        break;
                    }
                    const int na = min(KA, t.kb1 - kb);  // K atoms in this stage
                    mbar_arrive_expect_tx(&sh.full[s], na * box);
                    for (int a = 0; a < na; ++a)
                        tma_load_2d(smem + s * C::kStage + off + a * box, map, &sh.full[s], (kb + a) * p.kb_elems, row);
                }
            }
            // our copies in flight must land before the CTA exits: wait for
            // the stage's phase, or give up after the limit (the other
            // producer's arrival is part of the phase)
            for (int i = max(0, g - STAGES); i < g; ++i) {
                if (!mbar_wait(&sh.full[i % STAGES], (i / STAGES) & 1)) {
                    atomicCAS(p.err, 0, kErrTimeoutDrain);
                    break;
                }
            }
        }
    } else if (warp == 2) {
        if (lane == 0) {
            // ---- MMA issuer ----
            constexpr uint32_t idesc = make_idesc<KIND>(128, BT);
            int g = 0, j = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++j) {
                const Unit t = unit_coords<WT, BT>(p, u);
                const int buf = j & 1, use = j >> 1;
                if (use >= 1 && !wait_or_abort(&sh.tempty[buf], (use - 1) & 1, sh.abort)) {
                    if (!*sh.abort) fail(p, sh, kErrTimeoutAccum);
                    break;
                }
                tc_fence_after();
                const uint32_t d0 = tmem_base + static_cast<uint32_t>(buf * C::kAcc * BT);
                for (int kb = t.kb0; kb < t.kb1; kb += KA, ++g) {
                    const int s = g % STAGES;
                    const uint32_t ph = (g / STAGES) & 1;
                    if (!wait_or_abort(&sh.full[s], ph, sh.abort)) {
                        if (!*sh.abort) fail(p, sh, kErrTimeoutFull);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const int na = min(KA, t.kb1 - kb);
                    const uint32_t wa = smem_u32(smem + s * C::kStage);
                    const uint32_t aa = wa + C::kWBytes;
#pragma unroll
                    for (int a = 0; a < KA; ++a) {
                        if (a < na) {
#pragma unroll
                            for (int ks = 0; ks < kKBytes / 32; ++ks) {
#pragma unroll
                                for (int acc = 0; acc < C::kAcc; ++acc)
                                    tc_mma<KIND>(d0 + acc * BT,
                                                 smem_desc_k128(wa + a * C::kWBox + acc * 128 * kKBytes + ks * 32),
                                                 smem_desc_k128(aa + a * C::kABox + ks * 32), idesc,
                                                 (kb != t.kb0 || a != 0 || ks != 0) ? 1u : 0u);
                            }
                        }
                    }
                    tc_commit(&sh.empty[s]);
                }
                if (ok) tc_commit(&sh.tfull[buf]);
            }
            // our MMAs must finish before TMEM is released
            tc_commit(sh.drain);
            if (!mbar_wait(sh.drain, 0)) atomicCAS(p.err, 0, kErrTimeoutDrain);
        }
        __syncwarp();
    } else {
        // ---- epilogue warps 3..10 ----
        const int e = warp - 3;
        const int q = warp & 3;   // TMEM lane quarter this warp may access
        const int half = e >> 2;  // 0 or 1
        const int etid = threadIdx.x - 96;
        bool waited_dep = false;
        int j = 0;
        for (int u = blockIdx.x; u < p.units; u += gridDim.x, ++j) {
            const Unit t = unit_coords<WT, BT>(p, u);
            const int buf = j & 1, use = j >> 1;
            int ready = 0;
            if (lane == 0) ready = wait_or_abort(&sh.tfull[buf], use & 1, sh.abort) ? 1 : 0;
            ready = __shfl_sync(0xffffffffu, ready, 0);
            if (!ready && lane == 0 && !*sh.abort) fail(p, sh, kErrTimeoutAccum);
            if (!waited_dep) {
                griddep_wait();
                waited_dep = true;
            }
            // accumulator and output column this thread handles
            const int acc = C::kAcc == 2 ? half : 0;
            const int col = t.n0 + acc * 128 + q * 32 + lane;
            const bool col_ok = col < p.n;
            const int mi = member_of(p, col);
            float* out = p.out[mi];
            const long long ldo = p.ldo[mi];
            const int ocol = col - p.n_start[mi];
            float wsc = 0.0f;
            if constexpr (KIND == 0) wsc = col_ok ? p.w_scale[col] : 0.0f;
            const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                       static_cast<uint32_t>((buf * C::kAcc + acc) * BT);
            // with one accumulator the two halves split the token columns
            const int c_first = C::kAcc == 2 ? 0 : half * 16;
            const int c_step = C::kAcc == 2 ? 16 : 32;
            const bool split = KIND == 0 && p.ksplit > 1;
            if (ready) {
                tc_fence_after();
                const float* __restrict__ a_scale = p.a_scale;
                int32_t* __restrict__ acc_out = p.acc_out;
                int32_t* __restrict__ wsp = p.ws;
#pragma unroll 1
                for (int c = c_first; c < BT; c += c_step) {
                    // the chunk's token scales, loaded before any store of
                    // the chunk (stores could otherwise order every load)
                    float asv[16];
                    if constexpr (KIND == 0) {
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj) {
                            const int m = t.m0 + c + jj;
                            asv[jj] = (!split && m < p.m) ? __ldg(a_scale + m) : 0.0f;
                        }
                    }
                    uint32_t r[16];
                    tmem_ld16(lane_base + c, r);
                    tmem_ld_wait();
                    if (col_ok) {
                        float* __restrict__ o = out + static_cast<long long>(t.m0 + c) * ldo + ocol;
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj) {
                            const int m = t.m0 + c + jj;
                            if (m < p.m) {
                                if constexpr (KIND == 0) {
                                    if (split) {
                                        atomicAdd(wsp + static_cast<long long>(m) * p.n + col, static_cast<int>(r[jj]));
                                    } else {
                                        const float v =
                                            __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[jj])), asv[jj]), wsc);
                                        if (p.copies > 1) {
                                            const long long off = static_cast<long long>(m) * ldo + ocol;
#pragma unroll 1
                                            for (int cp = 0; cp < p.copies; ++cp) p.copy_out[cp][off] = v;
                                        } else {
                                            o[jj * ldo] = v;
                                        }
                                        if (acc_out) acc_out[static_cast<long long>(m) * p.acc_ld + col] = r[jj];
                                    }
                                } else if (p.copies > 1) {
                                    const long long off = static_cast<long long>(m) * ldo + ocol;
#pragma unroll 1
                                    for (int cp = 0; cp < p.copies; ++cp) p.copy_out[cp][off] = __uint_as_float(r[jj]);
                                } else {
                                    o[jj * ldo] = __uint_as_float(r[jj]);
                                }
                            }
                        }
                    }
                }
            }
            // the TMEM buffer is free for the next unit's MMAs
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.tempty[buf]);
            if (split) {
                __threadfence();
                epilogue_bar();
                if (etid == 0) {
                    const unsigned prev = atomicAdd(p.counters + t.tile, 1u);
                    *sh.last_flag = (prev == static_cast<unsigned>(p.ksplit - 1)) ? 1u : 0u;
                }
                epilogue_bar();
                if (*sh.last_flag) {
                    __threadfence();
                    finalize_split<WT, BT>(p, t, etid, etid == 0);
                }
            }
        }
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::kTmemCols);
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

template <int KIND, int WT, int BT, int KA, int STAGES>
int launch_cfg(GemmParams& p, int grid, cudaStream_t s) {
    using C = Cfg<WT, BT, KA, STAGES>;
    auto kern = gemm_tc_kernel<KIND, WT, BT, KA, STAGES>;
    static bool attr_done[64] = {};
    const int dev = current_device();
    if (dev < 0 || dev >= 64 || !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kBytes);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_done[dev] = true;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

// The instantiated tile configurations: (WT, BT, K atoms per stage,
// stages), each about 200 KB of shared memory.
template <int KIND>
int launch_kind(const GemmPlan& pl, GemmParams& p, cudaStream_t s) {
    const int grid = std::min(p.units, sm_count());
    if (pl.wt == 256) {
        switch (pl.bt) {
            case 16: return launch_cfg<KIND, 256, 16, 1, 6>(p, grid, s);
            case 32: return launch_cfg<KIND, 256, 32, 1, 5>(p, grid, s);
            case 64: return launch_cfg<KIND, 256, 64, 1, 5>(p, grid, s);
            default: return launch_cfg<KIND, 256, 128, 1, 4>(p, grid, s);
        }
    }
    switch (pl.bt) {
        case 16: return launch_cfg<KIND, 128, 16, 2, 5>(p, grid, s);
        case 32: return launch_cfg<KIND, 128, 32, 2, 5>(p, grid, s);
        case 64: return launch_cfg<KIND, 128, 64, 2, 4>(p, grid, s);
        case 128: return launch_cfg<KIND, 128, 128, 2, 3>(p, grid, s);
        default: return launch_cfg<KIND, 128, 256, 1, 4>(p, grid, s);
    }
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

// K atoms per pipeline stage of a tile configuration (matches launch_kind).
int k_atoms(int wt, int bt) { return (wt == 128 && bt <= 128) ? 2 : 1; }

// Tile plan.  Cost model, measured on B200: a stage costs the larger of
//  - the MMA thread's work: an M=128 tcgen05.mma takes max(55, N/2) cycles
//    (a 256-row tile issues two per K step, ~15% dearer than one MMA of twice
//    the N) plus ~150 cycles of barrier wait, commit and loop per stage, and
//  - the stage's bytes over the L2 -> SM bandwidth when every SM streams,
//    ~60 bytes per cycle per SM (about 17 TB/s on 148 SMs).
// A persistent CTA runs ceil(units / SMs) units of ceil(K atoms / KA)
// stages; the estimate is the larger of that and the HBM time of the unique
// bytes.  Ties prefer more units (more SMs streaming), then the earlier
// option.  K is split only for long-K shapes that would leave most SMs idle.
GemmPlan plan_gemm(int kind, int m, int n, int k) {
    GemmPlan pl;
    const int eb = kind == 0 ? 1 : 2;
    const int num_kb = (k * eb + kKBytes - 1) / kKBytes;
    const int sms = sm_count();
    struct Opt {
        int wt, bt;
    };
    static const Opt opts[] = {{128, 256}, {256, 128}, {128, 128}, {256, 64}, {128, 64},
                               {256, 32},  {128, 32},  {256, 16},  {128, 16}};
    const double hbm_us = (static_cast<double>(n) * k * eb + static_cast<double>(m) * k * eb + 4.0 * m * n) / 6.5e6;
    double best = 1e30;
    int best_units = 0;
    for (const Opt& o : opts) {
        if (o.bt > 16 && o.bt >= 2 * m) continue;  // mostly empty token tiles
        const int ka = k_atoms(o.wt, o.bt);
        const int units = ((n + o.wt - 1) / o.wt) * ((m + o.bt - 1) / o.bt);
        const double mma_cyc = 4.0 * ka * (o.wt / 128) * std::max(55.0, o.bt / 2.0) * (o.wt == 256 ? 1.15 : 1.0);
        const double l2_cyc = ka * (o.wt + o.bt) * static_cast<double>(kKBytes) / 60.0;
        const double stage_cyc = std::max(mma_cyc + 150.0, l2_cyc);
        const double unit_cyc = ((num_kb + ka - 1) / ka) * stage_cyc;
        const double est = std::max(((units + sms - 1) / sms) * unit_cyc / 1900.0 + 1.0, hbm_us);
        if (est < best * 0.999 || (est < best * 1.001 && units > best_units)) {
            best = est;
            best_units = units;
            pl.wt = o.wt;
            pl.bt = o.bt;
        }
    }
    // tuning overrides, result bit-identical: ROCKNPU_B200_GEMM_WT (128/256),
    // ROCKNPU_B200_GEMM_BT (16..256), ROCKNPU_B200_GEMM_KSPLIT (>= 1)
    if (const char* v = std::getenv("ROCKNPU_B200_GEMM_WT")) {
        const int w = std::atoi(v);
        if (w == 128 || w == 256) pl.wt = w;
    }
    if (const char* v = std::getenv("ROCKNPU_B200_GEMM_BT")) {
        const int b = std::atoi(v);
        if (b == 16 || b == 32 || b == 64 || b == 128 || b == 256) pl.bt = b;
    }
    if (pl.wt == 256 && pl.bt > 128) pl.bt = 128;  // TMEM holds 2 x 2 x 128 columns
    const int ka = k_atoms(pl.wt, pl.bt);
    const int tiles = ((n + pl.wt - 1) / pl.wt) * ((m + pl.bt - 1) / pl.bt);
    int ksplit = 1;
    if (kind == 0 && 2 * tiles <= sms && k * eb >= 4096) {
        ksplit = sms / tiles;
        ksplit = std::min(ksplit, std::min(8, num_kb / 8));
        ksplit = std::max(ksplit, 1);
    }
    if (const char* v = std::getenv("ROCKNPU_B200_GEMM_KSPLIT")) {
        const int ks = std::atoi(v);
        if (ks >= 1 && kind == 0) ksplit = std::min(ks, std::max(1, num_kb));
    }
    // splits cover whole stages (a multiple of the K atoms per stage)
    int per = (num_kb + ksplit - 1) / ksplit;
    per = (per + ka - 1) / ka * ka;
    ksplit = (num_kb + per - 1) / per;  // no empty split
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
    if (outs.copies < 1 || outs.copies > kMaxCopies || (outs.copies > 1 && outs.count != 1))
        return cudaErrorInvalidValue;
    GemmPlan pl = plan_gemm(kind, m, n, k);
    if (pl.ksplit > 1 && (outs.copies > 1 || ws == nullptr || ws->ws == nullptr || ws->counters == nullptr ||
                          ws->ws_elems < pl.ws_elems || ws->counter_elems < pl.counter_elems)) {
        // no (large enough) workspace: one unit per tile over the whole K
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
    p.tiles_n = (n + pl.wt - 1) / pl.wt;
    p.tiles_m = (m + pl.bt - 1) / pl.bt;
    p.group_m = std::min(p.tiles_m, 8);
    if (const char* v = std::getenv("ROCKNPU_B200_GEMM_GROUP")) {
        const int gm = std::atoi(v);
        if (gm >= 1) p.group_m = std::min(p.tiles_m, gm);
    }
    p.ksplit = pl.ksplit;
    p.kb_per_split = pl.kb_per_split;
    p.units = p.tiles_n * p.tiles_m * p.ksplit;
    p.nmembers = outs.count;
    for (int i = 0; i < 5; ++i) p.n_start[i] = outs.n_start[i];
    for (int i = 0; i < 4; ++i) {
        p.out[i] = outs.out[i];
        p.ldo[i] = outs.ldo[i];
    }
    p.copies = outs.copies;
    for (int i = 0; i < kMaxCopies; ++i) p.copy_out[i] = i < outs.copies ? outs.copy_out[i] : nullptr;
    p.acc_out = acc_out;
    p.acc_ld = acc_ld;
    p.ws = pl.ksplit > 1 ? ws->ws : nullptr;
    p.counters = pl.ksplit > 1 ? ws->counters : nullptr;
    p.err = err;
    if (!make_map(&p.tmap_w, w, eb, k, n, ldw_bytes, pl.wt)) return cudaErrorInvalidValue;
    if (!make_map(&p.tmap_a, a, eb, k, m, lda_bytes, pl.bt)) return cudaErrorInvalidValue;
    return kind == 0 ? launch_kind<0>(pl, p, s) : launch_kind<1>(pl, p, s);
}

}  // namespace rk

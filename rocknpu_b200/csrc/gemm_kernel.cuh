// The tcgen05 GEMM kernel behind K3 (W8A8) and K4 (FP16): device code and
// launch templates, included by one translation unit per launch mode
// (gemm_plain.cu, gemm_fused.cu, gemm_gather.cu) so that each mode compiles
// only its own epilogue and prologue.  Host-side planning and tensor maps
// are in gemm.cu; the design notes are at the top of gemm.cu.
#pragma once

#include <cuda.h>

#include <algorithm>

#include "kernels.h"
#include "ptx.cuh"
#include "quant_math.cuh"

namespace rk {
namespace gemm_detail {

constexpr int kKBytes = 128;  // K bytes per stage atom (one swizzle row)
constexpr int kEpiWarps = 8;
constexpr int kThreads = (3 + kEpiWarps) * 32;
constexpr int kQuantSeg = 2048;  // fused quantiser: floats of a row one warp holds

// Launch modes (compile-time):
//   kPlain   int8 (or f16) activations from memory; one or up to four
//            concatenated output members;
//   kFused   W8A8 with the per-token quantiser in the prologue (f32 in);
//   kGather  W8A8 whose epilogue stores every element into `copies` output
//            buffers (the peer all-gather of an N-sharded GEMM).
enum Mode : int { kPlain = 0, kFused = 1, kGather = 2 };

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
    int copies;                   // kGather: output buffers
    float* copy_out[kMaxCopies];  // kGather: at out[0]'s offsets
    int32_t* acc_out;
    long long acc_ld;
    int32_t* ws;         // split-K partial sums [m][n], all zero between launches
    unsigned* counters;  // split-K arrivals per tile, all zero between launches
    int* err;
    int store_guard;  // OutMembers::store_guard
    // kFused
    const float* q_a;
    long long q_lda;
    int q_k;
    int8_t* q_a8;
    long long q_ld8;
    float* q_scale;
    unsigned* q_ready;  // [tiles_m] rows published per token tile
    unsigned* q_exit;   // CTAs finished (the last one re-zeroes the counters)
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
    // per epilogue warp, the token scales of its current unit
    static constexpr int kScaleOffset = (kBarOffset + kNumBars * 8 + 32 + 15) & ~15;  // 16-byte aligned
    static constexpr int kBytes = kScaleOffset + kEpiWarps * BT * 4 + 1024;  // + alignment slack
    // accumulator buffers: two (the epilogue of one unit overlaps the next
    // unit's MMAs) when they fit TMEM's 512 columns, else one (256 x 256)
    static constexpr int kBufs = 2 * kAcc * BT <= 512 ? 2 : 1;
    static constexpr uint32_t kTmemCols = kBufs * kAcc * BT < 32 ? 32 : kBufs * kAcc * BT;
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
    float* red;  // [kEpiWarps] cross-warp maxima of the fused quantiser
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

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Bounded wait until *counter >= need (another role's abort also ends it).
__device__ __forceinline__ bool wait_count(const unsigned* counter, unsigned need, volatile uint32_t* abort) {
    if (ld_acquire_gpu(counter) >= need) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        __nanosleep(64);
        if (ld_acquire_gpu(counter) >= need) return true;
        if (*abort) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}

__device__ __forceinline__ void epilogue_bar() {
    asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
}

// Fused K2 in the prologue (quantize_symmetric_into, capi/src/lib.rs:614-654):
// the epilogue warps of every CTA quantise token rows before their first
// tile.  A row is held in registers by ceil(k / 2048) warps (64 floats per
// lane, all loads in flight at once); its absmax is a warp-shuffle reduction
// then a max over the row's warps through shared memory; scale = absmax / 127
// (1 for an all-zero row); q = round(x / scale) clamped to +-127 through the
// same quant_math.cuh functions as quant_rows_kernel, so the same bits.  Each
// pass quantises gridDim.x * (8 / warps-per-row) rows; after a pass every row
// is published on its token tile's counter.  The async-proxy fence orders the generic int8
// stores before the TMA reads that follow the counter's acquire in the
// activation producer.  Requires k % 16 == 0, k <= 16384 and 16-byte
// aligned rows (checked on the host).
template <int BT>
__device__ __forceinline__ void fused_quant(const GemmParams& p, const Shared& sh, int e, int lane) {
    const int k = p.q_k;
    const int wpr = (k + kQuantSeg - 1) / kQuantSeg;
    const int rpc = kEpiWarps / wpr;
    const int row_in = e / wpr, seg = e - (e / wpr) * wpr;
    const int per_pass = gridDim.x * rpc;
    const int passes = (p.m + per_pass - 1) / per_pass;
    const int s0 = seg * kQuantSeg;
    for (int pass = 0; pass < passes; ++pass) {
        const int r = pass * per_pass + blockIdx.x * rpc + row_in;
        const bool has_row = row_in < rpc && r < p.m;
        float4 v[16];
        float amax = 0.0f;
        bool finite = true;
        if (has_row) {
            const float* __restrict__ src = p.q_a + static_cast<long long>(r) * p.q_lda;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int idx = s0 + j * 128 + lane * 4;
                v[j] = idx < k ? __ldg(reinterpret_cast<const float4*>(src + idx)) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                finite &= isfinite(v[j].x) && isfinite(v[j].y) && isfinite(v[j].z) && isfinite(v[j].w);
                amax = fmaxf(fmaxf(amax, fmaxf(fabsf(v[j].x), fabsf(v[j].y))), fmaxf(fabsf(v[j].z), fabsf(v[j].w)));
            }
        }
        amax = warp_max(amax);
        const bool bad = __any_sync(0xffffffffu, !finite);
        if (lane == 0) sh.red[e] = amax;
        epilogue_bar();
        if (has_row) {
            float rmax = 0.0f;
            for (int w = 0; w < wpr; ++w) rmax = fmaxf(rmax, sh.red[row_in * wpr + w]);
            const float scale = row_scale(rmax);
            const float inv = row_inv(scale);
            if (bad && lane == 0) atomicExch(p.err, kErrNonFinite);
            int8_t* dst = p.q_a8 + static_cast<long long>(r) * p.q_ld8;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int idx = s0 + j * 128 + lane * 4;
                if (idx < k) *reinterpret_cast<uint32_t*>(dst + idx) = quant_pack4(v[j], scale, inv);
            }
            if (seg == 0 && lane == 0) p.q_scale[r] = scale;
            asm volatile("fence.proxy.async.global;" ::: "memory");
        }
        epilogue_bar();  // the pass's rows are stored; red[] is free again
        // the release is cumulative over the row's stores by the other
        // threads, which the barrier ordered before it
        if (has_row && seg == 0 && lane == 0)
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.q_ready + r / BT) : "memory");
    }
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

template <int MODE>
__device__ __forceinline__ float load_scale(const float* p) {
    // scales written by this launch's own quantiser bypass the read-only path
    if constexpr (MODE == kFused) return __ldcg(p);
    return __ldg(p);
}

// Last unit of a split-K tile: read the summed int32 tile from the
// workspace (vector loads, several rows in flight per thread), rescale,
// write the outputs, and return the cells and the tile counter to zero.
template <int WT, int BT, int MODE>
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
                    a_sv[t] = m < mend ? load_scale<MODE>(p.a_scale + m) : 0.0f;
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
                    __fmul_rn(__fmul_rn(__int2float_rn(acc), load_scale<MODE>(p.a_scale + m)), p.w_scale[col]);
                if (p.acc_out) p.acc_out[m * p.acc_ld + col] = acc;
            }
        }
    }
    if (leader) p.counters[u.tile] = 0u;
}

template <int KIND, int WT, int BT, int KA, int STAGES, int MODE>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ GemmParams p) {
    static_assert(KIND == 0 || MODE == kPlain, "f16 GEMMs run in the plain mode only");
    using C = Cfg<WT, BT, KA, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    __shared__ float red[kEpiWarps];
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
    sh.red = red;

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
    // every CTA is resident: the next programmatic launch on the stream may
    // start its prologue and weight prefetch on SMs as they free up (it reads
    // anything this launch writes only after its own griddepcontrol.wait)
    if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == 0 || warp == 1) {
        if (lane == 0) {
            // ---- producers: warp 0 weights, warp 1 activations ----
            const bool is_w = warp == 0;
            const CUtensorMap* map = is_w ? &p.tmap_w : &p.tmap_a;
            const uint32_t box = is_w ? C::kWBox : C::kABox;
            const int off = is_w ? 0 : C::kWBytes;
            // the first unit's coordinates (runtime divisions) are ready
            // before the dependency wait, so its first copy issues at once
            Unit t = unit_coords<WT, BT>(p, blockIdx.x);
            if (!is_w) griddep_wait();
            int g = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
                if (u != static_cast<int>(blockIdx.x)) t = unit_coords<WT, BT>(p, u);
                const int row = is_w ? t.n0 : t.m0;
                if constexpr (MODE == kFused) {
                    // the fused quantiser must have published this token tile
                    if (!is_w) {
                        if (!wait_count(p.q_ready + t.m0 / BT, static_cast<unsigned>(min(BT, p.m - t.m0)),
                                        sh.abort)) {
                            if (!*sh.abort) fail(p, sh, kErrTimeoutQuant);
                            break;
                        }
                        asm volatile("fence.proxy.async.global;" ::: "memory");
                    }
                }
                for (int kb = t.kb0; kb < t.kb1; kb += KA, ++g) {
                    const int s = g % STAGES;
                    const uint32_t ph = (g / STAGES) & 1;
                    if (g >= STAGES && !wait_or_abort(&sh.empty[s], ph ^ 1, sh.abort)) {
                        if (!*sh.abort) fail(p, sh, kErrTimeoutEmpty);
                        ok = false;
                        break;
                    }
                    // always KA atoms: an atom past the end of K (the last
                    // stage of an odd atom count) is zero-filled by the copy
                    // and adds nothing, which keeps the MMA loop branch-free
                    mbar_arrive_expect_tx(&sh.full[s], KA * box);
#pragma unroll
                    for (int a = 0; a < KA; ++a)
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
                const int buf = j % C::kBufs, use = j / C::kBufs;
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
                    const uint32_t wa = smem_u32(smem + s * C::kStage);
                    const uint32_t aa = wa + C::kWBytes;
                    const uint32_t acc0 = kb != t.kb0 ? 1u : 0u;  // the unit's first MMA overwrites
                    // straight-line MMAs (a guard around the second atom
                    // measured ~9 % slower per stage on B200)
#pragma unroll
                    for (int a = 0; a < KA; ++a) {
#pragma unroll
                        for (int ks = 0; ks < kKBytes / 32; ++ks) {
#pragma unroll
                            for (int acc = 0; acc < C::kAcc; ++acc)
                                tc_mma<KIND>(d0 + acc * BT,
                                             smem_desc_k128(wa + a * C::kWBox + acc * 128 * kKBytes + ks * 32),
                                             smem_desc_k128(aa + a * C::kABox + ks * 32), idesc,
                                             (a != 0 || ks != 0) ? 1u : acc0);
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
        bool live = true;  // false: the call was rejected, store nothing
        if constexpr (MODE == kFused) {
            griddep_wait();  // the f32 activations come from the preceding work
            waited_dep = true;
            fused_quant<BT>(p, sh, e, lane);
        }
        float* tok_scale = reinterpret_cast<float*>(smem + C::kScaleOffset) + e * BT;
        int j = 0;
        for (int u = blockIdx.x; u < p.units; u += gridDim.x, ++j) {
            const Unit t = unit_coords<WT, BT>(p, u);
            const int buf = j % C::kBufs, use = j / C::kBufs;
            const bool split = KIND == 0 && MODE != kGather && p.ksplit > 1;
            if (!waited_dep) {
                griddep_wait();  // the token scales come from the preceding work
                waited_dep = true;
                if (p.store_guard) live = *reinterpret_cast<volatile const int*>(p.err) == 0;
            }
            // accumulator and output column this thread handles
            const int acc = C::kAcc == 2 ? half : 0;
            const int col = t.n0 + acc * 128 + q * 32 + lane;
            const bool col_ok = live && col < p.n;
            const int mi = member_of(p, col);
            float* out = p.out[mi];
            const long long ldo = p.ldo[mi];
            const int ocol = col - p.n_start[mi];
            // this unit's scales, loaded while its MMAs still run
            float wsc = 0.0f;
            if constexpr (KIND == 0) wsc = col_ok ? __ldg(p.w_scale + col) : 0.0f;
            if constexpr (KIND == 0 && MODE != kFused) {
                if (!split) {
                    for (int i = lane; i < BT; i += 32) {
                        const int m = t.m0 + i;
                        tok_scale[i] = m < p.m ? __ldg(p.a_scale + m) : 0.0f;
                    }
                    __syncwarp();
                }
            }
            int ready = 0;
            if (lane == 0) ready = wait_or_abort(&sh.tfull[buf], use & 1, sh.abort) ? 1 : 0;
            ready = __shfl_sync(0xffffffffu, ready, 0);
            if (!ready && lane == 0 && !*sh.abort) fail(p, sh, kErrTimeoutAccum);
            const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                       static_cast<uint32_t>((buf * C::kAcc + acc) * BT);
            // with one accumulator the two halves split the token columns
            const int c_first = C::kAcc == 2 ? 0 : half * 16;
            const int c_step = C::kAcc == 2 ? 16 : 32;
            if constexpr (MODE == kFused) {
                // token scales written by other CTAs' quantiser warps
                if (ready && lane == 0) (void)ld_acquire_gpu(p.q_ready + t.m0 / BT);
                __syncwarp();
            }
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
                    if constexpr (KIND == 0 && MODE == kFused) {
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj) {
                            const int m = t.m0 + c + jj;
                            asv[jj] = (!split && m < p.m) ? load_scale<MODE>(a_scale + m) : 0.0f;
                        }
                    } else if constexpr (KIND == 0) {
                        // four 16-byte reads (tok_scale and c are 16-byte aligned)
#pragma unroll
                        for (int jj = 0; jj < 16; jj += 4) {
                            const float4 s4 = *reinterpret_cast<const float4*>(tok_scale + c + jj);
                            asv[jj] = s4.x;
                            asv[jj + 1] = s4.y;
                            asv[jj + 2] = s4.z;
                            asv[jj + 3] = s4.w;
                        }
                    }
                    uint32_t r[16];
                    tmem_ld16(lane_base + c, r);
                    tmem_ld_wait();
                    if (col_ok && !split && acc_out == nullptr && t.m0 + c + 16 <= p.m && MODE != kGather) {
                        // a whole chunk, no per-element branch: the 16
                        // conversions and stores are independent and interleave
                        float* __restrict__ o = out + static_cast<long long>(t.m0 + c) * ldo + ocol;
                        float v[16];
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj) {
                            if constexpr (KIND == 0)
                                v[jj] = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[jj])), asv[jj]), wsc);
                            else
                                v[jj] = __uint_as_float(r[jj]);
                        }
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj) o[jj * ldo] = v[jj];
                    } else if (col_ok) {
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
                                        if constexpr (MODE == kGather) {
                                            const long long off = static_cast<long long>(m) * ldo + ocol;
#pragma unroll 1
                                            for (int cp = 0; cp < p.copies; ++cp) p.copy_out[cp][off] = v;
                                        } else {
                                            o[jj * ldo] = v;
                                        }
                                        if (acc_out) acc_out[static_cast<long long>(m) * p.acc_ld + col] = r[jj];
                                    }
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
                    finalize_split<WT, BT, MODE>(p, t, etid, etid == 0);
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
    if constexpr (MODE == kFused) {
        // every CTA is past its waits: the last one out re-zeroes the
        // fused quantiser's counters for the next launch
        if (threadIdx.x == 0) {
            __threadfence();
            *sh.last_flag = atomicAdd(p.q_exit, 1u) == gridDim.x - 1 ? 1u : 0u;
        }
        __syncthreads();
        if (*sh.last_flag) {
            for (int t = threadIdx.x; t < p.tiles_m; t += blockDim.x) p.q_ready[t] = 0u;
            if (threadIdx.x == 0) *p.q_exit = 0u;
        }
    }
}

template <int KIND, int WT, int BT, int KA, int STAGES, int MODE>
int launch_cfg(GemmParams& p, int grid, cudaStream_t s) {
    using C = Cfg<WT, BT, KA, STAGES>;
    auto kern = gemm_tc_kernel<KIND, WT, BT, KA, STAGES, MODE>;
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
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
// stages), each about 200 KB of shared memory.  (A 256 x 256 tile, with a
// single TMEM accumulator buffer, measured 8 % slower than 128 x 256 on the
// cfg5 GEMM: its epilogue no longer overlaps the next unit's MMAs.)  k_atoms() in gemm.cu must
// agree with the KA values here.
template <int KIND, int MODE>
int launch_kind(const GemmPlan& pl, GemmParams& p, cudaStream_t s) {
    const int grid = std::min(p.units, sm_count());
    if (pl.wt == 256) {
        switch (pl.bt) {
            case 16: return launch_cfg<KIND, 256, 16, 1, 6, MODE>(p, grid, s);
            case 32: return launch_cfg<KIND, 256, 32, 1, 5, MODE>(p, grid, s);
            case 64: return launch_cfg<KIND, 256, 64, 1, 5, MODE>(p, grid, s);
            default: return launch_cfg<KIND, 256, 128, 1, 4, MODE>(p, grid, s);
        }
    }
    switch (pl.bt) {
        case 16: return launch_cfg<KIND, 128, 16, 2, 5, MODE>(p, grid, s);
        case 32: return launch_cfg<KIND, 128, 32, 2, 5, MODE>(p, grid, s);
        case 64: return launch_cfg<KIND, 128, 64, 2, 4, MODE>(p, grid, s);
        case 128: return launch_cfg<KIND, 128, 128, 2, 3, MODE>(p, grid, s);
        default: return launch_cfg<KIND, 128, 256, 1, 4, MODE>(p, grid, s);
    }
}

// One per translation unit (gemm_plain.cu, gemm_fused.cu, gemm_gather.cu,
// gemm_pair.cu).
int launch_plain(int kind, const GemmPlan& pl, GemmParams& p, cudaStream_t s);
int launch_fused(const GemmPlan& pl, GemmParams& p, cudaStream_t s);
int launch_gather(const GemmPlan& pl, GemmParams& p, cudaStream_t s);
int launch_pair(int kind, const GemmPlan& pl, GemmParams& p, cudaStream_t s);
// Two-SM pairs of the 256 x bt configuration resident at once.
int pair_capacity(int kind, int bt);

}  // namespace gemm_detail
}  // namespace rk

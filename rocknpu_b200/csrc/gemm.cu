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

#include "gemm_kernel.cuh"

namespace rk {
namespace {

using gemm_detail::GemmParams;
using gemm_detail::kKBytes;

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

// K atoms per pipeline stage of a tile configuration (matches launch_kind in
// gemm_kernel.cuh).
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
// Two-SM pair tiles (256 x bt over two CTAs, gemm_pair.cu) are taken for
// long-K shapes with at least one full wave of pair units, where they
// measured faster on B200 (cfg5 n=28672 k=8192: +8 % at m=1024, +5 % at
// m=16384); on the prefill shapes (k <= 2048, or a partial wave of pairs)
// the one-SM tiles measured faster, against what the per-SM byte count
// alone predicts.
GemmPlan plan_gemm(int kind, int m, int n, int k, bool allow_pair) {
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
    // two-SM pairs
    const char* pair_env = std::getenv("ROCKNPU_B200_GEMM_PAIR");
    const bool pair_off = pair_env != nullptr && pair_env[0] == '0';
    const bool pair_force = pair_env != nullptr && pair_env[0] == '1';
    const bool tile_forced =
        std::getenv("ROCKNPU_B200_GEMM_WT") != nullptr || std::getenv("ROCKNPU_B200_GEMM_BT") != nullptr;
    if (allow_pair && !pair_off && (pair_force || !tile_forced)) {
        const int bt = m >= 256 ? 256 : 128;
        const int units = ((n + 255) / 256) * ((m + bt - 1) / bt);
        if (pair_force || (num_kb >= 32 && m >= 256 && units >= gemm_detail::pair_capacity(kind, bt))) {
            pl.wt = 256;
            pl.bt = bt;
            pl.pair = true;
        }
        if (pair_force) {
            if (const char* v = std::getenv("ROCKNPU_B200_GEMM_BT")) {
                const int b = std::atoi(v);
                if (b == 128 || b == 256) pl.bt = b;
            }
        }
    }
    if (pl.pair) {
        pl.ksplit = 1;
        pl.kb_per_split = num_kb;
        pl.tiles = ((n + 255) / 256) * ((m + pl.bt - 1) / pl.bt);
        return pl;
    }
    // tuning overrides, result bit-identical: ROCKNPU_B200_GEMM_WT (128/256),
    // ROCKNPU_B200_GEMM_BT (16..256), ROCKNPU_B200_GEMM_KSPLIT (>= 1),
    // ROCKNPU_B200_GEMM_PAIR (0: never two-SM tiles, 1: always, bt from
    // ROCKNPU_B200_GEMM_BT when 128 or 256)
    if (const char* v = std::getenv("ROCKNPU_B200_GEMM_WT")) {
        const int w = std::atoi(v);
        if (w == 128 || w == 256) pl.wt = w;
    }
    if (const char* v = std::getenv("ROCKNPU_B200_GEMM_BT")) {
        const int b = std::atoi(v);
        if (b == 16 || b == 32 || b == 64 || b == 128 || b == 256) pl.bt = b;
    }
    if (pl.wt == 256 && pl.bt > 128) pl.bt = 128;  // TMEM holds 2 x 2 x 128 columns
    // Long-K shapes planned with tiny token tiles (BT <= 32) pay the MMA
    // issue floor (~58 cycles per tcgen05.mma whatever N is) on every stage
    // of every unit.  64-token tiles split over K so that the units about
    // fill the SMs do the same work in fewer, fuller MMAs; taken when that
    // cuts a unit's stages by more than 40 % (measured on B200, the pp128
    // down call n=2048 k=5632 m=128: 11.1 us against 13.5 us).
    bool wide_split = false;
    if (kind == 0 && !tile_forced && pl.wt == 128 && pl.bt <= 32 && m > 32 && k * eb >= 4096) {
        const int cur_stages = (num_kb + k_atoms(pl.wt, pl.bt) - 1) / k_atoms(pl.wt, pl.bt);
        const int t64 = ((n + 127) / 128) * ((m + 63) / 64);
        const int ks64 = std::max(1, std::min(8, sms / std::max(t64, 1)));
        const int stages64 = ((num_kb + ks64 - 1) / ks64 + 1) / 2;
        if (cur_stages >= 16 && ks64 >= 2 && stages64 * 10 < cur_stages * 6) {
            pl.bt = 64;
            wide_split = true;
        }
    }
    const int ka = k_atoms(pl.wt, pl.bt);
    const int tiles = ((n + pl.wt - 1) / pl.wt) * ((m + pl.bt - 1) / pl.bt);
    int ksplit = 1;
    if (kind == 0 && (wide_split || 2 * tiles <= sms) && k * eb >= 4096) {
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

size_t fused_quant_sync_elems(int m, int n, int k) {
    const GemmPlan pl = plan_gemm(0, m, n, k, false);  // fused launches run one-SM tiles
    return static_cast<size_t>((m + pl.bt - 1) / pl.bt) + 1;
}

bool fused_quant_enabled(int m, int k) {
    // a row must fit the quantiser's 8 epilogue warps (16384 floats) in
    // 16-byte vectors
    if (k % 16 != 0 || k > 8 * gemm_detail::kQuantSeg) return false;
    // Off unless ROCKNPU_B200_FUSED_QUANT=1.  Measured on B200 (TinyLlama
    // pp512 calls replayed in a CUDA graph): the standalone quantiser, which
    // triggers the GEMM's programmatic launch at its start, costs ~4 us per
    // call; in the prologue the same rows take ~8 us, because only the 8
    // epilogue warps per SM work on them (latency-bound at that occupancy)
    // and they can start only once the previous launch has fully drained.
    const char* v = std::getenv("ROCKNPU_B200_FUSED_QUANT");
    return v != nullptr && v[0] == '1' && static_cast<long long>(m) * k <= (8ll << 20);
}

int launch_gemm_tc(int kind, const void* w, long long ldw_bytes, const void* a, long long lda_bytes, int m, int n,
                   int k, const float* w_scale, const float* a_scale, const OutMembers& outs, int32_t* acc_out,
                   long long acc_ld, int* err, cudaStream_t s, const GemmWorkspace* ws, const FusedQuant* fq) {
    if (m <= 0 || n <= 0 || k <= 0) return cudaErrorInvalidValue;
    if ((ldw_bytes % 16) || (lda_bytes % 16) || (reinterpret_cast<uintptr_t>(w) % 16) ||
        (reinterpret_cast<uintptr_t>(a) % 16))
        return cudaErrorInvalidValue;
    const int eb = kind == 0 ? 1 : 2;
    if (outs.copies < 1 || outs.copies > kMaxCopies || (outs.copies > 1 && outs.count != 1))
        return cudaErrorInvalidValue;
    GemmPlan pl = plan_gemm(kind, m, n, k, fq == nullptr && outs.copies == 1);
    if (pl.ksplit > 1 && (outs.copies > 1 || outs.store_guard || ws == nullptr || ws->ws == nullptr ||
                          ws->counters == nullptr || ws->ws_elems < pl.ws_elems ||
                          ws->counter_elems < pl.counter_elems)) {
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
    p.store_guard = outs.store_guard ? 1 : 0;
    if (fq) {
        const long long k16 = (k + 15) & ~15;
        if (kind != 0 || outs.copies > 1 || !fq->a || !fq->a8 || !fq->scales || !fq->sync || fq->ld8 % 16 ||
            fq->ld8 < k16 || fq->lda < k || fq->lda % 4 || k % 16 || k > 8 * gemm_detail::kQuantSeg ||
            (reinterpret_cast<uintptr_t>(fq->a) % 16) || (reinterpret_cast<uintptr_t>(fq->a8) % 16) ||
            a != fq->a8 || a_scale != fq->scales || fq->sync_elems < static_cast<size_t>(p.tiles_m) + 1)
            return cudaErrorInvalidValue;
        p.q_a = fq->a;
        p.q_lda = fq->lda;
        p.q_k = k;
        p.q_a8 = fq->a8;
        p.q_ld8 = fq->ld8;
        p.q_scale = fq->scales;
        p.q_ready = fq->sync;
        p.q_exit = fq->sync + p.tiles_m;
    }
    if (pl.pair) {
        // each CTA of a pair loads 128 weight rows and bt/2 token rows
        if (!make_map(&p.tmap_w, w, eb, k, n, ldw_bytes, 128)) return cudaErrorInvalidValue;
        if (!make_map(&p.tmap_a, a, eb, k, m, lda_bytes, pl.bt / 2)) return cudaErrorInvalidValue;
        return gemm_detail::launch_pair(kind, pl, p, s);
    }
    if (!make_map(&p.tmap_w, w, eb, k, n, ldw_bytes, pl.wt)) return cudaErrorInvalidValue;
    if (!make_map(&p.tmap_a, a, eb, k, m, lda_bytes, pl.bt)) return cudaErrorInvalidValue;
    if (fq) return gemm_detail::launch_fused(pl, p, s);
    if (outs.copies > 1) return kind == 0 ? gemm_detail::launch_gather(pl, p, s) : cudaErrorInvalidValue;
    return gemm_detail::launch_plain(kind, pl, p, s);
}

}  // namespace rk

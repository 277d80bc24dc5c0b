// K3 / K4 on two-SM pairs (tcgen05 cta_group::2): the W8A8 GEMM and the FP16
// executor for shapes with many output tiles.
//
// A cluster of two CTAs computes one 256 x BT output tile: CTA r of the pair
// loads weight rows [n0 + 128 r, n0 + 128 r + 128) and token rows
// [m0 + r BT/2, m0 + (r + 1) BT/2) of each 128-byte K atom into its own
// shared memory, and one thread of the even CTA issues M = 256 MMAs that read
// both CTAs' halves; each CTA's TMEM receives its 128 weight rows x all BT
// tokens.  Per SM and K atom that is 128 + BT/2 rows of operand traffic for
// 128 x BT products -- a 256 x 256 pair tile moves a third fewer bytes from L2
// per product than a one-SM 128 x 256 tile -- while each CTA still holds two
// accumulator buffers (2 x BT <= 512 TMEM columns), so a unit's epilogue
// overlaps the next unit's MMAs.
//
// Barriers: full[s] lives in the even CTA and receives both CTAs' copy bytes
// (the loads name it through the cluster window); empty[s] and tfull[b] are
// signalled in both CTAs by one tcgen05.commit with a two-CTA mask; tempty[b]
// in the even CTA counts the epilogue warps of both CTAs.  Every CTA reads
// only its own operand halves from global memory.  Every wait is bounded
// (kWaitLimitNs) and every path reaches the final cluster barrier, so both
// CTAs of a pair leave together.
#include "gemm_kernel.cuh"

namespace rk {
namespace gemm_detail {

template <int BT>
struct PairCfg {
    static constexpr int kWBox = 128 * kKBytes;       // this CTA's weight rows, one K atom
    static constexpr int kABox = (BT / 2) * kKBytes;  // this CTA's token rows, one K atom
    static constexpr int kStage = kWBox + kABox;
    static constexpr int kStages = (192 * 1024) / kStage;
    static constexpr int kBarOffset = kStages * kStage;
    static constexpr int kNumBars = 2 * kStages + 5;
    // per epilogue warp, the token scales of its current unit
    static constexpr int kScaleOffset = (kBarOffset + kNumBars * 8 + 32 + 15) & ~15;  // 16-byte aligned
    static constexpr int kBytes = kScaleOffset + kEpiWarps * BT * 4 + 1024;  // + alignment slack
    static constexpr uint32_t kTmemCols = 2 * BT;                         // two accumulator buffers
    static_assert(BT == 128 || BT == 256, "pair token tile");
    static_assert(kBytes <= 232448, "shared memory");
};

__device__ __forceinline__ bool wait_cluster_or_abort(uint64_t* bar, uint32_t parity, volatile uint32_t* abort) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
#pragma unroll 1
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait_cluster(bar, parity)) return true;
        if (*abort) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}

template <int KIND, int BT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ GemmParams p) {
    using C = PairCfg<BT>;
    constexpr int S = C::kStages;
    extern __shared__ uint8_t smem_raw[];
    // same offset in both CTAs: the MMA addresses the peer's half by it
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
    uint64_t* full = bars;
    uint64_t* empty = bars + S;
    uint64_t* tfull = bars + 2 * S;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile uint32_t* abort = tmem_slot + 1;
    Shared sh{};
    sh.abort = abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 2);  // the leader's two producers
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 2 * kEpiWarps);  // epilogue warps of both CTAs
        }
        mbar_init(drain, 1);
        *abort = 0u;
        fence_mbar_init();
        prefetch_tmap(&p.tmap_w);
        prefetch_tmap(&p.tmap_a);
    }
    if (warp == 2) {
        tmem_alloc_pair(tmem_slot, C::kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    const int pair = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);

    if (warp == 0 || warp == 1) {
        if (lane == 0) {
            // ---- producers: warp 0 this CTA's weight rows, warp 1 its token rows ----
            const bool is_w = warp == 0;
            const CUtensorMap* map = is_w ? &p.tmap_w : &p.tmap_a;
            const uint32_t box = is_w ? C::kWBox : C::kABox;
            const int off = is_w ? 0 : C::kWBox;
            // first unit's coordinates before the dependency wait
            Unit t = unit_coords<256, BT>(p, pair);
            if (!is_w) griddep_wait();
            int g = 0;
            bool ok = true;
            for (int u = pair; ok && u < p.units; u += npairs) {
                if (u != pair) t = unit_coords<256, BT>(p, u);
                const int row =
                    is_w ? t.n0 + 128 * static_cast<int>(rank) : t.m0 + (BT / 2) * static_cast<int>(rank);
                for (int kb = t.kb0; kb < t.kb1; ++kb, ++g) {
                    const int s = g % S;
                    const uint32_t ph = (g / S) & 1;
                    if (g >= S && !wait_or_abort(&empty[s], ph ^ 1, abort)) {
                        if (!*abort) fail(p, sh, kErrTimeoutEmpty);
                        ok = false;
                        break;
                    }
                    // the leader expects both CTAs' bytes of this operand
                    if (leader) mbar_arrive_expect_tx(&full[s], 2 * box);
                    tma_load_2d_pair(smem + s * C::kStage + off, map, map_cluster(smem_u32(&full[s]), 0),
                                     kb * p.kb_elems, row);
                }
            }
            // every stage this producer filled must be consumed (so its copy
            // has landed) before the CTA leaves
            for (int i = max(0, g - S); i < g; ++i) {
                if (!mbar_wait(&empty[i % S], (i / S) & 1)) {
                    atomicCAS(p.err, 0, kErrTimeoutDrain);
                    break;
                }
            }
        }
    } else if (warp == 2) {
        if (lane == 0 && leader) {
            // ---- MMA issuer (even CTA) ----
            constexpr uint32_t idesc = make_idesc<KIND>(256, BT);
            int g = 0, j = 0;
            bool ok = true;
            for (int u = pair; ok && u < p.units; u += npairs, ++j) {
                const Unit t = unit_coords<256, BT>(p, u);
                const int buf = j & 1, use = j >> 1;
                if (use >= 1 && !wait_cluster_or_abort(&tempty[buf], (use - 1) & 1, abort)) {
                    if (!*abort) fail(p, sh, kErrTimeoutAccum);
                    break;
                }
                tc_fence_after();
                const uint32_t d0 = tmem_base + static_cast<uint32_t>(buf * BT);
                for (int kb = t.kb0; kb < t.kb1; ++kb, ++g) {
                    const int s = g % S;
                    const uint32_t ph = (g / S) & 1;
                    if (!wait_or_abort(&full[s], ph, abort)) {
                        if (!*abort) fail(p, sh, kErrTimeoutFull);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t wa = smem_u32(smem + s * C::kStage);
                    const uint32_t aa = wa + C::kWBox;
#pragma unroll
                    for (int ks = 0; ks < kKBytes / 32; ++ks)
                        tc_mma_pair<KIND>(d0, smem_desc_k128(wa + ks * 32), smem_desc_k128(aa + ks * 32), idesc,
                                          (kb != t.kb0 || ks != 0) ? 1u : 0u);
                    tc_commit_pair(&empty[s], 0x3);
                }
                if (ok) tc_commit_pair(&tfull[buf], 0x3);
            }
            // the pair's MMAs must finish before either CTA releases TMEM
            tc_commit_pair(drain, 0x3);
            if (!mbar_wait(drain, 0)) atomicCAS(p.err, 0, kErrTimeoutDrain);
        } else if (lane == 0) {
            // odd CTA: the leader's MMAs write this CTA's TMEM too
            if (!mbar_wait(drain, 0)) atomicCAS(p.err, 0, kErrTimeoutDrain);
        }
        __syncwarp();
    } else {
        // ---- epilogue warps 3..10: this CTA's 128 weight rows x BT tokens ----
        const int e = warp - 3;
        const int q = warp & 3;   // TMEM lane quarter this warp may access
        const int half = e >> 2;  // the two halves split the token columns
        bool waited_dep = false;
        bool live = true;
        const uint32_t tempty_leader0 = map_cluster(smem_u32(&tempty[0]), 0);
        const uint32_t tempty_leader1 = map_cluster(smem_u32(&tempty[1]), 0);
        float* tok_scale = reinterpret_cast<float*>(smem + C::kScaleOffset) + e * BT;
        int j = 0;
        for (int u = pair; u < p.units; u += npairs, ++j) {
            const Unit t = unit_coords<256, BT>(p, u);
            const int buf = j & 1, use = j >> 1;
            if (!waited_dep) {
                griddep_wait();  // the token scales come from the preceding work
                waited_dep = true;
                if (p.store_guard) live = *reinterpret_cast<volatile const int*>(p.err) == 0;
            }
            const int col = t.n0 + 128 * static_cast<int>(rank) + q * 32 + lane;
            const bool col_ok = live && col < p.n;
            const int mi = member_of(p, col);
            float* out = p.out[mi];
            const long long ldo = p.ldo[mi];
            const int ocol = col - p.n_start[mi];
            // this unit's scales, loaded while its MMAs still run
            float wsc = 0.0f;
            if constexpr (KIND == 0) {
                wsc = col_ok ? __ldg(p.w_scale + col) : 0.0f;
                for (int i = lane; i < BT; i += 32) {
                    const int m = t.m0 + i;
                    tok_scale[i] = m < p.m ? __ldg(p.a_scale + m) : 0.0f;
                }
                __syncwarp();
            }
            int ready = 0;
            if (lane == 0) ready = wait_or_abort(&tfull[buf], use & 1, abort) ? 1 : 0;
            ready = __shfl_sync(0xffffffffu, ready, 0);
            if (!ready && lane == 0 && !*abort) fail(p, sh, kErrTimeoutAccum);
            const uint32_t lane_base =
                tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * BT);
            if (ready) {
                tc_fence_after();
                int32_t* __restrict__ acc_out = p.acc_out;
#pragma unroll 1
                for (int c = half * 16; c < BT; c += 32) {
                    float asv[16];
                    if constexpr (KIND == 0) {
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
                    if (col_ok && acc_out == nullptr && t.m0 + c + 16 <= p.m) {
                        // a whole chunk, no per-element branch
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
                                    o[jj * ldo] =
                                        __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[jj])), asv[jj]), wsc);
                                    if (acc_out) acc_out[static_cast<long long>(m) * p.acc_ld + col] = r[jj];
                                } else {
                                    o[jj * ldo] = __uint_as_float(r[jj]);
                                }
                            }
                        }
                    }
                }
            }
            // this CTA's half of the TMEM buffer is free for the next unit
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (leader)
                    mbar_arrive(&tempty[buf]);
                else
                    mbar_arrive_remote(buf == 0 ? tempty_leader0 : tempty_leader1);
            }
        }
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    // neither CTA leaves (or releases TMEM) while the pair may still touch
    // its shared memory, barriers or TMEM
    cluster_sync();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, C::kTmemCols);
    }
}

template <int KIND, int BT>
int launch_pair_cfg(GemmParams& p, int npairs, cudaStream_t s) {
    using C = PairCfg<BT>;
    auto kern = gemm_pair_kernel<KIND, BT>;
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kBytes);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_done[dev] = true;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(2 * npairs), 1, 1);
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

// Pairs that can be resident at once for this configuration (clusters of
// two need two SMs of one GPC), cached per device.
template <int KIND, int BT>
int pair_slots() {
    static int slots[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && slots[dev] > 0) return slots[dev];
    using C = PairCfg<BT>;
    auto kern = gemm_pair_kernel<KIND, BT>;
    int n = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kBytes) == cudaSuccess) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(2 * 74, 1, 1);
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.dynamicSmemBytes = C::kBytes;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();
    if (n <= 0) n = sm_count() / 2 - 4;  // conservative when the query fails
    if (dev >= 0 && dev < 64) slots[dev] = n;
    return n;
}

int pair_capacity(int kind, int bt) {
    if (kind == 0) return bt == 128 ? pair_slots<0, 128>() : pair_slots<0, 256>();
    return bt == 128 ? pair_slots<1, 128>() : pair_slots<1, 256>();
}

int launch_pair(int kind, const GemmPlan& pl, GemmParams& p, cudaStream_t s) {
    const int npairs = std::min(p.units, pair_capacity(kind, pl.bt));
    if (npairs < 1) return cudaErrorInvalidValue;
    if (kind == 0) return pl.bt == 128 ? launch_pair_cfg<0, 128>(p, npairs, s) : launch_pair_cfg<0, 256>(p, npairs, s);
    return pl.bt == 128 ? launch_pair_cfg<1, 128>(p, npairs, s) : launch_pair_cfg<1, 256>(p, npairs, s);
}

}  // namespace gemm_detail
}  // namespace rk

// W8A8 GEMM with the per-token quantiser fused into its prologue
// (gemm_kernel.cuh, fused_quant).
#include "gemm_kernel.cuh"

namespace rk {
namespace gemm_detail {

int launch_fused(const GemmPlan& pl, GemmParams& p, cudaStream_t s) { return launch_kind<0, kFused>(pl, p, s); }

}  // namespace gemm_detail
}  // namespace rk

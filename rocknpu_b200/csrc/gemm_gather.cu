// W8A8 GEMM whose epilogue all-gathers over peer memory: every element is
// stored into each rank's output buffer (gemm_kernel.cuh, kGather).
#include "gemm_kernel.cuh"

namespace rk {
namespace gemm_detail {

int launch_gather(const GemmPlan& pl, GemmParams& p, cudaStream_t s) { return launch_kind<0, kGather>(pl, p, s); }

}  // namespace gemm_detail
}  // namespace rk

// Plain-mode instantiations of the tcgen05 GEMM (gemm_kernel.cuh): W8A8 on
// int8 activations from memory (K3) and the FP16 executor (K4).
#include "gemm_kernel.cuh"

namespace rk {
namespace gemm_detail {

int launch_plain(int kind, const GemmPlan& pl, GemmParams& p, cudaStream_t s) {
    return kind == 0 ? launch_kind<0, kPlain>(pl, p, s) : launch_kind<1, kPlain>(pl, p, s);
}

}  // namespace gemm_detail
}  // namespace rk

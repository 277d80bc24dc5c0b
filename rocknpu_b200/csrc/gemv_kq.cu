// K5b: M=1 decode GEMV straight from K-quant superblocks, y[n] = W[n, k] . x[k]
// with W dequantised in registers (no tensor cores, no int8 copy) -- the
// layout and launch entry points for both kinds.  The kernels run on the
// stage pipeline of gemv_stage.cuh: Q4_K in gemv_q4k.cu, Q6_K in gemv_q6k.cu.
//
// Why: a decode step streams every weight once, so its time is the weight
// bytes over HBM bandwidth.  Q4_K is 0.5625 bytes per weight, Q6_K 0.8203,
// the prepared int8 rows of the W8A8 path 1 + 4/k -- the reference keeps
// M=1 on llama.cpp's K-quant kernels for exactly that reason
// (ggml-rocknpu.cpp:305-312).
//
// Numerics: every weight is ggml's f32 dequantisation, applied per sub-block
// rather than per weight (sum_i w_i x_i = A * sum_i q_i x_i - B * sum_i x_i).
// x is held as 16-bit fixed point per block of 64 (Q4_K) or 32 (Q6_K) values
// (X = rint(x * 32767 / max|x|), x ~ X * s), so sum_i q_i X_i is an exact
// int32 dp2a sum.  Representing x that way moves each x by at most 1/65534 of
// its block's largest magnitude; the outputs land within ~1e-6 of sum |w x|
// of the exact dot product of the f32 weights (the tests assert the
// north_star's 1e-3 relative bound with that cancellation term).
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace rk {

// Q4_K: n * nb * 144 (code and header planes); Q6_K: n * nb * 210 (plane 1
// and the d plane) + 16 bytes of padding read by rounded-up stage copies.
size_t kq_layout_bytes(int kind, size_t k, size_t n) {
    if (k % 256 != 0) return 0;
    const size_t nb = k / 256;
    if (kind == kQ4K) return n * nb * 144;
    if (kind == kQ6K) return n * nb * 210 + 16;
    return 0;
}

int launch_kq_layout(int kind, const uint8_t* blocks, int k, int n, uint8_t* layout, cudaStream_t s) {
    if (kind == kQ4K) return launch_q4k_layout(blocks, k, n, layout, s);
    if (kind == kQ6K) return launch_q6k_layout(blocks, k, n, layout, s);
    return cudaErrorInvalidValue;
}

// k up to 24576 (the stage ring and the lane-order x fit shared memory well
// beyond that, but the documented limit stays what the tests cover).
int launch_gemv_kq(int kind, const uint8_t* layout, int k, int n, const float* x, float* y, int* err,
                   cudaStream_t s, bool host_out) {
    if (k > 24576) return cudaErrorInvalidValue;
    if (kind == kQ4K) return launch_gemv_q4k(layout, k, n, x, y, err, s, host_out);
    if (kind == kQ6K) return launch_gemv_q6k(layout, k, n, x, y, err, s, host_out);
    return cudaErrorInvalidValue;
}

}  // namespace rk

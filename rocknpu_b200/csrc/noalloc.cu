// W8A8 MUL_MAT on device pointers for callers that cannot allocate GPU memory.
//
// rocknpu_b200_matmul_w8a8 keeps its int8 activations, per-token scales and
// split-K partial sums in buffers the context allocates on demand.  Some
// callers cannot let a library call cudaMalloc: a runtime that fixes its
// whole memory plan at start-up and forbids allocation afterwards (real-time
// serving loops, embedded deployments with a static budget), or a host
// framework whose own allocator must own every byte.
// For them this file keeps that scratch in one fixed-size array in the
// library's device memory, so the call only launches kernels.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../include/rocknpu_b200.h"
#include "kernels.h"

namespace {

// Scratch of the allocation-free path, shared by every call on a device:
// per-token scales, int8 activations and (when the tile plan splits K) the
// split-K counters and partial sums.  Every GPU that loads the library holds
// these 16 MiB until the process exits.
constexpr size_t kScratchBytes = 16u << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Device address of g_noalloc_scratch on the current device.  In host code
// the array's name is only a host-side stand-in, so the address comes from
// cudaGetSymbolAddress, once per device, with that device current.
unsigned char* scratch_for_current_device() {
    static std::mutex mu;
    static unsigned char* addr[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (addr[dev] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            std::fprintf(stderr, "rocknpu_b200_matmul_w8a8_noalloc: cudaGetSymbolAddress failed on device %d: %s\n",
                         dev, cudaGetErrorString(e));
            return nullptr;
        }
        addr[dev] = static_cast<unsigned char*>(p);
    }
    return addr[dev];
}

}  // namespace

extern "C" int rocknpu_b200_matmul_w8a8_noalloc(const float* a, const int8_t* w_i8, const float* w_scales, float* out,
                                                size_t m, size_t k, size_t n, int* status, rocknpu_stream stream) {
    // k % 16: the int8 rows are read by the GEMV in 16-byte vectors and by
    // the GEMM's tensor maps with a k-byte weight pitch (multiples of 16)
    if (!a || !w_i8 || !w_scales || !out || !status || m == 0 || k == 0 || n == 0 || m > 0x7fffffff ||
        n > 0x7fffffff || k > 0x7fffffff || k % 16 != 0)
        return ROCKNPU_STATUS_INVALID_ARGUMENT;
    const size_t ld8 = k;
    const size_t scales_off = 0;
    const size_t a8_off = align256(m * sizeof(float));
    const size_t needed = a8_off + align256(m * ld8);
    if (needed > kScratchBytes) {
        std::fprintf(stderr,
                     "rocknpu_b200_matmul_w8a8_noalloc: m=%zu, k=%zu needs %zu bytes of scratch; the fixed scratch "
                     "holds %zu (m * k + 4 * m, each rounded up to 256 bytes)\n",
                     m, k, needed, kScratchBytes);
        return ROCKNPU_STATUS_INVALID_ARGUMENT;
    }
    unsigned char* base = scratch_for_current_device();
    if (base == nullptr) return ROCKNPU_STATUS_DEVICE_ERROR;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* a_scales = reinterpret_cast<float*>(base + scales_off);
    int8_t* a8 = reinterpret_cast<int8_t*>(base + a8_off);

    if (cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess) return ROCKNPU_STATUS_EXECUTION_ERROR;
    rk::launch_quant_rows(a, static_cast<int>(m), static_cast<int>(k), static_cast<long long>(k), a8,
                          static_cast<long long>(ld8), a_scales, status, s);
    if (cudaGetLastError() != cudaSuccess) return ROCKNPU_STATUS_EXECUTION_ERROR;
    if (m == 1) {
        rk::launch_gemv_w8a8(w_i8, w_scales, a8, a_scales, static_cast<int>(k), static_cast<int>(n), out, s);
        return cudaGetLastError() == cudaSuccess ? ROCKNPU_STATUS_OK : ROCKNPU_STATUS_EXECUTION_ERROR;
    }
    // Split-K partial sums use what is left of the scratch; the GEMM runs
    // without K splits when the plan's workspace does not fit.  The region
    // must start at zero and a previous call may have stopped mid-way, so it
    // is cleared here.
    rk::GemmWorkspace gws;
    const rk::GemmPlan pl = rk::plan_gemm(0, static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), false);
    if (pl.ksplit > 1) {
        const size_t ws_off = needed;
        const size_t cbytes = align256(pl.counter_elems * sizeof(unsigned));
        const size_t wbytes = pl.ws_elems * sizeof(int32_t);
        if (ws_off + cbytes + wbytes <= kScratchBytes) {
            gws.counters = reinterpret_cast<unsigned*>(base + ws_off);
            gws.counter_elems = pl.counter_elems;
            gws.ws = reinterpret_cast<int32_t*>(base + ws_off + cbytes);
            gws.ws_elems = pl.ws_elems;
            if (cudaMemsetAsync(base + ws_off, 0, cbytes + wbytes, s) != cudaSuccess)
                return ROCKNPU_STATUS_EXECUTION_ERROR;
        }
    }
    rk::OutMembers om;
    om.count = 1;
    om.n_start[1] = static_cast<int>(n);
    om.out[0] = out;
    om.ldo[0] = static_cast<long long>(n);
    const int e = rk::launch_gemm_tc(0, w_i8, static_cast<long long>(k), a8, static_cast<long long>(ld8),
                                     static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), w_scales, a_scales,
                                     om, nullptr, 0, status, s, &gws);
    if (e == cudaErrorInvalidValue) return ROCKNPU_STATUS_INVALID_ARGUMENT;
    return e == cudaSuccess ? ROCKNPU_STATUS_OK : ROCKNPU_STATUS_EXECUTION_ERROR;
}

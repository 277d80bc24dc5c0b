// Page-locked host buffers for the host-pointer entry points.
//
// The C ABI's callers hand it host activations and receive host outputs; the
// copies between those buffers and HBM are the end-to-end cost of a MUL_MAT
// offload.  Measured on the B200 hosts (pinned host <-> device, 1-64 MB):
// device-to-host copies run at 47-57 GB/s from any page-locked memory, but
// host-to-device copies out of cudaHostAlloc memory (4 KB pages) vary between
// 12 and 52 GB/s from one size to the next, while the same copies out of
// memory backed by 2 MB transparent huge pages and registered with
// cudaHostRegister run at 46-55 GB/s at every size.  So these buffers are
// anonymous mappings aligned to 2 MB, advised MADV_HUGEPAGE, faulted in and
// registered (portable, device-mapped).  Where the kernel gives no huge pages
// they are still page-locked 4 KB pages: correct, only the copy rate differs.
#include <cuda_runtime.h>
#include <sys/mman.h>

#include <cstdint>
#include <map>
#include <mutex>

#include "../../include/rocknpu_b200.h"

namespace {

constexpr size_t kHuge = size_t(2) << 20;

std::mutex g_mu;
std::map<uintptr_t, size_t> g_blocks;  // base -> mapped length

}  // namespace

extern "C" {

void* rocknpu_b200_host_alloc(size_t bytes) {
    if (bytes == 0 || bytes > (size_t(1) << 46)) return nullptr;
    const size_t len = (bytes + kHuge - 1) / kHuge * kHuge;
    void* raw = mmap(nullptr, len + kHuge, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
    if (raw == MAP_FAILED) return nullptr;
    // keep the 2 MB-aligned part, give back the unaligned head and tail
    const uintptr_t r = reinterpret_cast<uintptr_t>(raw);
    const uintptr_t base = (r + kHuge - 1) / kHuge * kHuge;
    if (base > r) munmap(raw, base - r);
    const uintptr_t end = r + len + kHuge;
    if (end > base + len) munmap(reinterpret_cast<void*>(base + len), end - (base + len));
    void* p = reinterpret_cast<void*>(base);
    madvise(p, len, MADV_HUGEPAGE);  // best effort
    // fault every page in before registering it
    for (size_t off = 0; off < len; off += 4096) static_cast<volatile char*>(p)[off] = 0;
    if (cudaHostRegister(p, len, cudaHostRegisterPortable | cudaHostRegisterMapped) != cudaSuccess) {
        cudaGetLastError();  // clear the error for the caller's next CUDA call
        munmap(p, len);
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    g_blocks[base] = len;
    return p;
}

int rocknpu_b200_host_free(void* ptr) {
    if (ptr == nullptr) return ROCKNPU_STATUS_OK;
    size_t len = 0;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        auto it = g_blocks.find(reinterpret_cast<uintptr_t>(ptr));
        if (it == g_blocks.end()) return ROCKNPU_STATUS_INVALID_ARGUMENT;
        len = it->second;
        g_blocks.erase(it);
    }
    const cudaError_t e = cudaHostUnregister(ptr);
    munmap(ptr, len);
    return e == cudaSuccess ? ROCKNPU_STATUS_OK : ROCKNPU_STATUS_EXECUTION_ERROR;
}

}  // extern "C"

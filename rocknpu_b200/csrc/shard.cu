// Multi-GPU N-sharding of the W8A8 MUL_MAT (one process per GPU, one node).
//
// The reference splits the weight rows (output columns) of a GEMM over its
// NPU cores: n / 32 blocks of 32 rows, an even split with the remainder to
// the first workers (rocknpu-matmul/src/int8_decode_pool.rs:1484-1491 and
// split_blocks, :1505-1522).  Here the workers are GPUs.  Each rank holds its
// prepared weight rows resident, every rank sees the whole activation matrix,
// and the output columns are exchanged in one of two ways:
//
//  * all-gather route: each rank writes its [m][width] block into a
//    rank-major buffer [world][m][shard_ld], NCCL all-gathers that buffer,
//    and gather_shards_kernel lays it out as ggml's row-major [m][n];
//  * peer route: the GEMM epilogue writes each output tile straight into the
//    [m][n] buffers of every rank over NVLink (CUDA IPC mappings, plain
//    stores, no multicast), so the exchange overlaps the tensor-core work,
//    and peer_barrier_kernel orders those stores before the consumers.
//
// Peer buffers: virtual-memory allocations (cuMemCreate, exported as a POSIX
// file descriptor that the other ranks receive over a Unix socket and map with
// cuMemMap at the allocation granularity).  Measured on B200: stores into
// legacy CUDA IPC mappings (cudaIpcOpenMemHandle) of a 1.9 GB buffer ran
// ~60x slower than into the same memory mapped this way, so legacy IPC is
// only the fallback when the driver cannot export a descriptor.  Each buffer
// starts with a 4 KB signal area (one flag word per source rank, and this
// rank's barrier epoch) followed by the data.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <poll.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <new>

#include "../../include/rocknpu_b200.h"
#include "kernels.h"
#include "ptx.cuh"

namespace {

constexpr int kMaxRanks = ROCKNPU_B200_MAX_RANKS;
constexpr size_t kSignalBytes = 4096;  // flags[kMaxRanks] at 0, epoch at 512
constexpr size_t kEpochOffset = 512;

// Wait limit of the peer barrier's flag spin (process-wide; the library's
// 2 s default unless rocknpu_b200_set_peer_wait_limit_ms changed it).
std::atomic<unsigned long long> g_peer_wait_limit_ns{rk::kWaitLimitNs};

struct PeerPtrs {
    unsigned* sig[kMaxRanks];  // every rank's signal area, mapped here
};

// Device-side barrier over the ranks of one node.  Thread t (< world)
// publishes this rank's new epoch in rank t's flag slot `rank` and waits until
// rank t's epoch has arrived in this rank's slot `t`.  The fence before the
// release store orders every earlier write of this GPU (the preceding
// kernels' peer stores included) before the flag.  Waits are bounded by
// limit_ns; on timeout the kernel records kErrTimeoutPeer and returns.
__global__ void peer_barrier_kernel(PeerPtrs peers, unsigned* local_sig, int rank, int world, int* err,
                                    unsigned long long limit_ns) {
    __shared__ unsigned epoch;
    volatile unsigned* ep = local_sig + kEpochOffset / sizeof(unsigned);
    if (threadIdx.x == 0) epoch = *ep + 1u;
    __syncthreads();
    const unsigned e = epoch;
    const int t = threadIdx.x;
    if (t < world) {
        __threadfence_system();
        unsigned* flag = peers.sig[t] + rank;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(e) : "memory");
        const unsigned* mine = local_sig + t;
        const uint64_t t0 = rk::globaltimer_ns();
        while (true) {
            unsigned v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
            if (static_cast<int>(v - e) >= 0) break;
            if (rk::globaltimer_ns() - t0 > limit_ns) {
                atomicCAS(err, 0, rk::kErrTimeoutPeer);
                break;
            }
            __nanosleep(200);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) *ep = e;
}

// Rank-major [world][m][shard_ld] (shard r at src + r * shard_elems) ->
// row-major out[m][ldo], shard r at columns [starts[r], starts[r] + widths[r]).
struct ShardTable {
    long long start[kMaxRanks];
    int width[kMaxRanks];
};

template <bool VEC>
__global__ void gather_shards_kernel(const float* __restrict__ src, long long shard_elems, long long shard_ld, int m,
                                     ShardTable tab, float* __restrict__ out, long long ldo) {
    const int r = blockIdx.y;
    const int w = tab.width[r];
    const float* s = src + r * shard_elems;
    float* o = out + tab.start[r];
    for (int row = blockIdx.x; row < m; row += gridDim.x) {
        const float* sr = s + row * shard_ld;
        float* orow = o + row * ldo;
        if (VEC) {
            for (int c = threadIdx.x * 4; c < w; c += blockDim.x * 4)
                __stcs(reinterpret_cast<float4*>(orow + c), __ldcs(reinterpret_cast<const float4*>(sr + c)));
        } else {
            for (int c = threadIdx.x; c < w; c += blockDim.x) orow[c] = sr[c];
        }
    }
}

}  // namespace

namespace {

// Driver entry points of the virtual-memory API (the runtime is linked
// statically; the driver is reached through the runtime's entry-point query).
struct Vmm {
    PFN_cuMemGetAllocationGranularity granularity = nullptr;
    PFN_cuMemCreate create = nullptr;
    PFN_cuMemRelease release = nullptr;
    PFN_cuMemAddressReserve reserve = nullptr;
    PFN_cuMemAddressFree free_va = nullptr;
    PFN_cuMemMap map = nullptr;
    PFN_cuMemUnmap unmap = nullptr;
    PFN_cuMemSetAccess set_access = nullptr;
    PFN_cuMemExportToShareableHandle export_handle = nullptr;
    PFN_cuMemImportFromShareableHandle import_handle = nullptr;
    bool ok = false;
};

template <class F>
bool entry(const char* name, F* fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPointByVersion(name, &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
        return false;
    *fn = reinterpret_cast<F>(p);
    return true;
}

const Vmm& vmm() {
    static Vmm v = [] {
        Vmm r;
        r.ok = entry("cuMemGetAllocationGranularity", &r.granularity) && entry("cuMemCreate", &r.create) &&
               entry("cuMemRelease", &r.release) && entry("cuMemAddressReserve", &r.reserve) &&
               entry("cuMemAddressFree", &r.free_va) && entry("cuMemMap", &r.map) && entry("cuMemUnmap", &r.unmap) &&
               entry("cuMemSetAccess", &r.set_access) &&
               entry("cuMemExportToShareableHandle", &r.export_handle) &&
               entry("cuMemImportFromShareableHandle", &r.import_handle);
        return r;
    }();
    return v;
}

// The 64-byte handle of a virtual-memory peer buffer: tag, mapped size and
// the abstract Unix socket on which the owner hands out its descriptor.
struct VmmBlob {
    char tag[8];  // "RNPUVMM1"
    uint64_t size;
    char sock[48];
};
static_assert(sizeof(VmmBlob) == ROCKNPU_B200_IPC_HANDLE_BYTES, "handle size");
constexpr char kVmmTag[8] = {'R', 'N', 'P', 'U', 'V', 'M', 'M', '1'};
constexpr int kSockTimeoutMs = 60000;

socklen_t abstract_addr(const char* name, sockaddr_un* a) {
    std::memset(a, 0, sizeof(*a));
    a->sun_family = AF_UNIX;
    const size_t len = strnlen(name, sizeof(a->sun_path) - 2);
    std::memcpy(a->sun_path + 1, name, len);  // leading NUL: abstract namespace
    return static_cast<socklen_t>(offsetof(sockaddr_un, sun_path) + 1 + len);
}

// Send `fd` (and our rank) to the socket `name`; retried while the peer's
// listener is not up yet.
bool send_fd(const char* name, int fd, int rank) {
    sockaddr_un a;
    const socklen_t alen = abstract_addr(name, &a);
    for (int attempt = 0; attempt < 600; ++attempt) {
        const int s = socket(AF_UNIX, SOCK_STREAM, 0);
        if (s < 0) return false;
        if (connect(s, reinterpret_cast<sockaddr*>(&a), alen) == 0) {
            msghdr msg{};
            iovec iov{&rank, sizeof(rank)};
            msg.msg_iov = &iov;
            msg.msg_iovlen = 1;
            alignas(cmsghdr) char ctrl[CMSG_SPACE(sizeof(int))] = {};
            msg.msg_control = ctrl;
            msg.msg_controllen = sizeof(ctrl);
            cmsghdr* c = CMSG_FIRSTHDR(&msg);
            c->cmsg_level = SOL_SOCKET;
            c->cmsg_type = SCM_RIGHTS;
            c->cmsg_len = CMSG_LEN(sizeof(int));
            std::memcpy(CMSG_DATA(c), &fd, sizeof(int));
            const bool ok = sendmsg(s, &msg, 0) == static_cast<ssize_t>(sizeof(rank));
            close(s);
            return ok;
        }
        close(s);
        usleep(100000);
    }
    return false;
}

// Accept one connection on `listener` (bounded wait) and take its descriptor.
bool recv_fd(int listener, int* fd, int* from) {
    pollfd p{listener, POLLIN, 0};
    if (poll(&p, 1, kSockTimeoutMs) != 1) return false;
    const int s = accept(listener, nullptr, nullptr);
    if (s < 0) return false;
    pollfd q{s, POLLIN, 0};
    bool ok = poll(&q, 1, kSockTimeoutMs) == 1;
    if (ok) {
        msghdr msg{};
        iovec iov{from, sizeof(*from)};
        msg.msg_iov = &iov;
        msg.msg_iovlen = 1;
        alignas(cmsghdr) char ctrl[CMSG_SPACE(sizeof(int))] = {};
        msg.msg_control = ctrl;
        msg.msg_controllen = sizeof(ctrl);
        ok = recvmsg(s, &msg, 0) == static_cast<ssize_t>(sizeof(*from));
        cmsghdr* c = ok ? CMSG_FIRSTHDR(&msg) : nullptr;
        ok = ok && c && c->cmsg_type == SCM_RIGHTS;
        if (ok) std::memcpy(fd, CMSG_DATA(c), sizeof(int));
    }
    close(s);
    return ok;
}

}  // namespace

struct rocknpu_b200_peer_buffer {
    int rank = 0, world = 1, device = 0;
    size_t bytes = 0;
    unsigned char* local = nullptr;         // signal area + data on this GPU
    unsigned char* mapped[kMaxRanks] = {};  // every rank's buffer in this process
    // legacy IPC fallback
    bool opened[kMaxRanks] = {};  // IPC mappings to close
    // virtual-memory path
    bool vmm = false;
    size_t alloc = 0, granularity = 0;
    CUmemGenericAllocationHandle handle[kMaxRanks] = {};  // own (at rank) and imported
    size_t mapped_size[kMaxRanks] = {};
    int export_fd = -1, listener = -1;
};

namespace {

// A virtual-memory allocation of `b->bytes` + the signal area, exported as a
// descriptor, with a listening socket to hand it out.  False: not available.
bool create_vmm(rocknpu_b200_peer_buffer* b, VmmBlob* blob) {
    const Vmm& v = vmm();
    if (!v.ok) return false;
    CUmemAllocationProp prop{};
    prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    prop.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    prop.location.id = b->device;
    size_t gran = 0;
    if (v.granularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED) != CUDA_SUCCESS || gran == 0) return false;
    const size_t alloc = (kSignalBytes + b->bytes + gran - 1) / gran * gran;
    CUmemGenericAllocationHandle h = 0;
    if (v.create(&h, alloc, &prop, 0) != CUDA_SUCCESS) return false;
    CUdeviceptr va = 0;
    CUmemAccessDesc acc{};
    acc.location = prop.location;
    acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    int fd = -1;
    bool ok = v.reserve(&va, alloc, gran, 0, 0) == CUDA_SUCCESS;
    ok = ok && v.map(va, alloc, 0, h, 0) == CUDA_SUCCESS;
    ok = ok && v.set_access(va, alloc, &acc, 1) == CUDA_SUCCESS;
    ok = ok && v.export_handle(&fd, h, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0) == CUDA_SUCCESS;
    static std::atomic<unsigned> serial{0};
    char name[48];
    std::snprintf(name, sizeof(name), "rocknpu-b200-%d-%d-%u", static_cast<int>(getpid()), b->rank, serial++);
    int listener = ok ? socket(AF_UNIX, SOCK_STREAM, 0) : -1;
    if (listener >= 0) {
        sockaddr_un a;
        const socklen_t alen = abstract_addr(name, &a);
        ok = bind(listener, reinterpret_cast<sockaddr*>(&a), alen) == 0 && listen(listener, kMaxRanks * 2) == 0;
    } else {
        ok = false;
    }
    ok = ok && cudaMemset(reinterpret_cast<void*>(va), 0, kSignalBytes) == cudaSuccess;
    if (!ok) {
        if (listener >= 0) close(listener);
        if (fd >= 0) close(fd);
        if (va) {
            v.unmap(va, alloc);
            v.free_va(va, alloc);
        }
        v.release(h);
        return false;
    }
    b->vmm = true;
    b->alloc = alloc;
    b->granularity = gran;
    b->handle[b->rank] = h;
    b->mapped_size[b->rank] = alloc;
    b->local = reinterpret_cast<unsigned char*>(va);
    b->export_fd = fd;
    b->listener = listener;
    std::memcpy(blob->tag, kVmmTag, sizeof(kVmmTag));
    blob->size = alloc;
    std::snprintf(blob->sock, sizeof(blob->sock), "%s", name);
    return true;
}

// Exchange descriptors with every other rank (all ranks call this together)
// and map their allocations.
int open_vmm(rocknpu_b200_peer_buffer* b, const VmmBlob* blobs) {
    const Vmm& v = vmm();
    for (int r = 0; r < b->world; ++r) {
        if (r == b->rank) continue;
        if (std::memcmp(blobs[r].tag, kVmmTag, sizeof(kVmmTag)) != 0) return ROCKNPU_STATUS_INVALID_ARGUMENT;
        if (!send_fd(blobs[r].sock, b->export_fd, b->rank)) {
            std::fprintf(stderr, "rocknpu_b200_peer_buffer_open: rank %d cannot reach rank %d\n", b->rank, r);
            return ROCKNPU_STATUS_EXECUTION_ERROR;
        }
    }
    int fds[kMaxRanks];
    for (int r = 0; r < kMaxRanks; ++r) fds[r] = -1;
    for (int i = 0; i < b->world - 1; ++i) {
        int fd = -1, from = -1;
        if (!recv_fd(b->listener, &fd, &from) || from < 0 || from >= b->world || from == b->rank || fds[from] >= 0) {
            if (fd >= 0) close(fd);
            for (int r = 0; r < kMaxRanks; ++r)
                if (fds[r] >= 0) close(fds[r]);
            std::fprintf(stderr, "rocknpu_b200_peer_buffer_open: rank %d did not receive every peer's buffer\n",
                         b->rank);
            return ROCKNPU_STATUS_EXECUTION_ERROR;
        }
        fds[from] = fd;
    }
    int st = ROCKNPU_STATUS_OK;
    CUmemAccessDesc acc{};
    acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    acc.location.id = b->device;
    acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    for (int r = 0; r < b->world; ++r) {
        if (r == b->rank) continue;
        CUmemGenericAllocationHandle h = 0;
        CUdeviceptr va = 0;
        const size_t size = blobs[r].size;
        bool ok = st == ROCKNPU_STATUS_OK &&
                  v.import_handle(&h, reinterpret_cast<void*>(static_cast<uintptr_t>(fds[r])),
                                  CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR) == CUDA_SUCCESS;
        close(fds[r]);
        if (!ok) {
            st = ROCKNPU_STATUS_EXECUTION_ERROR;
            continue;
        }
        b->handle[r] = h;
        ok = v.reserve(&va, size, b->granularity, 0, 0) == CUDA_SUCCESS;
        if (ok && v.map(va, size, 0, h, 0) != CUDA_SUCCESS) {
            v.free_va(va, size);
            ok = false;
        }
        if (ok && v.set_access(va, size, &acc, 1) != CUDA_SUCCESS) {
            v.unmap(va, size);
            v.free_va(va, size);
            ok = false;
        }
        if (!ok) {
            st = ROCKNPU_STATUS_EXECUTION_ERROR;
            continue;
        }
        b->mapped[r] = reinterpret_cast<unsigned char*>(va);
        b->mapped_size[r] = size;
    }
    return st;
}

}  // namespace

extern "C" {

size_t rocknpu_b200_shard_rows(size_t n, size_t world, size_t* starts, size_t* widths) {
    if (world == 0 || !starts || !widths) return 0;
    for (size_t r = 0; r < world; ++r) starts[r] = widths[r] = 0;
    const size_t blocks = (n + 31) / 32;
    if (blocks == 0) return 0;
    const size_t active = world < blocks ? world : blocks;
    const size_t base = blocks / active, extra = blocks % active;
    size_t start = 0;
    for (size_t r = 0; r < active; ++r) {
        size_t w = (base + (r < extra ? 1 : 0)) * 32;
        if (start + w > n) w = n - start;  // the last block may be short
        starts[r] = start;
        widths[r] = w;
        start += w;
    }
    for (size_t r = active; r < world; ++r) starts[r] = n;
    return active;
}

int rocknpu_b200_peer_buffer_create(size_t bytes, int rank, int world, void* handle_out,
                                    rocknpu_b200_peer_buffer** out) {
    if (!out || !handle_out || bytes == 0 || world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
        return ROCKNPU_STATUS_INVALID_ARGUMENT;
    *out = nullptr;
    auto* b = new (std::nothrow) rocknpu_b200_peer_buffer();
    if (!b) return ROCKNPU_STATUS_EXECUTION_ERROR;
    b->rank = rank;
    b->world = world;
    b->bytes = bytes;
    if (cudaGetDevice(&b->device) != cudaSuccess || cudaFree(nullptr) != cudaSuccess) {
        delete b;
        return ROCKNPU_STATUS_DEVICE_ERROR;
    }
    VmmBlob blob{};
    if (world > 1 && create_vmm(b, &blob)) {
        std::memcpy(handle_out, &blob, sizeof(blob));
        b->mapped[rank] = b->local;
        *out = b;
        return ROCKNPU_STATUS_OK;
    }
    void* p = nullptr;
    if (cudaMalloc(&p, kSignalBytes + bytes) != cudaSuccess) {
        delete b;
        return ROCKNPU_STATUS_EXECUTION_ERROR;
    }
    b->local = static_cast<unsigned char*>(p);
    cudaIpcMemHandle_t h;
    if (cudaMemset(p, 0, kSignalBytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaFree(p);
        delete b;
        return ROCKNPU_STATUS_EXECUTION_ERROR;
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == ROCKNPU_B200_IPC_HANDLE_BYTES, "IPC handle size");
    std::memcpy(handle_out, &h, sizeof(h));
    b->mapped[rank] = b->local;
    *out = b;
    return ROCKNPU_STATUS_OK;
}

int rocknpu_b200_peer_buffer_open(rocknpu_b200_peer_buffer* b, const void* handles) {
    if (!b || !handles) return ROCKNPU_STATUS_INVALID_ARGUMENT;
    if (cudaSetDevice(b->device) != cudaSuccess) return ROCKNPU_STATUS_DEVICE_ERROR;
    if (b->vmm) return open_vmm(b, static_cast<const VmmBlob*>(handles));
    const auto* hs = static_cast<const unsigned char*>(handles);
    for (int r = 0; r < b->world; ++r) {
        if (r == b->rank || b->mapped[r]) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hs + static_cast<size_t>(r) * sizeof(h), sizeof(h));
        void* p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            std::fprintf(stderr, "rocknpu_b200_peer_buffer_open: rank %d cannot map rank %d's buffer: %s\n", b->rank,
                         r, cudaGetErrorString(e));
            return ROCKNPU_STATUS_EXECUTION_ERROR;
        }
        b->mapped[r] = static_cast<unsigned char*>(p);
        b->opened[r] = true;
    }
    return ROCKNPU_STATUS_OK;
}

void* rocknpu_b200_peer_buffer_ptr(rocknpu_b200_peer_buffer* b, int r) {
    if (!b || r < 0 || r >= b->world || !b->mapped[r]) return nullptr;
    return b->mapped[r] + kSignalBytes;
}

int rocknpu_b200_set_peer_wait_limit_ms(uint32_t ms) {
    if (ms > 600000u) return ROCKNPU_STATUS_INVALID_ARGUMENT;
    g_peer_wait_limit_ns.store(ms == 0 ? rk::kWaitLimitNs : static_cast<unsigned long long>(ms) * 1000000ull,
                               std::memory_order_relaxed);
    return ROCKNPU_STATUS_OK;
}

int rocknpu_b200_peer_barrier(rocknpu_b200_peer_buffer* b, int* status, rocknpu_stream stream) {
    if (!b || !status) return ROCKNPU_STATUS_INVALID_ARGUMENT;
    PeerPtrs pp{};
    for (int r = 0; r < b->world; ++r) {
        if (!b->mapped[r]) return ROCKNPU_STATUS_INVALID_ARGUMENT;  // not opened yet
        pp.sig[r] = reinterpret_cast<unsigned*>(b->mapped[r]);
    }
    peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        pp, reinterpret_cast<unsigned*>(b->local), b->rank, b->world, status,
        g_peer_wait_limit_ns.load(std::memory_order_relaxed));
    return cudaGetLastError() == cudaSuccess ? ROCKNPU_STATUS_OK : ROCKNPU_STATUS_EXECUTION_ERROR;
}

void rocknpu_b200_peer_buffer_destroy(rocknpu_b200_peer_buffer* b) {
    if (!b) return;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(b->device);
    if (b->vmm) {
        cudaDeviceSynchronize();
        const Vmm& v = vmm();
        for (int r = 0; r < b->world; ++r) {
            if (b->mapped[r]) {
                const CUdeviceptr va = reinterpret_cast<CUdeviceptr>(b->mapped[r]);
                v.unmap(va, b->mapped_size[r]);
                v.free_va(va, b->mapped_size[r]);
            }
            if (b->handle[r]) v.release(b->handle[r]);
        }
        if (b->export_fd >= 0) close(b->export_fd);
        if (b->listener >= 0) close(b->listener);
        cudaSetDevice(cur);
        delete b;
        return;
    }
    for (int r = 0; r < b->world; ++r)
        if (b->opened[r]) cudaIpcCloseMemHandle(b->mapped[r]);
    cudaFree(b->local);
    cudaSetDevice(cur);
    delete b;
}

int rocknpu_b200_gather_shards(const float* src, size_t shard_elems, size_t shard_ld, size_t m, size_t world,
                               const size_t* starts, const size_t* widths, float* out, size_t ldo,
                               rocknpu_stream stream) {
    if (!src || !starts || !widths || !out || m == 0 || world == 0 || world > kMaxRanks || m > 0x7fffffff)
        return ROCKNPU_STATUS_INVALID_ARGUMENT;
    ShardTable tab{};
    bool vec = (reinterpret_cast<uintptr_t>(src) % 16 == 0) && (reinterpret_cast<uintptr_t>(out) % 16 == 0) &&
               shard_ld % 4 == 0 && shard_elems % 4 == 0 && ldo % 4 == 0;
    for (size_t r = 0; r < world; ++r) {
        if (widths[r] > shard_ld || starts[r] + widths[r] > ldo || m * shard_ld > shard_elems)
            return ROCKNPU_STATUS_INVALID_ARGUMENT;
        tab.start[r] = static_cast<long long>(starts[r]);
        tab.width[r] = static_cast<int>(widths[r]);
        vec = vec && starts[r] % 4 == 0 && widths[r] % 4 == 0;
    }
    const int sms = rk::sm_count();
    const unsigned rows_grid = static_cast<unsigned>(std::min<size_t>(m, static_cast<size_t>(sms) * 8));
    dim3 grid(rows_grid, static_cast<unsigned>(world));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (vec)
        gather_shards_kernel<true><<<grid, 256, 0, s>>>(src, static_cast<long long>(shard_elems),
                                                        static_cast<long long>(shard_ld), static_cast<int>(m), tab, out,
                                                        static_cast<long long>(ldo));
    else
        gather_shards_kernel<false><<<grid, 256, 0, s>>>(src, static_cast<long long>(shard_elems),
                                                         static_cast<long long>(shard_ld), static_cast<int>(m), tab,
                                                         out, static_cast<long long>(ldo));
    return cudaGetLastError() == cudaSuccess ? ROCKNPU_STATUS_OK : ROCKNPU_STATUS_EXECUTION_ERROR;
}

}  // extern "C"

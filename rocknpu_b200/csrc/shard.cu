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
// Peer buffers: cudaMalloc'd memory exported with cudaIpcGetMemHandle and
// mapped by the other ranks with cudaIpcOpenMemHandle.  Each buffer starts
// with a 4 KB signal area (one flag word per source rank, and this rank's
// barrier epoch) followed by the data.
#include <cuda_runtime.h>

#include <algorithm>
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

struct PeerPtrs {
    unsigned* sig[kMaxRanks];  // every rank's signal area, mapped here
};

// Device-side barrier over the ranks of one node.  Thread t (< world)
// publishes this rank's new epoch in rank t's flag slot `rank` and waits until
// rank t's epoch has arrived in this rank's slot `t`.  The fence before the
// release store orders every earlier write of this GPU (the preceding
// kernels' peer stores included) before the flag.  Waits are bounded; on
// timeout the kernel records kErrTimeoutPeer and returns.
__global__ void peer_barrier_kernel(PeerPtrs peers, unsigned* local_sig, int rank, int world, int* err) {
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
            if (rk::globaltimer_ns() - t0 > rk::kWaitLimitNs) {
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

struct rocknpu_b200_peer_buffer {
    int rank = 0, world = 1, device = 0;
    size_t bytes = 0;
    unsigned char* local = nullptr;              // cudaMalloc'd: signal area + data
    unsigned char* mapped[kMaxRanks] = {};       // every rank's buffer in this process
    bool opened[kMaxRanks] = {};                 // IPC mappings to close
};

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
    if (cudaGetDevice(&b->device) != cudaSuccess) {
        delete b;
        return ROCKNPU_STATUS_DEVICE_ERROR;
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

int rocknpu_b200_peer_barrier(rocknpu_b200_peer_buffer* b, int* status, rocknpu_stream stream) {
    if (!b || !status) return ROCKNPU_STATUS_INVALID_ARGUMENT;
    PeerPtrs pp{};
    for (int r = 0; r < b->world; ++r) {
        if (!b->mapped[r]) return ROCKNPU_STATUS_INVALID_ARGUMENT;  // not opened yet
        pp.sig[r] = reinterpret_cast<unsigned*>(b->mapped[r]);
    }
    peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        pp, reinterpret_cast<unsigned*>(b->local), b->rank, b->world, status);
    return cudaGetLastError() == cudaSuccess ? ROCKNPU_STATUS_OK : ROCKNPU_STATUS_EXECUTION_ERROR;
}

void rocknpu_b200_peer_buffer_destroy(rocknpu_b200_peer_buffer* b) {
    if (!b) return;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(b->device);
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

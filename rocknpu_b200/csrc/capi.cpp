// The RockNPU C ABI (include/rocknpu.h) on B200.
//
// Host side of every entry point: argument validation in the reference's
// order, the reference's route decision (which numerics a shape gets), the
// resident-weight caches keyed like the reference's DecodeWeightKey
// (address, bytes, k, n, kind; capi/src/lib.rs:33-39), and one CUDA stream
// per context.  All arithmetic runs in the sm_100a kernels (kernels.h);
// there is no CPU compute path.  Citations are file:line in the
// darkautism/RockNPU tree; "L" is crates/rocknpu-capi/src/lib.rs.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <unordered_map>
#include <vector>

#include "../../include/rocknpu.h"
#include "../../include/rocknpu_b200.h"
#include "kernels.h"
#include "ptx.cuh"

namespace {

constexpr int kOk = ROCKNPU_STATUS_OK;
constexpr int kInvalid = ROCKNPU_STATUS_INVALID_ARGUMENT;
constexpr int kDeviceError = ROCKNPU_STATUS_DEVICE_ERROR;
constexpr int kExecError = ROCKNPU_STATUS_EXECUTION_ERROR;

// Kind tags of cached weights: the reference's K-quant kinds, plus the two
// raw forms the W8 / FP16 entry points receive.
constexpr int kKindW8 = 8;
constexpr int kKindF16 = 16;

// env_enabled (L:290-298): set, non-empty and not "0".
bool env_enabled(const char* name) {
    const char* v = std::getenv(name);
    return v != nullptr && v[0] != '\0' && std::strcmp(v, "0") != 0;
}

// mtile_shape_enabled (L:330-344).
bool mtile_shape_enabled(size_t k, size_t n) {
    if (!env_enabled("ROCKNPU_W8_MTILE")) return false;
    const char* scope = std::getenv("ROCKNPU_W8_MTILE_SCOPE");
    if (scope == nullptr || scope[0] == '\0' || !std::strcmp(scope, "all")) return true;
    if (!std::strcmp(scope, "kv")) return k == 2048 && n == 256;
    if (!std::strcmp(scope, "qo")) return k == 2048 && n == 2048;
    if (!std::strcmp(scope, "ffn")) return (k == 2048 && n == 5632) || (k == 5632 && n == 2048);
    if (!std::strcmp(scope, "attn")) return k == 2048 && (n == 256 || n == 2048);
    if (!std::strcmp(scope, "safe")) return k == 2048 && (n == 256 || n == 5632);
    return false;
}

// native_mtile_routes_enabled (L:1998-2003).
bool native_routes() {
    return env_enabled("ROCKNPU_NATIVE_MTILE") && env_enabled("ROCKNPU_MTILE_PERSIST") &&
           env_enabled("ROCKNPU_W8_MTILE") && env_enabled("ROCKNPU_MTILE_MC");
}

bool mtile_rows(size_t m) {  // MTILE_ROWS (L:1992)
    return m == 4 || m == 8 || m == 12 || m == 16 || m == 32 || m == 48 || m == 64 || m == 128;
}

size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Split-K workspace of one GEMM inside a caller- or context-owned buffer:
// tile counters first (256-byte aligned), then the int32 partial sums.
size_t gemm_ws_bytes(const rk::GemmPlan& pl) {
    if (pl.ksplit <= 1) return 0;
    return round_up(pl.counter_elems * sizeof(unsigned), 256) + pl.ws_elems * sizeof(int32_t);
}

rk::GemmWorkspace gemm_ws_view(void* base, size_t bytes, const rk::GemmPlan& pl) {
    rk::GemmWorkspace w;
    if (pl.ksplit <= 1 || !base || bytes < gemm_ws_bytes(pl)) return w;
    w.counters = static_cast<unsigned*>(base);
    w.counter_elems = pl.counter_elems;
    w.ws = reinterpret_cast<int32_t*>(static_cast<char*>(base) + round_up(pl.counter_elems * sizeof(unsigned), 256));
    w.ws_elems = pl.ws_elems;
    return w;
}

// Column chunk width of split_wide_mtile (L:2140-2141) for n > 8192.
size_t wide_chunk(size_t n) {
    const size_t chunks = (n + 8191) / 8192;
    return ((n / 32 + chunks - 1) / chunks) * 32;
}

enum class Route { W8A8, FP16, Invalid };

// Which numerics rocknpu_matmul_q{4,6}_k_f32_f32 (L:4933-5256, 5380-5671)
// gives an M>1 call.  Every W8A8 branch of the reference (row tiles, 64-row
// halves, column chunks, K zero-padding, K- or N-split across cores) yields
// the same per-element result -- per-row int8 weights, per-token int8
// activations, exact int32 sums, (f32(acc)*a_s)*w_s -- so only the branch
// family matters.  Shapes no W8A8 branch accepts take the FP16 route
// (execute_cached_prefill / the uncached FP16 bridge: f16 weights and
// activations, f32 accumulation).
Route route_q46_prompt(size_t m, size_t k, size_t n) {
    const bool native = native_routes();
    const bool NATIVE = env_enabled("ROCKNPU_NATIVE_MTILE"), PERSIST = env_enabled("ROCKNPU_MTILE_PERSIST"),
               MC = env_enabled("ROCKNPU_MTILE_MC"), DOWN = env_enabled("ROCKNPU_NATIVE_MTILE_DOWN");
    size_t nc = n;
    size_t mt = m;
    if (native) {
        if (n > 8192 && n % 32 == 0) nc = wide_chunk(n);  // split_wide_mtile (L:2136-2160)
        if (!mtile_rows(m)) mt = 128;                      // run_mtile_row_chunks (L:2216-2256)
        if (mt == 128 && round_up(k, 512) > 2048 && !(round_up(k, 512) > 4096 && round_up(k, 512) <= 6144))
            mt = 64;                                       // 64-row halves (L:2110-2128)
    } else if (!mtile_rows(m)) {
        return Route::FP16;
    }
    const size_t kp = round_up(k, 512);
    const bool ncols = nc % 32 == 0 && nc <= 8192;
    // padded-K route (L:5031-5048)
    if (native && DOWN && k % 512 != 0 && kp <= 3 * 4096 && ncols) return Route::W8A8;
    // K-split route (L:5050-5075)
    if (k > 4096 && k <= 3 * 4096 && k % 512 == 0 && ncols && NATIVE && DOWN && PERSIST && MC &&
        mtile_shape_enabled(k, nc))
        return Route::W8A8;
    // N-split / single-core route (L:5077-5105)
    if (mt != 16 && NATIVE && PERSIST && k <= 4096 && k % 512 == 0 && ncols && mtile_shape_enabled(k, nc))
        return Route::W8A8;
    // M=16 route (L:5107-5148)
    if (mt == 16 && k <= 4096 && k % 512 == 0 && ncols && mtile_shape_enabled(k, nc)) return Route::W8A8;
    return Route::FP16;
}

// rocknpu_matmul_q5_k_f32_f32 (L:5270-5378): W8A8 or nothing.
Route route_q5_prompt(size_t m, size_t k, size_t n) {
    const bool native = native_routes();
    size_t nc = n;
    if (native) {
        if (n > 8192 && n % 32 == 0) nc = wide_chunk(n);
    } else if (!mtile_rows(m)) {
        return Route::Invalid;
    }
    if (env_enabled("ROCKNPU_NATIVE_MTILE") && env_enabled("ROCKNPU_MTILE_PERSIST") && k <= 4096 && k % 512 == 0 &&
        nc % 32 == 0 && nc <= 8192 && mtile_shape_enabled(k, nc))
        return Route::W8A8;
    return Route::Invalid;
}

// ---- device memory ---------------------------------------------------------

struct DevBuf {
    void* ptr = nullptr;
    size_t cap = 0;
    bool zeroed = false;  // keep the buffer all-zero on (re)allocation
    cudaError_t ensure(size_t bytes) {
        if (bytes <= cap) return cudaSuccess;
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        cap = 0;
        const size_t want = std::max(bytes, round_up(bytes + bytes / 4, 1 << 20));
        cudaError_t e = cudaMalloc(&ptr, want);
        if (e != cudaSuccess) {
            ptr = nullptr;
            return e;
        }
        if (zeroed && (e = cudaMemset(ptr, 0, want)) != cudaSuccess) {
            cudaFree(ptr);
            ptr = nullptr;
            return e;
        }
        cap = want;
        return cudaSuccess;
    }
    void release() {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        cap = 0;
    }
    template <class T>
    T* as() const {
        return static_cast<T*>(ptr);
    }
};

// Page-locked host memory mapped into the device's address space (dptr: the
// device's address of it), grown like DevBuf; the owner makes sure no copy or
// kernel that uses it is in flight when it grows or is released.
struct HostBuf {
    void* ptr = nullptr;
    void* dptr = nullptr;
    size_t cap = 0;
    cudaError_t ensure(size_t bytes) {
        if (bytes <= cap) return cudaSuccess;
        release();
        const size_t want = round_up(bytes + bytes / 4, 64 << 10);
        cudaError_t e = cudaHostAlloc(&ptr, want, cudaHostAllocMapped);
        if (e == cudaSuccess) e = cudaHostGetDevicePointer(&dptr, ptr, 0);
        if (e != cudaSuccess) {
            if (ptr) cudaFreeHost(ptr);
            ptr = dptr = nullptr;
            return e;
        }
        cap = want;
        return cudaSuccess;
    }
    void release() {
        if (ptr) cudaFreeHost(ptr);
        ptr = dptr = nullptr;
        cap = 0;
    }
    template <class T>
    T* as() const {
        return static_cast<T*>(ptr);
    }
};

// Resident prepared int8 rows [n][k] + per-row scales [n].
struct PreparedW8 {
    int8_t* w = nullptr;
    float* scales = nullptr;
    size_t n = 0, k = 0;
    std::vector<size_t> member_n;  // concatenated groups: rows per member
    ~PreparedW8() {
        if (w) cudaFree(w);
        if (scales) cudaFree(scales);
    }
    size_t bytes() const { return n * k + n * sizeof(float); }
};

// Resident K5b decode layout of one Q4_K / Q6_K weight (rk::kq_layout_bytes
// bytes, built by rk::launch_kq_layout from the K-quant blocks).
struct PreparedKq {
    uint8_t* layout = nullptr;
    int kind = 0;
    size_t n = 0, k = 0, len = 0;
    ~PreparedKq() {
        if (layout) cudaFree(layout);
    }
    size_t bytes() const { return len; }
};

// Resident f16 rows [n][ld].
struct PreparedF16 {
    __half* w = nullptr;
    size_t n = 0, k = 0, ld = 0;
    ~PreparedF16() {
        if (w) cudaFree(w);
    }
    size_t bytes() const { return n * ld * sizeof(__half); }
};

struct Key {
    uintptr_t address;
    size_t bytes, k, n;
    int kind;
    bool operator<(const Key& o) const {
        return std::tie(address, bytes, k, n, kind) < std::tie(o.address, o.bytes, o.k, o.n, o.kind);
    }
    bool operator==(const Key& o) const {
        return address == o.address && bytes == o.bytes && k == o.k && n == o.n && kind == o.kind;
    }
};

using KeyList = std::vector<Key>;
using W8Ptr = std::shared_ptr<PreparedW8>;
using F16Ptr = std::shared_ptr<PreparedF16>;
using KqPtr = std::shared_ptr<PreparedKq>;

uint64_t now_ns() {
    return static_cast<uint64_t>(
        std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now().time_since_epoch())
            .count());
}

}  // namespace

struct RockNpuContext {
    int device = 0;
    cudaStream_t stream = nullptr;   // kernels
    cudaStream_t h2d = nullptr;      // host -> device copies of activation chunks
    cudaStream_t d2h = nullptr;      // device -> host copies of output chunks
    static constexpr int kMaxChunks = 16;
    cudaEvent_t ev_in[kMaxChunks] = {}, ev_out[kMaxChunks] = {};
    bool direct_submit = false;  // ROCKNPU_W8_DIRECT_SUBMIT at creation (int8_decode_pool.rs:509)

    int* d_status = nullptr;  // device error word
    int* h_status = nullptr;  // pinned mirror

    DevBuf a_f32, a_i8, a_scale, a_f16, out_f32, staging;
    DevBuf gemm_ws;      // split-K workspace, all-zero between launches
    DevBuf quant_sync;   // fused-quantiser counters, all-zero between launches
    DevBuf hilo_a, hilo_out;  // HILO stacked activations [2m][k], summed outputs
    // M=1 staging (m1_call): a page-locked, device-mapped host block
    // [y: outputs][status word, 16 bytes][x: k floats] that the kernels write
    // y and the status into, and a device block of the same layout whose x
    // part receives the one copy of a call.
    DevBuf m1_dev;
    HostBuf m1_host;
    bool in_hilo = false;     // inside a HILO-encoded call (HiloInner, L:2025-2043)

    // Prompt-path (M-tile) resident weights: single projections and
    // concatenated same-input groups (L:1808-1849, L:2351-2384).
    std::map<Key, W8Ptr> mtile;
    std::map<KeyList, W8Ptr> groups;
    // Decode (M=1) resident weights: single, pair, triple (L:1605-1650,
    // L:3264-3600).
    std::map<Key, W8Ptr> decode;
    std::map<KeyList, W8Ptr> decode_groups;
    // Opt-in K5b decode route (ROCKNPU_B200_DECODE_KQ at creation): M=1
    // Q4_K / Q6_K members are served from decode layouts of their K-quant
    // bytes, one cached layout per same-kind group of a call's members.
    bool decode_kq = false;
    std::map<KeyList, KqPtr> kq;  // one layout per same-kind group of a call's members
    // FP16 executor weights and the FP16 route's dequantised weights.
    std::map<Key, F16Ptr> f16;

    // decode-cache statistics (rocknpu_decode_cache_stats)
    size_t hits = 0, misses = 0;
    uint64_t hit_ns = 0, miss_ns = 0;
    size_t m1_calls = 0;
    std::set<std::pair<size_t, size_t>> m1_shapes;

    // prompt-path profile (ROCKNPU_MTILE_PROFILE, L:3900-3996)
    bool profile = false;
    size_t mtile_calls = 0, mtile_hits = 0, mtile_misses = 0;
    uint64_t mtile_ns = 0, prepare_ns = 0;
    // host-pointer W8A8 pipeline phases: queueing every chunk's copies and
    // launches, then waiting for the kernels (+ status word), then for the
    // last output copy
    uint64_t issue_ns = 0, compute_wait_ns = 0, copy_wait_ns = 0;

    rocknpu_overlap_fn overlap = nullptr;
    void* overlap_user = nullptr;
};

namespace {

using Ctx = RockNpuContext;

int cuda_status(cudaError_t e) { return e == cudaSuccess ? kOk : kExecError; }

// Host wait for a stream's work: poll for up to 2 ms, then block.  A call of
// a prompt step completes in tens to hundreds of microseconds, and a blocking
// synchronisation measured ~10-15 us of wake-up latency on top (a 4-byte copy
// plus sync round trip took 18 us on the B200 hosts).
cudaError_t wait_stream(cudaStream_t s) {
    const uint64_t t0 = now_ns();
    for (;;) {
        const cudaError_t e = cudaStreamQuery(s);
        if (e != cudaErrorNotReady) return e;
        if (now_ns() - t0 > 2000000ull) return cudaStreamSynchronize(s);
    }
}

// Copy the device error word behind the work queued on `strm`, wait, and map
// it to a status.  `strm` must be ordered after every kernel of the call (the
// compute stream, or the output-copy stream once it has waited for them).
int finish_on(Ctx* c, cudaStream_t strm) {
    cudaError_t e = cudaMemcpyAsync(c->h_status, c->d_status, sizeof(int), cudaMemcpyDeviceToHost, strm);
    if (e == cudaSuccess) e = wait_stream(strm);
    if (e != cudaSuccess) return kExecError;
    const int s = *c->h_status;
    if (s == rk::kErrNone) return kOk;
    // a launch that stopped early may leave split-K partials behind
    if (s != rk::kErrNonFinite && c->gemm_ws.ptr) cudaMemset(c->gemm_ws.ptr, 0, c->gemm_ws.cap);
    if (s != rk::kErrNonFinite && c->quant_sync.ptr) cudaMemset(c->quant_sync.ptr, 0, c->quant_sync.cap);
    cudaMemset(c->d_status, 0, sizeof(int));
    return s == rk::kErrNonFinite ? kInvalid : kExecError;
}

int finish(Ctx* c) { return finish_on(c, c->stream); }

// Context split-K workspace sized for a W8A8 GEMM of this shape.
int context_ws(Ctx* c, size_t m, size_t n, size_t k, rk::GemmWorkspace* out) {
    const rk::GemmPlan pl = rk::plan_gemm(0, static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), false);
    const size_t bytes = gemm_ws_bytes(pl);
    *out = rk::GemmWorkspace{};
    if (bytes == 0) return kOk;
    if (c->gemm_ws.ensure(bytes) != cudaSuccess) return kExecError;
    *out = gemm_ws_view(c->gemm_ws.ptr, c->gemm_ws.cap, pl);
    return kOk;
}

int reset_status(Ctx* c) { return cuda_status(cudaMemsetAsync(c->d_status, 0, sizeof(int), c->stream)); }

// K2 + K3 over activation rows already in HBM: the quantiser runs fused into
// the GEMM's prologue when that pays (rk::fused_quant_enabled), else as its
// own launch.  Returns a cudaError_t value.
int launch_w8a8(Ctx* c, const int8_t* w, const float* w_scales, const float* a_dev, size_t m, size_t k, size_t n,
                int8_t* a8, size_t ld8, float* as, const rk::OutMembers& om, const rk::GemmWorkspace* gws,
                cudaStream_t s, bool allow_fused = true) {
    const int mi = static_cast<int>(m), ki = static_cast<int>(k), ni = static_cast<int>(n);
    if (allow_fused && rk::fused_quant_enabled(mi, ki) && reinterpret_cast<uintptr_t>(a_dev) % 16 == 0) {
        const size_t elems = rk::fused_quant_sync_elems(mi, ni, ki);
        if (c->quant_sync.ensure(elems * sizeof(unsigned)) != cudaSuccess) return cudaErrorMemoryAllocation;
        rk::FusedQuant fq;
        fq.a = a_dev;
        fq.lda = static_cast<long long>(k);
        fq.a8 = a8;
        fq.ld8 = static_cast<long long>(ld8);
        fq.scales = as;
        fq.sync = c->quant_sync.as<unsigned>();
        fq.sync_elems = c->quant_sync.cap / sizeof(unsigned);
        return rk::launch_gemm_tc(0, w, static_cast<long long>(k), a8, static_cast<long long>(ld8), mi, ni, ki,
                                  w_scales, as, om, nullptr, 0, c->d_status, s, gws, &fq);
    }
    rk::launch_quant_rows(a_dev, mi, ki, static_cast<long long>(k), a8, static_cast<long long>(ld8), as, c->d_status,
                          s);
    return rk::launch_gemm_tc(0, w, static_cast<long long>(k), a8, static_cast<long long>(ld8), mi, ni, ki, w_scales,
                              as, om, nullptr, 0, c->d_status, s, gws);
}

// Dequantise + requantise host K-quant rows into w/scales (device), rows of
// one member of a (possibly concatenated) prepared weight.
int prepare_member(Ctx* c, int kind, const uint8_t* host, size_t bytes, size_t k, size_t n, int8_t* w,
                   float* scales) {
    const size_t bb = rk::qblock_bytes(kind);
    if (bb == 0 || k == 0 || n == 0 || k % 256 != 0 || bytes != n * (k / 256) * bb) return kInvalid;
    if (c->staging.ensure(bytes) != cudaSuccess) return kExecError;
    if (cudaMemcpyAsync(c->staging.ptr, host, bytes, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
        return kExecError;
    rk::launch_prep_w8(kind, c->staging.as<uint8_t>(), static_cast<int>(k), static_cast<int>(n), w, scales,
                       c->d_status, c->stream);
    return cuda_status(cudaGetLastError());
}

struct Member {
    int kind;
    const uint8_t* host;  // K-quant bytes, or int8 rows for kKindW8
    const float* host_scales;  // kKindW8 only
    size_t bytes, n;
};

// Build one resident int8 weight from 1..4 members concatenated along N.
int build_w8(Ctx* c, const Member* members, size_t count, size_t k, W8Ptr& out) {
    auto p = std::make_shared<PreparedW8>();
    size_t total = 0;
    for (size_t i = 0; i < count; ++i) total += members[i].n;
    p->n = total;
    p->k = k;
    if (cudaMalloc(&p->w, total * k) != cudaSuccess || cudaMalloc(&p->scales, total * sizeof(float)) != cudaSuccess)
        return kExecError;
    int st = reset_status(c);
    if (st != kOk) return st;
    size_t row = 0;
    for (size_t i = 0; i < count && st == kOk; ++i) {
        const Member& mb = members[i];
        if (mb.kind == kKindW8) {
            if (cudaMemcpyAsync(p->w + row * k, mb.host, mb.n * k, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
                cudaMemcpyAsync(p->scales + row, mb.host_scales, mb.n * sizeof(float), cudaMemcpyHostToDevice,
                                c->stream) != cudaSuccess)
                st = kExecError;
        } else {
            st = prepare_member(c, mb.kind, mb.host, mb.bytes, k, mb.n, p->w + row * k, p->scales + row);
            // the staging buffer is reused by the next member: finish this one
            if (st == kOk && i + 1 < count) st = cuda_status(wait_stream(c->stream));
        }
        p->member_n.push_back(mb.n);
        row += mb.n;
    }
    if (st == kOk) st = finish(c);
    if (st != kOk) return st;
    out = std::move(p);
    return kOk;
}

struct OutSeg {
    float* host;  // [m][n] host output of one member
    size_t n;
};

// Rows per pipeline chunk of a host-pointer call: the activation copy of
// chunk i+1, the kernels of chunk i and the output copy of chunk i-1 run
// concurrently (rows are independent: per-token scales, per-row outputs).
// Chunks carry at least ~1.5 MB in their larger direction -- smaller copies
// lose PCIe bandwidth to per-copy cost -- and there are at most kMaxChunks.
size_t chunk_rows(size_t m, size_t k, size_t total_n) {
    // tuning override, results unchanged: ROCKNPU_B200_CHUNK_ROWS (multiple of 16)
    if (const char* v = std::getenv("ROCKNPU_B200_CHUNK_ROWS")) {
        const size_t r = static_cast<size_t>(std::atol(v));
        if (r >= 16 && r % 16 == 0) return std::min(m, std::max(r, (m + RockNpuContext::kMaxChunks - 1) /
                                                                       RockNpuContext::kMaxChunks));
    }
    // >= ~2 MB per copy and >= 128 rows per chunk: measured on B200 at
    // m = 512 for the TinyLlama calls, smaller chunks lose more to per-copy
    // and per-launch latency than they gain in overlap
    const size_t row_bytes = std::max(k, total_n) * sizeof(float);
    size_t rows = std::max<size_t>(128, ((size_t(2) << 20) + row_bytes - 1) / row_bytes);
    rows = std::max(rows, (m + RockNpuContext::kMaxChunks - 1) / RockNpuContext::kMaxChunks);
    return std::min(m, round_up(rows, 16));
}

PFN_cuPointerGetAttributes_v7000 pointer_attributes_fn() {
    static PFN_cuPointerGetAttributes_v7000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void* f = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuPointerGetAttributes", &f, 7000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuPointerGetAttributes_v7000>(f);
    });
    return fn;
}

// True when kernels may read and write the host range [p, p + bytes) at the
// same address: the whole range lies in one page-locked host allocation that
// is mapped into the device's address space at its host address (memory from
// cudaHostAlloc / cudaMallocHost under unified addressing; not pageable
// memory, not write-combined or separately mapped registrations).
bool host_mapped(const void* p, size_t bytes) {
    PFN_cuPointerGetAttributes_v7000 fn = pointer_attributes_fn();
    if (fn == nullptr || p == nullptr || bytes == 0) return false;
    CUpointer_attribute attrs[4] = {CU_POINTER_ATTRIBUTE_MEMORY_TYPE, CU_POINTER_ATTRIBUTE_DEVICE_POINTER,
                                    CU_POINTER_ATTRIBUTE_RANGE_START_ADDR, CU_POINTER_ATTRIBUTE_RANGE_SIZE};
    unsigned int type = 0;
    CUdeviceptr dptr = 0, start = 0;
    size_t size = 0;
    void* data[4] = {&type, &dptr, &start, &size};
    const CUdeviceptr addr = reinterpret_cast<CUdeviceptr>(p);
    // cuPointerGetAttributes reports unknown (pageable) pointers as type 0
    // without an error; any failure also means "not mapped"
    if (fn(4, attrs, data, addr) != CUDA_SUCCESS) return false;
    return type == CU_MEMORYTYPE_HOST && dptr == addr && size != 0 && start <= addr && addr - start <= size &&
           bytes <= size - (addr - start);
}

// Direct host access for host-pointer calls (ROCKNPU_B200_ZERO_COPY; results
// are identical either way): "1" = inputs and outputs, "in", "out", "0" or
// unset = neither (copies through device buffers).  Only buffers for which
// host_mapped() holds are accessed directly; others are copied.  Off by
// default: on B200 over PCIe 5 the copy engines move the TinyLlama calls'
// rows faster (gate/up group at m = 512: 520 us copied, 568 us in place)
// than the kernels' own 128-byte loads and stores to host memory.
void zero_copy_mode(bool* in, bool* out) {
    const char* v = std::getenv("ROCKNPU_B200_ZERO_COPY");
    if (v != nullptr && !std::strcmp(v, "1")) {
        *in = *out = true;
    } else {
        *in = v != nullptr && !std::strcmp(v, "in");
        *out = v != nullptr && !std::strcmp(v, "out");
    }
}

// One M=1 call from host buffers, for both decode routes.  The host zeroes
// the status word and writes x into the page-locked, device-mapped staging
// block; one copy moves x to the device, and the kernels queued by
// `launch(x, y, err)` on c->stream write y and any error straight into the
// host block through its mapping (plain stores: launch_gemv_w8a8_x,
// kq::set_err); the host waits once.  Each copy or memset in a stream costs a
// call a few microseconds on B200, so the sequence has two operations (copy,
// kernels) where the general path has seven.  On an error the caller's
// outputs are untouched; a non-finite x is INVALID_ARGUMENT, as on the
// general path.
template <class Launch>
int m1_call(Ctx* c, const float* a, size_t k, const OutSeg* segs, size_t nseg, bool overlap, Launch&& launch) {
    size_t total = 0;
    for (size_t i = 0; i < nseg; ++i) total += segs[i].n;
    const size_t y_bytes = round_up(total * sizeof(float), 16);
    const size_t bytes = y_bytes + 16 + k * sizeof(float);
    if (c->m1_dev.ensure(bytes) != cudaSuccess || c->m1_host.ensure(bytes) != cudaSuccess) return kExecError;
    uint8_t* hb = c->m1_host.as<uint8_t>();
    uint8_t* hd = static_cast<uint8_t*>(c->m1_host.dptr);
    uint8_t* db = c->m1_dev.as<uint8_t>();
    int* h_st = reinterpret_cast<int*>(hb + y_bytes);
    std::memset(h_st, 0, 16);
    std::memcpy(hb + y_bytes + 16, a, k * sizeof(float));
    if (cudaMemcpyAsync(db + y_bytes + 16, hb + y_bytes + 16, k * sizeof(float), cudaMemcpyHostToDevice, c->stream))
        return kExecError;
    if (launch(reinterpret_cast<const float*>(db + y_bytes + 16), reinterpret_cast<float*>(hd),
               reinterpret_cast<int*>(hd + y_bytes)) != cudaSuccess)
        return kExecError;
    if (overlap && c->overlap) {
        // one-shot host work while the GPU runs (take_overlap, L:264-273)
        rocknpu_overlap_fn fn = c->overlap;
        void* user = c->overlap_user;
        c->overlap = nullptr;
        c->overlap_user = nullptr;
        fn(user);
    }
    if (wait_stream(c->stream) != cudaSuccess) return kExecError;
    const int s = *h_st;
    if (s != rk::kErrNone) return s == rk::kErrNonFinite ? kInvalid : kExecError;
    const float* y = reinterpret_cast<const float*>(hb);
    for (size_t i = 0; i < nseg; ++i) {
        std::memcpy(segs[i].host, y, segs[i].n * sizeof(float));
        y += segs[i].n;
    }
    return kOk;
}

// Quantisation + GEMM (GEMV for m == 1) of host activations against a
// resident int8 weight, member outputs copied back, pipelined over row
// chunks on three streams.  Page-locked, device-mapped host buffers are not
// copied: the quantiser reads the activation rows from host memory and the
// GEMM epilogue stores the outputs into host memory, so the transfers overlap
// the compute tile by tile.  On INVALID_ARGUMENT (a non-finite activation)
// output rows of chunks that were already copied back hold their results.
// With `dev_a` the activations are already in device memory (one chunk, no
// copy in), and with `keep` the outputs stay in c->out_f32 (member i's
// [m][n_i] block at column offset start_i * m) instead of being copied out.
int run_w8a8(Ctx* c, const PreparedW8& pw, const float* host_a, size_t m, size_t k, const OutSeg* segs, size_t nseg,
             bool m1_overlap, const float* dev_a = nullptr, bool keep = false) {
    const size_t ld8 = round_up(k, 16);
    const size_t total_n = pw.n;
    if (m == 1 && k % 16 == 0 && !dev_a) {
        // K2 + K5 fused into one launch (the row quantiser's bits)
        return m1_call(c, host_a, k, segs, nseg, m1_overlap, [&](const float* x, float* y, int* err) {
            rk::launch_gemv_w8a8_x(pw.w, pw.scales, x, static_cast<int>(k), static_cast<int>(total_n), y, err,
                                   c->stream, /*host_out=*/true);
            return cudaGetLastError();
        });
    }
    if ((!dev_a && c->a_f32.ensure(m * k * sizeof(float))) || c->a_i8.ensure(m * ld8) ||
        c->a_scale.ensure(m * sizeof(float)) || c->out_f32.ensure(m * total_n * sizeof(float)))
        return kExecError;
    int st = reset_status(c);
    if (st != kOk) return st;
    float* out = c->out_f32.as<float>();
    if (dev_a) {
        rk::GemmWorkspace gws;
        if (context_ws(c, m, total_n, k, &gws) != kOk) return kExecError;
        rk::OutMembers om;
        om.count = static_cast<int>(nseg);
        size_t start = 0;
        for (size_t i = 0; i < nseg; ++i) {
            om.n_start[i] = static_cast<int>(start);
            om.out[i] = out + m * start;
            om.ldo[i] = static_cast<long long>(segs[i].n);
            start += segs[i].n;
        }
        om.n_start[nseg] = static_cast<int>(start);
        if (launch_w8a8(c, pw.w, pw.scales, dev_a, m, k, total_n, c->a_i8.as<int8_t>(), ld8, c->a_scale.as<float>(),
                        om, &gws, c->stream) != cudaSuccess)
            return kExecError;
        st = finish(c);
        if (st != kOk || keep) return st;
        start = 0;
        for (size_t i = 0; i < nseg; ++i) {
            if (cudaMemcpyAsync(segs[i].host, out + m * start, m * segs[i].n * sizeof(float), cudaMemcpyDeviceToHost,
                                c->stream))
                return kExecError;
            start += segs[i].n;
        }
        return cuda_status(wait_stream(c->stream));
    }
    float* a_dev = c->a_f32.as<float>();
    int8_t* a8 = c->a_i8.as<int8_t>();
    float* as = c->a_scale.as<float>();

    const uint64_t t_issue = c->profile ? now_ns() : 0;
    bool zin = false, zout = false;
    zero_copy_mode(&zin, &zout);
    zin = zin && host_mapped(host_a, m * k * sizeof(float));
    for (size_t i = 0; i < nseg && zout; ++i) zout = host_mapped(segs[i].host, m * segs[i].n * sizeof(float));

    rk::GemmWorkspace gws;
    // with both sides in host memory the whole call is one launch pair
    const size_t rows = zin && zout ? m : chunk_rows(m, k, total_n);
    // the pipeline reuses one split-K workspace per chunk: size it for the
    // largest chunk (stream order keeps chunk launches from overlapping);
    // direct host outputs run without K splits (the epilogue's store guard
    // does not cover the split-K fixup)
    if (!zout && context_ws(c, rows, total_n, k, &gws) != kOk) return kExecError;
    int chunk = 0;
    for (size_t r0 = 0; r0 < m; r0 += rows, ++chunk) {
        const size_t mr = std::min(rows, m - r0);
        cudaEvent_t ein = c->ev_in[chunk % RockNpuContext::kMaxChunks];
        cudaEvent_t eout = c->ev_out[chunk % RockNpuContext::kMaxChunks];
        if (chunk >= RockNpuContext::kMaxChunks) return kExecError;  // chunk_rows bounds the count
        const float* a_src = zin ? host_a + r0 * k : a_dev + r0 * k;
        if (!zin && (cudaMemcpyAsync(a_dev + r0 * k, host_a + r0 * k, mr * k * sizeof(float), cudaMemcpyHostToDevice,
                                     c->h2d) ||
                     cudaEventRecord(ein, c->h2d) || cudaStreamWaitEvent(c->stream, ein, 0)))
            return kExecError;
        rk::OutMembers om;
        om.count = static_cast<int>(nseg);
        om.store_guard = zout;
        size_t start = 0;
        for (size_t i = 0; i < nseg; ++i) {
            om.n_start[i] = static_cast<int>(start);
            om.out[i] = zout ? segs[i].host + r0 * segs[i].n : out + m * start + r0 * segs[i].n;
            om.ldo[i] = static_cast<long long>(segs[i].n);
            start += segs[i].n;
        }
        om.n_start[nseg] = static_cast<int>(start);
        const int e = launch_w8a8(c, pw.w, pw.scales, a_src, mr, k, total_n, a8 + r0 * ld8, ld8, as + r0, om,
                                  zout ? nullptr : &gws, c->stream, /*allow_fused=*/!zout);
        if (e != cudaSuccess) return kExecError;
        if (zout) continue;  // the epilogue stored this chunk's rows in place
        if (cudaEventRecord(eout, c->stream) || cudaStreamWaitEvent(c->d2h, eout, 0)) return kExecError;
        if (rows >= m) {
            // one chunk: check the status first so a rejected call leaves
            // the caller's output untouched, as the reference does
            st = finish(c);
            if (st != kOk) return st;
        }
        start = 0;
        for (size_t i = 0; i < nseg; ++i) {
            if (cudaMemcpyAsync(segs[i].host + r0 * segs[i].n, out + m * start + r0 * segs[i].n,
                                mr * segs[i].n * sizeof(float), cudaMemcpyDeviceToHost, c->d2h))
                return kExecError;
            start += segs[i].n;
        }
    }
    const uint64_t t_wait = c->profile ? now_ns() : 0;
    // one wait per call: with output copies queued, the copy stream has waited
    // for every chunk's kernels, so the status word is read behind the last
    // copy; in place (zero-copy) outputs leave only the compute stream
    st = zout ? finish(c) : finish_on(c, c->d2h);
    const uint64_t t_done = c->profile ? now_ns() : 0;
    const int st2 = kOk;
    if (c->profile) {
        c->issue_ns += t_wait - t_issue;
        c->compute_wait_ns += t_done - t_wait;
        c->copy_wait_ns += now_ns() - t_done;
    }
    return st != kOk ? st : st2;
}

// FP16 executor on resident f16 rows: f16(a) . w^T in f32.  `dev_a` and
// `keep` as for run_w8a8 (the output stays in c->out_f32 as [m][n]).
int run_f16(Ctx* c, const PreparedF16& pw, const float* host_a, size_t m, size_t k, float* host_out,
            const float* dev_a = nullptr, bool keep = false) {
    const size_t ldh = round_up(k, 8);
    const size_t n = pw.n;
    if ((!dev_a && c->a_f32.ensure(m * k * sizeof(float))) || c->a_f16.ensure(m * ldh * sizeof(__half)) ||
        c->out_f32.ensure(m * n * sizeof(float)))
        return kExecError;
    int st = reset_status(c);
    if (st != kOk) return st;
    // page-locked, device-mapped host buffers are read / written in place
    bool zin = false, zout = false;
    if (!dev_a) {
        zero_copy_mode(&zin, &zout);
        zin = zin && host_mapped(host_a, m * k * sizeof(float));
        zout = zout && !keep && host_mapped(host_out, m * n * sizeof(float));
    }
    if (!dev_a && !zin &&
        cudaMemcpyAsync(c->a_f32.ptr, host_a, m * k * sizeof(float), cudaMemcpyHostToDevice, c->stream))
        return kExecError;
    rk::launch_f32_to_f16(dev_a ? dev_a : zin ? host_a : c->a_f32.as<float>(), static_cast<int>(m),
                          static_cast<int>(k), static_cast<long long>(k), c->a_f16.as<__half>(),
                          static_cast<long long>(ldh), c->stream);
    rk::OutMembers om;
    om.count = 1;
    om.n_start[1] = static_cast<int>(n);
    om.out[0] = zout ? host_out : c->out_f32.as<float>();
    om.ldo[0] = static_cast<long long>(n);
    om.store_guard = zout;
    const int e = rk::launch_gemm_tc(1, pw.w, static_cast<long long>(pw.ld * 2), c->a_f16.ptr,
                                     static_cast<long long>(ldh * 2), static_cast<int>(m), static_cast<int>(n),
                                     static_cast<int>(k), nullptr, nullptr, om, nullptr, 0, c->d_status, c->stream);
    if (e != cudaSuccess) return kExecError;
    st = finish(c);
    if (st != kOk || keep || zout) return st;
    if (cudaMemcpyAsync(host_out, c->out_f32.ptr, m * n * sizeof(float), cudaMemcpyDeviceToHost, c->stream))
        return kExecError;
    return cuda_status(wait_stream(c->stream));
}

// Resident f16 weights from a host K-quant tensor (the FP16 route's
// dequantize_q*_k_prefill_f16, L:393-455).
int build_f16_from_q(Ctx* c, int kind, const uint8_t* host, size_t bytes, size_t k, size_t n, F16Ptr& out) {
    auto p = std::make_shared<PreparedF16>();
    p->n = n;
    p->k = k;
    p->ld = k;  // k % 256 == 0
    if (cudaMalloc(&p->w, n * k * sizeof(__half)) != cudaSuccess) return kExecError;
    if (c->staging.ensure(bytes) || cudaMemcpyAsync(c->staging.ptr, host, bytes, cudaMemcpyHostToDevice, c->stream))
        return kExecError;
    rk::launch_dequant_f16(kind, c->staging.as<uint8_t>(), static_cast<int>(k), static_cast<int>(n), p->w,
                           static_cast<long long>(k), c->d_status, c->stream);
    if (cudaGetLastError() != cudaSuccess || wait_stream(c->stream) != cudaSuccess) return kExecError;
    out = std::move(p);
    return kOk;
}

int build_f16_raw(Ctx* c, const uint16_t* host, size_t k, size_t n, F16Ptr& out) {
    auto p = std::make_shared<PreparedF16>();
    p->n = n;
    p->k = k;
    p->ld = round_up(k, 8);
    if (cudaMalloc(&p->w, n * p->ld * sizeof(__half)) != cudaSuccess) return kExecError;
    if (p->ld != k && cudaMemsetAsync(p->w, 0, n * p->ld * sizeof(__half), c->stream)) return kExecError;
    if (cudaMemcpy2DAsync(p->w, p->ld * sizeof(__half), host, k * sizeof(__half), k * sizeof(__half), n,
                          cudaMemcpyHostToDevice, c->stream))
        return kExecError;
    if (wait_stream(c->stream) != cudaSuccess) return kExecError;
    out = std::move(p);
    return kOk;
}

Key make_key(const void* p, size_t bytes, size_t k, size_t n, int kind) {
    return Key{reinterpret_cast<uintptr_t>(p), bytes, k, n, kind};
}

bool bind(Ctx* c) { return cudaSetDevice(c->device) == cudaSuccess; }

// Prompt-path single projection with K-quant weights (every W8A8 branch of
// L:4933-5256).
int q_prompt_w8a8(Ctx* c, int kind, const uint8_t* w, size_t bytes, const float* a, float* out, size_t m, size_t k,
                  size_t n, const float* dev_a = nullptr, bool keep = false) {
    const uint64_t t0 = c->profile ? now_ns() : 0;
    const Key key = make_key(w, bytes, k, n, kind);
    auto it = c->mtile.find(key);
    if (it == c->mtile.end()) {
        W8Ptr p;
        const uint64_t p0 = c->profile ? now_ns() : 0;
        Member mb{kind, w, nullptr, bytes, n};
        const int st = build_w8(c, &mb, 1, k, p);
        if (st != kOk) return st;
        if (c->profile) c->prepare_ns += now_ns() - p0;
        it = c->mtile.emplace(key, std::move(p)).first;
        c->mtile_misses++;
    } else {
        c->mtile_hits++;
    }
    OutSeg seg{out, n};
    const int st = run_w8a8(c, *it->second, a, m, k, &seg, 1, false, dev_a, keep);
    if (c->profile) {
        c->mtile_calls++;
        c->mtile_ns += now_ns() - t0;
    }
    return st;
}

int q_prompt_f16(Ctx* c, int kind, const uint8_t* w, size_t bytes, const float* a, float* out, size_t m, size_t k,
                 size_t n, const float* dev_a = nullptr, bool keep = false) {
    const Key key = make_key(w, bytes, k, n, kind);
    F16Ptr p;
    auto it = c->f16.find(key);
    if (it != c->f16.end()) {
        p = it->second;
    } else {
        const int st = build_f16_from_q(c, kind, w, bytes, k, n, p);
        if (st != kOk) return st;
        // execute_cached_prefill keeps the weights only under
        // ROCKNPU_PREFILL_CACHE; the uncached bridge re-decodes per call.
        if (env_enabled("ROCKNPU_PREFILL_CACHE")) c->f16.emplace(key, p);
    }
    return run_f16(c, *p, a, m, k, out, dev_a, keep);
}

// One K5b decode layout for a group of same-kind members concatenated along
// N, from their K-quant bytes (staged through c->staging, repacked by
// rk::launch_kq_layout).
int build_kq(Ctx* c, const Member* const* group, size_t count, size_t k, KqPtr& out) {
    auto p = std::make_shared<PreparedKq>();
    p->kind = group[0]->kind;
    p->k = k;
    size_t bytes = 0;
    for (size_t i = 0; i < count; ++i) {
        p->n += group[i]->n;
        bytes += group[i]->bytes;
    }
    p->len = rk::kq_layout_bytes(p->kind, k, p->n);
    if (p->len == 0) return kInvalid;
    if (cudaMalloc(&p->layout, p->len) != cudaSuccess) return kExecError;
    if (c->staging.ensure(bytes) != cudaSuccess) return kExecError;
    // the members' blocks back to back: the blocks of the group's rows in order
    // (each member's bytes are a multiple of the 144- or 210-byte block)
    size_t off = 0;
    for (size_t i = 0; i < count; ++i) {
        if (cudaMemcpyAsync(c->staging.as<uint8_t>() + off, group[i]->host, group[i]->bytes, cudaMemcpyHostToDevice,
                            c->stream) != cudaSuccess)
            return kExecError;
        off += group[i]->bytes;
    }
    if (rk::launch_kq_layout(p->kind, c->staging.as<uint8_t>(), static_cast<int>(k), static_cast<int>(p->n),
                             p->layout, c->stream) != cudaSuccess)
        return kExecError;
    const int st = cuda_status(wait_stream(c->stream));
    if (st != kOk) return st;
    out = std::move(p);
    return kOk;
}

// The K5b route applies to M=1 calls whose members are all Q4_K / Q6_K
// bytes, when the context was created with ROCKNPU_B200_DECODE_KQ set and K
// is within the GEMV's limit (24576).  Other calls keep the W8A8 route.
bool kq_route(const Ctx* c, const Member* members, size_t count, size_t k) {
    if (!c->decode_kq || k > 24576) return false;
    for (size_t i = 0; i < count; ++i)
        if (members[i].kind != rk::kQ4K && members[i].kind != rk::kQ6K) return false;
    return true;
}

// M=1 on the K5b route: the GEMV reads the cached decode layouts (0.5625 B
// per weight for Q4_K, 0.82 for Q6_K, against 1 B of int8 rows) and returns
// f32 results within 1e-3 of the exact product of the dequantised weights
// and x, instead of the W8A8 route's bits.  Cache statistics count a call as
// a hit when every group's layout was resident.
int decode_kq_m1(Ctx* c, const KeyList& keys, const Member* members, size_t count, const float* a, OutSeg* segs,
                 size_t k) {
    const uint64_t t0 = now_ns();
    // members grouped by kind (in order of first appearance, keeping their
    // order inside a group): one layout and one GEMV launch per group, the
    // outputs in group order
    int order[4], ngroups = 0, gstart[5];
    size_t n_order = 0;
    for (size_t i = 0; i < count; ++i) {
        bool seen = false;
        for (size_t j = 0; j < i; ++j) seen = seen || members[j].kind == members[i].kind;
        if (seen) continue;
        gstart[ngroups++] = static_cast<int>(n_order);
        for (size_t j = i; j < count; ++j)
            if (members[j].kind == members[i].kind) order[n_order++] = static_cast<int>(j);
    }
    gstart[ngroups] = static_cast<int>(n_order);
    KqPtr p[4];
    bool hit = true;
    size_t total = 0;
    for (int g = 0; g < ngroups; ++g) {
        KeyList gkeys;
        const Member* gm[4];
        for (int t = gstart[g]; t < gstart[g + 1]; ++t) {
            gkeys.push_back(keys[order[t]]);
            gm[t - gstart[g]] = &members[order[t]];
            total += members[order[t]].n;
        }
        auto it = c->kq.find(gkeys);
        if (it != c->kq.end()) {
            p[g] = it->second;
            continue;
        }
        hit = false;
        const int st = build_kq(c, gm, static_cast<size_t>(gstart[g + 1] - gstart[g]), k, p[g]);
        if (st != kOk) return st;
        c->kq.emplace(gkeys, p[g]);
    }
    if (!hit) c->m1_shapes.insert({k, total});
    OutSeg osegs[4];
    for (size_t t = 0; t < n_order; ++t) osegs[t] = segs[order[t]];
    const int st = m1_call(c, a, k, osegs, count, true, [&](const float* x, float* y, int* err) {
        for (int g = 0; g < ngroups; ++g) {
            const int e = rk::launch_gemv_kq(p[g]->kind, p[g]->layout, static_cast<int>(k), static_cast<int>(p[g]->n),
                                             x, y, err, c->stream, /*host_out=*/true);
            if (e != cudaSuccess) return static_cast<cudaError_t>(e);
            y += p[g]->n;
        }
        return cudaSuccess;
    });
    if (st != kOk) return st;
    const uint64_t dt = now_ns() - t0;
    c->m1_calls++;
    if (hit) {
        c->hits++;
        c->hit_ns += dt;
    } else {
        c->misses++;
        c->miss_ns += dt;
    }
    return kOk;
}

// M=1 through the decode cache (execute_cached_w8a8_m1, L:1567-1701 and the
// pair/triple forms, L:3264-3600); `members` are concatenated along N.
int decode_m1(Ctx* c, const KeyList& keys, const Member* members, size_t count, const float* a, OutSeg* segs,
              size_t k) {
    if (kq_route(c, members, count, k)) return decode_kq_m1(c, keys, members, count, a, segs, k);
    const uint64_t t0 = now_ns();
    W8Ptr p;
    bool hit = false;
    if (count == 1) {
        auto it = c->decode.find(keys[0]);
        if (it != c->decode.end()) {
            p = it->second;
            hit = true;
        }
    } else {
        auto it = c->decode_groups.find(keys);
        if (it != c->decode_groups.end()) {
            p = it->second;
            hit = true;
        }
    }
    if (!hit) {
        const int st = build_w8(c, members, count, k, p);
        if (st != kOk) return st;
        if (count == 1)
            c->decode.emplace(keys[0], p);
        else
            c->decode_groups.emplace(keys, p);
        size_t total = 0;
        for (size_t i = 0; i < count; ++i) total += members[i].n;
        c->m1_shapes.insert({k, total});
    }
    const int st = run_w8a8(c, *p, a, 1, k, segs, count, true);
    if (st != kOk) return st;
    const uint64_t dt = now_ns() - t0;
    c->m1_calls++;
    if (hit) {
        c->hits++;
        c->hit_ns += dt;
    } else {
        c->misses++;
        c->miss_ns += dt;
    }
    return kOk;
}

bool scales_valid(const float* s, size_t n) {
    for (size_t i = 0; i < n; ++i)
        if (!std::isfinite(s[i]) || s[i] <= 0.0f) return false;
    return true;
}

bool mul_overflows(size_t a, size_t b, size_t* out) { return __builtin_mul_overflow(a, b, out); }

// ROCKNPU_PREFILL_HILO (hilo_mode, L:2005-2023): 0 off, 1 "down" (wide-K
// projections only), 2 "1"/"all".
int hilo_mode() {
    const char* v = std::getenv("ROCKNPU_PREFILL_HILO");
    if (!v) return 0;
    if (std::strcmp(v, "1") == 0 || std::strcmp(v, "all") == 0) return 2;
    if (std::strcmp(v, "down") == 0) return 1;
    return 0;
}

// hilo_stack's conditions (L:2045-2053), outside an encoded call.
bool hilo_applies(const Ctx* c, size_t m, size_t k) {
    const int mode = hilo_mode();
    if (mode == 0 || m < 2 || k == 0 || c->in_hilo) return false;
    return !(mode == 1 && k <= 4096 && k % 512 == 0);
}

// Two-part activation encoding around one prompt call (L:2484-2513,
// 4981-5001, 5428-5448): rows [x; x - dequant(quant(x))] go through `inner`
// as 2m device-resident rows, and the two halves of each member's output are
// summed (hilo_sum) into the caller's buffers.  A row that does not quantise
// (non-finite) sends the reference down its normal path; `normal` is that.
template <class Inner, class Normal>
int hilo_call(Ctx* c, const float* host_a, size_t m, size_t k, const OutSeg* segs, size_t nseg, Inner&& inner,
              Normal&& normal) {
    if (c->hilo_a.ensure(2 * m * k * sizeof(float)) != cudaSuccess) return kExecError;
    float* stacked = c->hilo_a.as<float>();
    int st = reset_status(c);
    if (st != kOk) return st;
    if (cudaMemcpyAsync(stacked, host_a, m * k * sizeof(float), cudaMemcpyHostToDevice, c->stream)) return kExecError;
    rk::launch_hilo_residual(stacked, static_cast<int>(m), static_cast<int>(k), static_cast<long long>(k),
                             stacked + m * k, static_cast<long long>(k), c->d_status, c->stream);
    if (cudaGetLastError() != cudaSuccess) return kExecError;
    st = finish(c);
    if (st == kInvalid) return normal();
    if (st != kOk) return st;
    c->in_hilo = true;
    st = inner(stacked, 2 * m);
    c->in_hilo = false;
    if (st != kOk) return st;
    size_t total = 0;
    for (size_t i = 0; i < nseg; ++i) total += segs[i].n;
    if (c->hilo_out.ensure(m * total * sizeof(float)) != cudaSuccess) return kExecError;
    const float* y = c->out_f32.as<float>();
    float* sum = c->hilo_out.as<float>();
    size_t start = 0;
    for (size_t i = 0; i < nseg; ++i) {
        const size_t len = m * segs[i].n;
        const float* blk = y + 2 * m * start;  // member i's [2m][n_i] block
        rk::launch_add_halves(blk, blk + len, sum + m * start, static_cast<long long>(len), c->stream);
        if (cudaMemcpyAsync(segs[i].host, sum + m * start, len * sizeof(float), cudaMemcpyDeviceToHost, c->stream))
            return kExecError;
        start += segs[i].n;
    }
    return cuda_status(wait_stream(c->stream));
}

// Shared body of rocknpu_matmul_q{4,5,6}_k_f32_f32.
int matmul_q(Ctx* c, int kind, const uint8_t* w, size_t bytes, const float* a, float* out, size_t m, size_t k,
             size_t n) {
    if (!c || !w || !a || !out || m == 0 || k == 0 || n == 0 || k % 256 != 0) return kInvalid;
    size_t a_len, out_len, blocks, expect;
    if (mul_overflows(m, k, &a_len) || mul_overflows(m, n, &out_len) || mul_overflows(n, k / 256, &blocks) ||
        mul_overflows(blocks, rk::qblock_bytes(kind), &expect) || bytes != expect)
        return kInvalid;
    if (!bind(c)) return kDeviceError;
    if (kind == rk::kQ5K) {
        if (m == 1) return kInvalid;  // L:5303-5305
        return route_q5_prompt(m, k, n) == Route::W8A8 ? q_prompt_w8a8(c, kind, w, bytes, a, out, m, k, n) : kInvalid;
    }
    if (m == 1) {
        // execute_cached_w8a8_m1's shape checks (L:1578-1585)
        if (k % 512 != 0 || n % 32 != 0 || n > 8192) return kInvalid;
        const Key key = make_key(w, bytes, k, n, kind);
        Member mb{kind, w, nullptr, bytes, n};
        OutSeg seg{out, n};
        return decode_m1(c, KeyList{key}, &mb, 1, a, &seg, k);
    }
    auto route = [&](const float* host, const float* dev, size_t rows, bool keep) {
        switch (route_q46_prompt(rows, k, n)) {
            case Route::W8A8: return q_prompt_w8a8(c, kind, w, bytes, host, out, rows, k, n, dev, keep);
            case Route::FP16: return q_prompt_f16(c, kind, w, bytes, host, out, rows, k, n, dev, keep);
            default: return kInvalid;
        }
    };
    if (native_routes() && hilo_applies(c, m, k)) {
        OutSeg seg{out, n};
        return hilo_call(
            c, a, m, k, &seg, 1, [&](const float* dev, size_t rows) { return route(nullptr, dev, rows, true); },
            [&] { return route(a, nullptr, m, false); });
    }
    return route(a, nullptr, m, false);
}

int quant_kind46(uint32_t kind) { return kind == 4 ? rk::kQ4K : kind == 6 ? rk::kQ6K : 0; }

// Concatenated-N prompt group (execute_cached_w8a8_mtile_concat, L:2262-2424):
// one GEMM over the group's resident rows, member outputs split by column.
int concat_group(Ctx* c, size_t count, const uint8_t* const* weights, const size_t* bytes, const int* kinds,
                 const size_t* ns, const float* a, float* const* outs, size_t m, size_t k, const float* dev_a = nullptr,
                 bool keep = false) {
    const uint64_t t0 = c->profile ? now_ns() : 0;
    KeyList keys;
    std::vector<Member> members;
    std::vector<OutSeg> segs;
    size_t total = 0;
    for (size_t i = 0; i < count; ++i) {
        keys.push_back(make_key(weights[i], bytes[i], k, ns[i], kinds[i]));
        members.push_back(Member{kinds[i], weights[i], nullptr, bytes[i], ns[i]});
        segs.push_back(OutSeg{outs[i], ns[i]});
        total += ns[i];
    }
    auto it = c->groups.find(keys);
    if (it == c->groups.end()) {
        W8Ptr p;
        const int st = build_w8(c, members.data(), count, k, p);
        if (st != kOk) return st;
        it = c->groups.emplace(keys, std::move(p)).first;
        c->mtile_misses++;
    } else {
        c->mtile_hits++;
    }
    const int st = run_w8a8(c, *it->second, a, m, k, segs.data(), count, false, dev_a, keep);
    if (c->profile) {
        c->mtile_calls++;
        c->mtile_ns += now_ns() - t0;
    }
    return st;
}


}  // namespace

// ============================================================================
// C ABI
// ============================================================================

extern "C" {

size_t rocknpu_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    size_t usable = 0;
    for (int d = 0; d < n; ++d) {
        int major = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d) == cudaSuccess && major == 10)
            ++usable;
    }
    return usable;
}

rocknpu_context* rocknpu_context_create(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess || major != 10)
        return nullptr;
    auto* c = new (std::nothrow) RockNpuContext();
    if (!c) return nullptr;
    c->device = dev;
    c->direct_submit = std::getenv("ROCKNPU_W8_DIRECT_SUBMIT") != nullptr;
    c->profile = env_enabled("ROCKNPU_MTILE_PROFILE");
    c->decode_kq = env_enabled("ROCKNPU_B200_DECODE_KQ");
    c->gemm_ws.zeroed = true;
    c->quant_sync.zeroed = true;
    bool events_ok = true;
    for (int i = 0; i < RockNpuContext::kMaxChunks && events_ok; ++i)
        events_ok = cudaEventCreateWithFlags(&c->ev_in[i], cudaEventDisableTiming) == cudaSuccess &&
                    cudaEventCreateWithFlags(&c->ev_out[i], cudaEventDisableTiming) == cudaSuccess;
    if (!events_ok || cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->h2d, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->d2h, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&c->d_status, sizeof(int)) != cudaSuccess ||
        cudaHostAlloc(&c->h_status, sizeof(int), cudaHostAllocDefault) != cudaSuccess ||
        cudaMemset(c->d_status, 0, sizeof(int)) != cudaSuccess) {
        rocknpu_context_destroy(c);
        return nullptr;
    }
    return c;
}

int rocknpu_context_decode_cache_stats(const rocknpu_context* context, rocknpu_decode_cache_stats* out) {
    if (!context || !out) return kInvalid;
    const Ctx* c = context;
    size_t resident = 0;
    for (auto& kv : c->decode) resident += kv.second->bytes();
    for (auto& kv : c->decode_groups) resident += kv.second->bytes();
    for (auto& kv : c->kq) resident += kv.second->bytes();
    rocknpu_decode_cache_stats s{};
    s.hits = c->hits;
    s.misses = c->misses;
    s.entries = c->decode.size() + c->decode_groups.size() + c->kq.size();
    s.resident_bytes = resident;
    s.hit_ns = c->hit_ns;
    s.miss_ns = c->miss_ns;
    s.tuned_shapes = c->m1_shapes.size();
    s.worker1_calls = c->m1_calls;
    s.worker2_calls = 0;
    s.worker3_calls = 0;
    s.ksplit_calls = 0;
    *out = s;
    return kOk;
}

void rocknpu_context_destroy(rocknpu_context* context) {
    if (!context) return;
    Ctx* c = context;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    if (c->profile) {
        std::fprintf(stderr,
                     "ROCKNPU MTILE PROFILE calls=%zu cache_hits=%zu cache_misses=%zu total_ms=%.3f "
                     "weight_prepare_ms=%.3f issue_ms=%.3f compute_wait_ms=%.3f copy_wait_ms=%.3f\n",
                     c->mtile_calls, c->mtile_hits, c->mtile_misses, c->mtile_ns / 1e6, c->prepare_ns / 1e6,
                     c->issue_ns / 1e6, c->compute_wait_ns / 1e6, c->copy_wait_ns / 1e6);
    }
    c->mtile.clear();
    c->groups.clear();
    c->decode.clear();
    c->decode_groups.clear();
    c->kq.clear();
    c->f16.clear();
    for (DevBuf* b : {&c->a_f32, &c->a_i8, &c->a_scale, &c->a_f16, &c->out_f32, &c->staging,
                      &c->gemm_ws, &c->quant_sync, &c->hilo_a, &c->hilo_out, &c->m1_dev})
        b->release();
    c->m1_host.release();
    if (c->d_status) cudaFree(c->d_status);
    if (c->h_status) cudaFreeHost(c->h_status);
    for (int i = 0; i < RockNpuContext::kMaxChunks; ++i) {
        if (c->ev_in[i]) cudaEventDestroy(c->ev_in[i]);
        if (c->ev_out[i]) cudaEventDestroy(c->ev_out[i]);
    }
    if (c->h2d) cudaStreamDestroy(c->h2d);
    if (c->d2h) cudaStreamDestroy(c->d2h);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

int rocknpu_context_set_overlap(rocknpu_context* context, rocknpu_overlap_fn callback, void* user_data) {
    if (!context) return kInvalid;
    context->overlap = callback;
    context->overlap_user = callback ? user_data : nullptr;
    return kOk;
}

int rocknpu_matmul_q4_k_f32_f32(rocknpu_context* context, const uint8_t* weights, size_t weights_bytes,
                                const float* a, float* out, size_t m, size_t k, size_t n) {
    return matmul_q(context, rk::kQ4K, weights, weights_bytes, a, out, m, k, n);
}

int rocknpu_matmul_q5_k_f32_f32(rocknpu_context* context, const uint8_t* weights, size_t weights_bytes,
                                const float* a, float* out, size_t m, size_t k, size_t n) {
    return matmul_q(context, rk::kQ5K, weights, weights_bytes, a, out, m, k, n);
}

int rocknpu_matmul_q6_k_f32_f32(rocknpu_context* context, const uint8_t* weights, size_t weights_bytes,
                                const float* a, float* out, size_t m, size_t k, size_t n) {
    return matmul_q(context, rk::kQ6K, weights, weights_bytes, a, out, m, k, n);
}

int rocknpu_matmul_q_concat_f32_f32_mtile(rocknpu_context* context, size_t count, const uint8_t* const* weights,
                                          const size_t* bytes, const uint32_t* kinds, const size_t* ns,
                                          const float* a, float* const* outputs, size_t m, size_t k) {
    // argument checks of L:2469-2482 and execute_cached_w8a8_mtile_concat's
    // shape checks (L:2272-2298); rows are independent, so the reference's
    // 128-row tiles and 64-row halves need no split here.
    if (!context || count < 1 || count > 4 || !weights || !bytes || !kinds || !ns || !a || !outputs || m == 0 ||
        k == 0)
        return kInvalid;
    int kd[4];
    size_t total = 0;
    for (size_t i = 0; i < count; ++i) {
        if (!weights[i] || !outputs[i] || ns[i] == 0) return kInvalid;
        kd[i] = quant_kind46(kinds[i]);
        if (!kd[i]) return kInvalid;
        if (ns[i] % 32 != 0) return kInvalid;
        total += ns[i];
    }
    if (!context->direct_submit || k % 512 != 0 || k > 4096 || total < 96 || total > 3 * 8192) return kInvalid;
    for (size_t i = 0; i < count; ++i)
        if (bytes[i] != ns[i] * (k / 256) * rk::qblock_bytes(kd[i])) return kInvalid;
    if (!bind(context)) return kDeviceError;
    if (hilo_applies(context, m, k)) {
        OutSeg segs[4];
        for (size_t i = 0; i < count; ++i) segs[i] = OutSeg{outputs[i], ns[i]};
        return hilo_call(
            context, a, m, k, segs, count,
            [&](const float* dev, size_t rows) {
                return concat_group(context, count, weights, bytes, kd, ns, nullptr, outputs, rows, k, dev, true);
            },
            [&] { return concat_group(context, count, weights, bytes, kd, ns, a, outputs, m, k); });
    }
    return concat_group(context, count, weights, bytes, kd, ns, a, outputs, m, k);
}

int rocknpu_mtile_release(rocknpu_context* context, size_t count, const uint8_t* const* weights) {
    if (!context || !weights || count < 1 || count > 4) return kInvalid;
    std::vector<uintptr_t> addr(count);
    for (size_t i = 0; i < count; ++i) addr[i] = reinterpret_cast<uintptr_t>(weights[i]);
    auto involved = [&](const Key& k) { return std::find(addr.begin(), addr.end(), k.address) != addr.end(); };
    if (!bind(context)) return kDeviceError;
    cudaStreamSynchronize(context->stream);
    for (auto it = context->mtile.begin(); it != context->mtile.end();)
        it = involved(it->first) ? context->mtile.erase(it) : std::next(it);
    for (auto it = context->groups.begin(); it != context->groups.end();) {
        const KeyList& keys = it->first;
        bool exact = keys.size() == count;
        for (size_t i = 0; exact && i < count; ++i) exact = keys[i].address == addr[i];
        bool any = false;
        for (const Key& k : keys) any |= involved(k);
        it = (!exact && any) ? context->groups.erase(it) : std::next(it);
    }
    return kOk;
}

int rocknpu_prewarm_quantized_m16(rocknpu_context* context, const uint8_t* weights, size_t weights_bytes,
                                  uint32_t quant_kind, size_t k, size_t n) {
    // L:4074-4121 and prewarm_quantized_m16_with (L:4001-4072): only the
    // shapes the reference pre-warms; others are a successful no-op.
    if (!context || !weights || k == 0 || n == 0) return kInvalid;
    const int kind = quant_kind46(quant_kind);
    if (!kind || k % 256 != 0) return kInvalid;
    if (weights_bytes != n * (k / 256) * rk::qblock_bytes(kind)) return kInvalid;
    const bool shape = (k == 2048 && (n == 256 || n == 2048 || n == 5632)) || (k == 5632 && n == 2048);
    if (!shape || !mtile_shape_enabled(k, n)) return kOk;
    if (!bind(context)) return kDeviceError;
    const Key key = make_key(weights, weights_bytes, k, n, kind);
    if (context->mtile.count(key)) return kOk;
    W8Ptr p;
    Member mb{kind, weights, nullptr, weights_bytes, n};
    const int st = build_w8(context, &mb, 1, k, p);
    if (st != kOk) return st;
    context->mtile.emplace(key, std::move(p));
    return kOk;
}

int rocknpu_matmul_f16_f32_f32(rocknpu_context* context, const uint16_t* weights, const float* a, float* out,
                               size_t m, size_t k, size_t n) {
    if (!context || !weights || !a || !out || m == 0 || k == 0 || n == 0) return kInvalid;
    size_t t;
    if (mul_overflows(m, k, &t) || mul_overflows(n, k, &t) || mul_overflows(m, n, &t)) return kInvalid;
    if (!bind(context)) return kDeviceError;
    const Key key = make_key(weights, n * k * 2, k, n, kKindF16);
    F16Ptr p;
    auto it = context->f16.find(key);
    if (it != context->f16.end()) {
        p = it->second;
    } else {
        const int st = build_f16_raw(context, weights, k, n, p);
        if (st != kOk) return st;
        context->f16.emplace(key, p);
    }
    return run_f16(context, *p, a, m, k, out);
}

int rocknpu_matmul_w8a8_f32_f32_m1(rocknpu_context* context, const int8_t* weights, const float* scales,
                                   const float* a, float* out, size_t k, size_t n) {
    if (!context || !weights || !scales || !a || !out || k == 0 || n == 0) return kInvalid;
    size_t len;
    if (mul_overflows(k, n, &len)) return kInvalid;
    if (!scales_valid(scales, n)) return kInvalid;
    if (k % 512 != 0 || n % 32 != 0 || n > 8192) return kInvalid;  // L:1578-1585
    if (!bind(context)) return kDeviceError;
    const Key key = make_key(weights, len, k, n, kKindW8);
    Member mb{kKindW8, reinterpret_cast<const uint8_t*>(weights), scales, len, n};
    OutSeg seg{out, n};
    return decode_m1(context, KeyList{key}, &mb, 1, a, &seg, k);
}

int rocknpu_matmul_w8a8_f32_f32_m1_nsplit(rocknpu_context* context, const int8_t* weights, const float* scales,
                                          const float* a, float* out, size_t k, size_t n, size_t chunk_n) {
    if (!context || !weights || !scales || !a || !out || k == 0 || n == 0 || chunk_n == 0 || chunk_n % 32 != 0 ||
        n % 32 != 0)
        return kInvalid;
    for (size_t off = 0; off < n;) {
        const size_t cur = std::min(chunk_n, n - off);
        const int st = rocknpu_matmul_w8a8_f32_f32_m1(context, weights + off * k, scales + off, a, out + off, k, cur);
        if (st != kOk) return st;
        off += cur;
    }
    return kOk;
}

int rocknpu_matmul_w8a8_f32_f32_m16(rocknpu_context* context, const int8_t* weights, const float* scales,
                                    const float* a, float* out, size_t k, size_t n) {
    constexpr size_t M = 16;
    if (!context || !weights || !scales || !a || !out || k == 0 || n == 0) return kInvalid;
    size_t len;
    if (mul_overflows(k, n, &len)) return kInvalid;
    if (!scales_valid(scales, n)) return kInvalid;
    // execute_cached_w8a8_mtile's checks (L:2818-2827)
    if (!(k <= 4096 || k == 5632) || k % 512 != 0 || n % 32 != 0 || n > 8192) return kInvalid;
    if (!bind(context)) return kDeviceError;
    const Key key = make_key(weights, len, k, n, kKindW8);
    auto it = context->mtile.find(key);
    if (it == context->mtile.end()) {
        W8Ptr p;
        Member mb{kKindW8, reinterpret_cast<const uint8_t*>(weights), scales, len, n};
        const int st = build_w8(context, &mb, 1, k, p);
        if (st != kOk) return st;
        it = context->mtile.emplace(key, std::move(p)).first;
    }
    OutSeg seg{out, n};
    return run_w8a8(context, *it->second, a, M, k, &seg, 1, false);
}

int rocknpu_matmul_w8a8_pair_f32_f32_m1(rocknpu_context* context, const int8_t* w1, const float* s1, size_t n1,
                                        const int8_t* w2, const float* s2, size_t n2, const float* a, float* o1,
                                        float* o2, size_t k) {
    if (!context || !w1 || !s1 || !w2 || !s2 || !a || !o1 || !o2 || k == 0 || n1 == 0 || n2 == 0) return kInvalid;
    size_t l1, l2;
    if (mul_overflows(k, n1, &l1) || mul_overflows(k, n2, &l2)) return kInvalid;
    if (!scales_valid(s1, n1) || !scales_valid(s2, n2)) return kInvalid;
    // execute_cached_w8a8_pair_m1's checks (L:3276-3291)
    if (k % 512 != 0 || n1 % 32 != 0 || n2 % 32 != 0 || n1 + n2 > 16384) return kInvalid;
    if (!bind(context)) return kDeviceError;
    KeyList keys{make_key(w1, l1, k, n1, kKindW8), make_key(w2, l2, k, n2, kKindW8)};
    Member mb[2] = {{kKindW8, reinterpret_cast<const uint8_t*>(w1), s1, l1, n1},
                    {kKindW8, reinterpret_cast<const uint8_t*>(w2), s2, l2, n2}};
    OutSeg segs[2] = {{o1, n1}, {o2, n2}};
    return decode_m1(context, keys, mb, 2, a, segs, k);
}

int rocknpu_matmul_w8a8_triple_f32_f32_m1(rocknpu_context* context, const int8_t* w1, const float* s1, size_t n1,
                                          const int8_t* w2, const float* s2, size_t n2, const int8_t* w3,
                                          const float* s3, size_t n3, const float* a, float* o1, float* o2,
                                          float* o3, size_t k) {
    if (!context || !w1 || !s1 || !w2 || !s2 || !w3 || !s3 || !a || !o1 || !o2 || !o3 || k == 0 || n1 == 0 ||
        n2 == 0 || n3 == 0)
        return kInvalid;
    size_t l1, l2, l3;
    if (mul_overflows(k, n1, &l1) || mul_overflows(k, n2, &l2) || mul_overflows(k, n3, &l3)) return kInvalid;
    if (!scales_valid(s1, n1) || !scales_valid(s2, n2) || !scales_valid(s3, n3)) return kInvalid;
    // execute_cached_w8a8_triple_m1's checks (L:3443-3466)
    if (k % 512 != 0 || n1 % 32 != 0 || n2 % 32 != 0 || n3 % 32 != 0 || n1 + n2 + n3 > 16384) return kInvalid;
    if (!bind(context)) return kDeviceError;
    KeyList keys{make_key(w1, l1, k, n1, kKindW8), make_key(w2, l2, k, n2, kKindW8), make_key(w3, l3, k, n3, kKindW8)};
    Member mb[3] = {{kKindW8, reinterpret_cast<const uint8_t*>(w1), s1, l1, n1},
                    {kKindW8, reinterpret_cast<const uint8_t*>(w2), s2, l2, n2},
                    {kKindW8, reinterpret_cast<const uint8_t*>(w3), s3, l3, n3}};
    OutSeg segs[3] = {{o1, n1}, {o2, n2}, {o3, n3}};
    return decode_m1(context, keys, mb, 3, a, segs, k);
}

int rocknpu_matmul_q_pair_f32_f32_m1(rocknpu_context* context, const uint8_t* w1, size_t b1, uint32_t kind1,
                                     size_t n1, const uint8_t* w2, size_t b2, uint32_t kind2, size_t n2,
                                     const float* a, float* o1, float* o2, size_t k) {
    if (!context || !w1 || !w2 || !a || !o1 || !o2 || k == 0 || n1 == 0 || n2 == 0) return kInvalid;
    const int k1 = quant_kind46(kind1), k2 = quant_kind46(kind2);
    if (!k1 || !k2) return kInvalid;
    if (k % 512 != 0 || n1 % 32 != 0 || n2 % 32 != 0 || n1 + n2 > 16384) return kInvalid;
    // prepare_q*_k_w8a8's byte check (L:713-717): a mismatch is INVALID
    if (b1 != n1 * (k / 256) * rk::qblock_bytes(k1) || b2 != n2 * (k / 256) * rk::qblock_bytes(k2)) return kInvalid;
    if (!bind(context)) return kDeviceError;
    KeyList keys{make_key(w1, b1, k, n1, k1), make_key(w2, b2, k, n2, k2)};
    Member mb[2] = {{k1, w1, nullptr, b1, n1}, {k2, w2, nullptr, b2, n2}};
    OutSeg segs[2] = {{o1, n1}, {o2, n2}};
    return decode_m1(context, keys, mb, 2, a, segs, k);
}

int rocknpu_matmul_q_triple_f32_f32_m1(rocknpu_context* context, const uint8_t* w1, size_t b1, uint32_t kind1,
                                       size_t n1, const uint8_t* w2, size_t b2, uint32_t kind2, size_t n2,
                                       const uint8_t* w3, size_t b3, uint32_t kind3, size_t n3, const float* a,
                                       float* o1, float* o2, float* o3, size_t k) {
    if (!context || !w1 || !w2 || !w3 || !a || !o1 || !o2 || !o3 || k == 0 || n1 == 0 || n2 == 0 || n3 == 0)
        return kInvalid;
    const int k1 = quant_kind46(kind1), k2 = quant_kind46(kind2), k3 = quant_kind46(kind3);
    if (!k1 || !k2 || !k3) return kInvalid;
    if (k % 512 != 0 || n1 % 32 != 0 || n2 % 32 != 0 || n3 % 32 != 0 || n1 + n2 + n3 > 16384) return kInvalid;
    if (b1 != n1 * (k / 256) * rk::qblock_bytes(k1) || b2 != n2 * (k / 256) * rk::qblock_bytes(k2) ||
        b3 != n3 * (k / 256) * rk::qblock_bytes(k3))
        return kInvalid;
    if (!bind(context)) return kDeviceError;
    KeyList keys{make_key(w1, b1, k, n1, k1), make_key(w2, b2, k, n2, k2), make_key(w3, b3, k, n3, k3)};
    Member mb[3] = {{k1, w1, nullptr, b1, n1}, {k2, w2, nullptr, b2, n2}, {k3, w3, nullptr, b3, n3}};
    OutSeg segs[3] = {{o1, n1}, {o2, n2}, {o3, n3}};
    return decode_m1(context, keys, mb, 3, a, segs, k);
}

int rocknpu_matmul_q_pair_f32_f32_mtile(rocknpu_context* context, const uint8_t* w1, size_t b1, uint32_t kind1,
                                        size_t n1, const uint8_t* w2, size_t b2, uint32_t kind2, size_t n2,
                                        const float* a, float* o1, float* o2, size_t m, size_t k) {
    if (!context || !w1 || !w2 || !a || !o1 || !o2 || m == 0 || k == 0 || n1 == 0 || n2 == 0) return kInvalid;
    const int k1 = quant_kind46(kind1), k2 = quant_kind46(kind2);
    if (!k1 || !k2) return kInvalid;
    // execute_cached_w8a8_mtile_pair_pool's checks (L:2628-2639)
    if (!mtile_rows(m) || n1 != n2 || k > 4096 || k % 512 != 0 || n1 < 2048 || n1 > 8192 || n1 % 32 != 0)
        return kInvalid;
    if (b1 != n1 * (k / 256) * rk::qblock_bytes(k1) || b2 != n2 * (k / 256) * rk::qblock_bytes(k2)) return kInvalid;
    if (!bind(context)) return kDeviceError;
    const uint8_t* ws[2] = {w1, w2};
    const size_t bs[2] = {b1, b2};
    const int kd[2] = {k1, k2};
    const size_t ns[2] = {n1, n2};
    float* outs[2] = {o1, o2};
    return concat_group(context, 2, ws, bs, kd, ns, a, outs, m, k);
}

int rocknpu_matmul_w8a8_swiglu_down_f32(rocknpu_context* context, const int8_t* gw, const float* gs,
                                        const int8_t* uw, const float* us, const int8_t* dw, const float* ds,
                                        const float* a, float* out, size_t projection_k, size_t ffn_n,
                                        size_t output_n) {
    if (!context || !gw || !gs || !uw || !us || !dw || !ds || !a || !out || projection_k == 0 || ffn_n == 0 ||
        output_n == 0)
        return kInvalid;
    size_t t;
    if (mul_overflows(projection_k, ffn_n, &t) || mul_overflows(ffn_n, output_n, &t)) return kInvalid;
    std::vector<float> gate(ffn_n), up(ffn_n);
    int st = rocknpu_matmul_w8a8_pair_f32_f32_m1(context, gw, gs, ffn_n, uw, us, ffn_n, a, gate.data(), up.data(),
                                                 projection_k);
    if (st != kOk) return st;
    // F32 SwiGLU on the host, where the reference computes it (L:4368-4373):
    // g * (1 / (1 + exp(-g))) * u with the C library's expf -- the function
    // Rust's f32::exp calls -- and no fused multiply-add, so the down
    // projection sees the reference's activation bits.
    for (size_t i = 0; i < ffn_n; ++i) {
        const float g = gate[i];
        const float sig = 1.0f / (1.0f + ::expf(-g));
        gate[i] = g * sig * up[i];
    }
    return rocknpu_matmul_w8a8_f32_f32_m1(context, dw, ds, gate.data(), out, ffn_n, output_n);
}


// ---- device-pointer entry points (rocknpu_b200.h) -------------------------

rocknpu_stream rocknpu_b200_context_stream(rocknpu_context* context) {
    return context ? static_cast<rocknpu_stream>(context->stream) : nullptr;
}

int rocknpu_b200_host_mapped(const void* ptr, size_t bytes) { return host_mapped(ptr, bytes) ? 1 : 0; }

int rocknpu_b200_context_prompt_cache_stats(const rocknpu_context* context, rocknpu_b200_prompt_cache_stats* out) {
    if (!context || !out) return kInvalid;
    *out = rocknpu_b200_prompt_cache_stats{};
    out->single_entries = context->mtile.size();
    out->group_entries = context->groups.size();
    out->hits = context->mtile_hits;
    out->misses = context->mtile_misses;
    for (const auto& kv : context->mtile) out->resident_bytes += kv.second->bytes();
    for (const auto& kv : context->groups) out->resident_bytes += kv.second->bytes();
    return kOk;
}

int rocknpu_b200_status_code(int device_status) {
    if (device_status == rk::kErrNone) return kOk;
    return device_status == rk::kErrNonFinite ? kInvalid : kExecError;
}

int rocknpu_b200_context_check(rocknpu_context* context) {
    if (!context) return kInvalid;
    if (!bind(context)) return kDeviceError;
    const int st = finish(context);
    if (st != kOk) cudaMemset(context->d_status, 0, sizeof(int));
    return st;
}

int rocknpu_b200_prepare_w8(uint32_t kind, const uint8_t* blocks, size_t k, size_t n, int8_t* w_i8, float* scales,
                            int* status, rocknpu_stream stream) {
    if ((kind != 4 && kind != 5 && kind != 6) || !blocks || !w_i8 || !scales || !status || k == 0 || n == 0 ||
        k % 256 != 0 || k > 56 * 1024 || n > 0x7fffffff || reinterpret_cast<uintptr_t>(blocks) % 4 != 0)
        return kInvalid;  // the kernels read the blocks in 4-byte (or wider) words
    rk::launch_prep_w8(static_cast<int>(kind), blocks, static_cast<int>(k), static_cast<int>(n), w_i8, scales, status,
                       static_cast<cudaStream_t>(stream));
    return cuda_status(cudaGetLastError());
}

int rocknpu_b200_quantize_rows(const float* a, size_t m, size_t k, int8_t* a_i8, size_t ld_i8, float* scales,
                               int* status, rocknpu_stream stream) {
    if (!a || !a_i8 || !scales || !status || m == 0 || k == 0 || ld_i8 < k || k > 56 * 1024 || m > 0x7fffffff)
        return kInvalid;
    rk::launch_quant_rows(a, static_cast<int>(m), static_cast<int>(k), static_cast<long long>(k), a_i8,
                          static_cast<long long>(ld_i8), scales, status, static_cast<cudaStream_t>(stream));
    return cuda_status(cudaGetLastError());
}

size_t rocknpu_b200_gemm_workspace_bytes(size_t m, size_t n, size_t k) {
    if (m == 0 || n == 0 || k == 0 || m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff) return 0;
    return gemm_ws_bytes(rk::plan_gemm(0, static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), false));
}

int rocknpu_b200_gemm_w8a8(const int8_t* a_i8, size_t ld_a, const float* a_scales, const int8_t* w_i8, size_t ld_w,
                           const float* w_scales, float* out, size_t ldo, int32_t* acc_out, size_t m, size_t k,
                           size_t n, void* workspace, size_t workspace_bytes, int* status, rocknpu_stream stream) {
    if (!a_i8 || !a_scales || !w_i8 || !w_scales || !out || !status || m == 0 || k == 0 || n == 0 || ld_a < k ||
        ld_w < k || ldo < n || m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff)
        return kInvalid;
    rk::OutMembers om;
    om.count = 1;
    om.n_start[1] = static_cast<int>(n);
    om.out[0] = out;
    om.ldo[0] = static_cast<long long>(ldo);
    const rk::GemmWorkspace gws =
        gemm_ws_view(workspace, workspace_bytes,
                     rk::plan_gemm(0, static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), false));
    const int e = rk::launch_gemm_tc(0, w_i8, static_cast<long long>(ld_w), a_i8, static_cast<long long>(ld_a),
                                     static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), w_scales, a_scales,
                                     om, acc_out, static_cast<long long>(n), status, static_cast<cudaStream_t>(stream),
                                     &gws);
    return e == cudaSuccess ? kOk : (e == cudaErrorInvalidValue ? kInvalid : kExecError);
}

int rocknpu_b200_matmul_w8a8(rocknpu_context* context, const float* a, const int8_t* w_i8, const float* w_scales,
                             float* out, size_t m, size_t k, size_t n, rocknpu_stream stream) {
    if (!context || !a || !w_i8 || !w_scales || !out || m == 0 || k == 0 || n == 0) return kInvalid;
    if (!bind(context)) return kDeviceError;
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : context->stream;
    const size_t ld8 = round_up(k, 16);
    if (context->a_i8.ensure(m * ld8) || context->a_scale.ensure(m * sizeof(float))) return kExecError;
    if (m == 1 && k % 16 == 0 && reinterpret_cast<uintptr_t>(a) % 16 == 0) {
        rk::launch_gemv_w8a8_x(w_i8, w_scales, a, static_cast<int>(k), static_cast<int>(n), out, context->d_status, s);
        return cuda_status(cudaGetLastError());
    }
    if (m == 1 && k % 16 == 0) {
        rk::launch_quant_rows(a, 1, static_cast<int>(k), static_cast<long long>(k), context->a_i8.as<int8_t>(),
                              static_cast<long long>(ld8), context->a_scale.as<float>(), context->d_status, s);
        rk::launch_gemv_w8a8(w_i8, w_scales, context->a_i8.as<int8_t>(), context->a_scale.as<float>(),
                             static_cast<int>(k), static_cast<int>(n), out, s);
        return cuda_status(cudaGetLastError());
    }
    rk::GemmWorkspace gws;
    if (context_ws(context, m, n, k, &gws) != kOk) return kExecError;
    rk::OutMembers om;
    om.count = 1;
    om.n_start[1] = static_cast<int>(n);
    om.out[0] = out;
    om.ldo[0] = static_cast<long long>(n);
    const int e = launch_w8a8(context, w_i8, w_scales, a, m, k, n, context->a_i8.as<int8_t>(), ld8,
                              context->a_scale.as<float>(), om, &gws, s);
    return e == cudaSuccess ? kOk : kExecError;
}

int rocknpu_b200_convert_f16(const float* a, size_t m, size_t k, size_t lda, uint16_t* out, size_t ldo,
                             rocknpu_stream stream) {
    if (!a || !out || m == 0 || k == 0 || lda < k || ldo < k || m > 0x7fffffff || k > 0x7fffffff) return kInvalid;
    rk::launch_f32_to_f16(a, static_cast<int>(m), static_cast<int>(k), static_cast<long long>(lda),
                          reinterpret_cast<__half*>(out), static_cast<long long>(ldo), static_cast<cudaStream_t>(stream));
    return cuda_status(cudaGetLastError());
}

int rocknpu_b200_gemm_f16(const uint16_t* a_f16, size_t ld_a, const uint16_t* w_f16, size_t ld_w, float* out,
                          size_t ldo, size_t m, size_t k, size_t n, int* status, rocknpu_stream stream) {
    if (!a_f16 || !w_f16 || !out || !status || m == 0 || k == 0 || n == 0 || ld_a < k || ld_w < k || ldo < n ||
        m > 0x7fffffff || n > 0x7fffffff)
        return kInvalid;
    rk::OutMembers om;
    om.count = 1;
    om.n_start[1] = static_cast<int>(n);
    om.out[0] = out;
    om.ldo[0] = static_cast<long long>(ldo);
    const int e = rk::launch_gemm_tc(1, w_f16, static_cast<long long>(ld_w * 2), a_f16,
                                     static_cast<long long>(ld_a * 2), static_cast<int>(m), static_cast<int>(n),
                                     static_cast<int>(k), nullptr, nullptr, om, nullptr, 0, status,
                                     static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? kOk : (e == cudaErrorInvalidValue ? kInvalid : kExecError);
}

int rocknpu_b200_gemm_w8a8_gather(const int8_t* a_i8, size_t ld_a, const float* a_scales, const int8_t* w_i8,
                                  size_t ld_w, const float* w_scales, float* const* outs, size_t copies, size_t col0,
                                  size_t ldo, size_t m, size_t k, size_t n_local, int* status, rocknpu_stream stream) {
    if (!a_i8 || !a_scales || !w_i8 || !w_scales || !outs || !status || copies == 0 ||
        copies > static_cast<size_t>(rk::kMaxCopies) || m == 0 || k == 0 || n_local == 0 || ld_a < k ||
        ld_w < k || col0 + n_local > ldo || m > 0x7fffffff || n_local > 0x7fffffff || k > 0x7fffffff)
        return kInvalid;
    rk::OutMembers om;
    om.count = 1;
    om.n_start[1] = static_cast<int>(n_local);
    om.ldo[0] = static_cast<long long>(ldo);
    om.copies = static_cast<int>(copies);
    for (size_t c = 0; c < copies; ++c) {
        if (!outs[c]) return kInvalid;
        om.copy_out[c] = outs[c] + col0;
    }
    om.out[0] = om.copy_out[0];
    const int e = rk::launch_gemm_tc(0, w_i8, static_cast<long long>(ld_w), a_i8, static_cast<long long>(ld_a),
                                     static_cast<int>(m), static_cast<int>(n_local), static_cast<int>(k), w_scales,
                                     a_scales, om, nullptr, 0, status, static_cast<cudaStream_t>(stream), nullptr);
    return e == cudaSuccess ? kOk : (e == cudaErrorInvalidValue ? kInvalid : kExecError);
}

int rocknpu_b200_gemv_w8a8(const int8_t* a_i8, const float* a_scale, const int8_t* w_i8, const float* w_scales,
                           float* out, size_t k, size_t n, rocknpu_stream stream) {
    if (!a_i8 || !a_scale || !w_i8 || !w_scales || !out || k == 0 || n == 0 || k % 16 != 0 || k > 200 * 1024 ||
        n > 0x7fffffff)
        return kInvalid;
    rk::launch_gemv_w8a8(w_i8, w_scales, a_i8, a_scale, static_cast<int>(k), static_cast<int>(n), out,
                         static_cast<cudaStream_t>(stream));
    return cuda_status(cudaGetLastError());
}

size_t rocknpu_b200_kq_layout_bytes(uint32_t kind, size_t k, size_t n) {
    if ((kind != 4 && kind != 6) || k == 0 || k % 256 != 0) return 0;
    return rk::kq_layout_bytes(static_cast<int>(kind), k, n);
}

int rocknpu_b200_kq_layout(uint32_t kind, const uint8_t* blocks, size_t k, size_t n, uint8_t* layout,
                           rocknpu_stream stream) {
    if ((kind != 4 && kind != 6) || !blocks || !layout || k == 0 || n == 0 || k % 256 != 0 || k > 0x7fffffff ||
        n > 0x7fffffff)
        return kInvalid;
    if (kind == 6 && (reinterpret_cast<uintptr_t>(blocks) % 2 || reinterpret_cast<uintptr_t>(layout) % 16))
        return kInvalid;
    return cuda_status(static_cast<cudaError_t>(rk::launch_kq_layout(static_cast<int>(kind), blocks,
                                                                     static_cast<int>(k), static_cast<int>(n), layout,
                                                                     static_cast<cudaStream_t>(stream))));
}

int rocknpu_b200_gemv_kq(uint32_t kind, const uint8_t* layout, size_t k, size_t n, const float* x, float* y,
                         int* status, rocknpu_stream stream) {
    if ((kind != 4 && kind != 6) || !layout || !x || !y || !status || k == 0 || n == 0 || k % 256 != 0 ||
        k > 0x7fffffff || n > 0x7fffffff)
        return kInvalid;
    const int e = rk::launch_gemv_kq(static_cast<int>(kind), layout, static_cast<int>(k), static_cast<int>(n), x, y,
                                     status, static_cast<cudaStream_t>(stream));
    if (e == cudaErrorInvalidValue) return kInvalid;
    return cuda_status(static_cast<cudaError_t>(e));
}

}  // extern "C"

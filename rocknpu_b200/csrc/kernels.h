// Host-side launchers of the sm_100a kernels (device pointers, one stream).
// The C ABI in capi.cpp is the only caller inside the library.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace rk {

enum QKind : int { kQ4K = 4, kQ5K = 5, kQ6K = 6 };

inline size_t qblock_bytes(int kind) {
    return kind == kQ4K ? 144 : kind == kQ5K ? 176 : kind == kQ6K ? 210 : 0;
}

constexpr int kMaxCopies = 16;  // ranks of one node an output tile can go to

// Up to four output members of one concatenated-N GEMM: member i owns the
// weight rows [n_start[i], n_start[i+1]) and writes out[i][m * ldo[i] + col].
// With one member, copies > 1 writes every element to copy_out[0..copies)
// at the same offset instead (copy 0 is usually out[0]): the all-gather of an
// N-sharded GEMM over peer memory.  Launches with copies > 1 do not split K.
struct OutMembers {
    int count = 1;
    int n_start[5] = {0, 0, 0, 0, 0};
    float* out[4] = {nullptr, nullptr, nullptr, nullptr};
    long long ldo[4] = {0, 0, 0, 0};
    int copies = 1;
    float* copy_out[kMaxCopies] = {};
    // no output store once *err != 0 at the start of the epilogue (after the
    // preceding quantiser has finished): outputs in the caller's own host
    // memory stay untouched when a call is rejected
    bool store_guard = false;
};

// K1: Q4_K/Q5_K/Q6_K rows -> int8 rows [n, k] + per-row scales [n].
void launch_prep_w8(int kind, const uint8_t* blocks, int k, int n, int8_t* w, float* scales, int* err,
                    cudaStream_t s);
// K1 (FP16 route): Q rows -> f16 rows [n, ldw] (dequantised, rounded to f16).
void launch_dequant_f16(int kind, const uint8_t* blocks, int k, int n, __half* w, long long ldw, int* err,
                        cudaStream_t s);
// K2: per-token symmetric int8 [m, ld8] + scales [m]; non-finite -> *err.
void launch_quant_rows(const float* a, int m, int k, long long lda, int8_t* a8, long long ld8, float* scales,
                       int* err, cudaStream_t s);
// FP16 executor input: f32 [m, k] -> f16 [m, ldo] (round to nearest even).
void launch_f32_to_f16(const float* a, int m, int k, long long lda, __half* out, long long ldo, cudaStream_t s);

// Split-K workspace of the W8A8 GEMM: int32 partial sums [m][n] and one
// arrival counter per output tile.  Both must be all-zero before the first
// launch; every launch leaves them all-zero again.
struct GemmWorkspace {
    int32_t* ws = nullptr;
    unsigned* counters = nullptr;
    size_t ws_elems = 0, counter_elems = 0;
};

// Per-token quantisation fused into the W8A8 GEMM (K2 in K3's prologue): the
// GEMM's epilogue warps quantise the f32 rows a[m][lda] into a8[m][ld8] +
// scales[m] (ld8 a multiple of 16, a8 16-byte aligned) before their first
// tile, and the activation producer waits per token tile until its rows are
// published.  `sync` holds fused_quant_sync_elems() counters, all zero
// between launches (every launch leaves them zero).  Every CTA of the launch
// must become resident within the 2 s wait limit (true unless another
// long-running kernel holds the GPU's SMs).
struct FusedQuant {
    const float* a = nullptr;
    long long lda = 0;
    int8_t* a8 = nullptr;
    long long ld8 = 0;
    float* scales = nullptr;
    unsigned* sync = nullptr;
    size_t sync_elems = 0;
};
size_t fused_quant_sync_elems(int m, int n, int k);
// Whether to fuse for this shape: only with ROCKNPU_B200_FUSED_QUANT=1, for
// activation matrices up to 8 Mi values with k % 16 == 0 and k <= 16384.
bool fused_quant_enabled(int m, int k);

// Tile plan of one GEMM launch: weight tile rows, token tile height, K
// splits and the workspace a split launch needs.
struct GemmPlan {
    int wt = 128, bt = 128, ksplit = 1, kb_per_split = 1, tiles = 1;
    bool pair = false;  // two-SM (cta_group::2) 256 x bt tiles, gemm_pair.cu
    size_t ws_elems = 0, counter_elems = 0;
};
// allow_pair: the launch may use the two-SM kernel (plain outputs only).
GemmPlan plan_gemm(int kind, int m, int n, int k, bool allow_pair = true);

// K3/K4: out = epilogue(W[n,k] . A[m,k]^T) on tcgen05.  kind 0: int8 inputs,
// int32 accumulators, out = (f32(acc) * a_scale[m]) * w_scale[n]; kind 1:
// f16 inputs, f32 accumulators, out = acc.  ld*_bytes are row pitches
// (multiples of 16).  acc_out (kind 0, optional) receives the raw int32.
// Returns a cudaError_t value.
// A null or too small `ws` runs the launch without K splits.
// With `fq` (kind 0 only) the launch quantises the activations itself: `a`
// must be fq->a8 and `a_scale` fq->scales.
int launch_gemm_tc(int kind, const void* w, long long ldw_bytes, const void* a, long long lda_bytes, int m, int n,
                   int k, const float* w_scale, const float* a_scale, const OutMembers& outs, int32_t* acc_out,
                   long long acc_ld, int* err, cudaStream_t s, const GemmWorkspace* ws = nullptr,
                   const FusedQuant* fq = nullptr);

// K5: M=1 W8A8 GEMV over resident int8 rows.
void launch_gemv_w8a8(const int8_t* w, const float* w_scale, const int8_t* a8, const float* a_scale, int k, int n,
                      float* out, cudaStream_t s);
// K2 + K5 fused for M=1: x f32 (16-byte aligned, k % 16 == 0) quantised per
// CTA with the row quantiser's bits, then the GEMV; kErrNonFinite into *err.
// host_out: out and err are mapped page-locked host memory (written with
// plain stores, the results 32 bytes per CTA).
void launch_gemv_w8a8_x(const int8_t* w, const float* w_scale, const float* x, int k, int n, float* out, int* err,
                        cudaStream_t s, bool host_out = false);

// K5b: M=1 GEMV straight from K-quant blocks (gemv_kq.cu dispatches to
// gemv_q4k.cu / gemv_q6k.cu).  The decode layout of a Q4_K weight is two
// planes, the 128 code bytes of every block [n][k/256][128] then a 16-byte
// header per block (d, dmin, scales and mins regrouped per sub-block pair);
// of a Q6_K weight, 208 bytes per block [n][k/256] (four 48-byte groups of
// ql / qh bytes, then the scales regrouped per group) followed by the f16 d
// values [n][k/256] and 16 bytes of padding.
size_t kq_layout_bytes(int kind, size_t k, size_t n);
int launch_q4k_layout(const uint8_t* blocks, int k, int n, uint8_t* layout, cudaStream_t s);
int launch_gemv_q4k(const uint8_t* layout, int k, int n, const float* x, float* y, int* err, cudaStream_t s,
                    bool host_out = false);
int launch_q6k_layout(const uint8_t* blocks, int k, int n, uint8_t* layout, cudaStream_t s);
int launch_gemv_q6k(const uint8_t* layout, int k, int n, const float* x, float* y, int* err, cudaStream_t s,
                    bool host_out = false);
int launch_kq_layout(int kind, const uint8_t* blocks, int k, int n, uint8_t* layout, cudaStream_t s);
// y[n] = dequant(W) . x in f32; layout and x 16-byte aligned, k % 256 == 0.
// Returns a cudaError_t value.
int launch_gemv_kq(int kind, const uint8_t* layout, int k, int n, const float* x, float* y, int* err,
                   cudaStream_t s, bool host_out = false);

// HILO two-part activations: residual rows res = x - dequant(quant(x)) of
// each f32 row (non-finite -> *err), and the elementwise sum of the two
// output halves.
void launch_hilo_residual(const float* a, int m, int k, long long lda, float* res, long long ldr, int* err,
                          cudaStream_t s);
void launch_add_halves(const float* hi, const float* lo, float* out, long long len, cudaStream_t s);


int sm_count();

}  // namespace rk

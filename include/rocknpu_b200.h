/*
 * rocknpu_b200.h -- what librocknpu.so adds beside the reference C ABI
 * (rocknpu.h).  Five groups:
 *
 *  1. The ggml plugin's host rules (adapters/ggml-rocknpu), exported so a
 *     plugin built against ggml can call them and tests can check them
 *     without ggml: the default route environment and the MUL_MAT
 *     supports_op decision, over a plain description of the node.
 *  2. Device-pointer ("resident") entry points: the same kernels as the
 *     host-pointer ABI, for callers whose tensors already live in HBM
 *     (multi-GPU N-sharding, graph capture, benchmarks).  Every pointer is
 *     a device pointer on the context's GPU, work is queued on `stream`
 *     (NULL = the context's own stream) and the call returns without
 *     waiting.  Kernels report errors in the device word `status`
 *     (0 = ok, 1 = non-finite input, >1 = a device-side wait ran out).
 *     Whenever that word is non-zero after the work has run, the call's
 *     outputs are unspecified (later kernels of the call may have run on
 *     scratch the failed step never wrote); only a zero status vouches for
 *     them.
 *  3. Multi-GPU N-sharding: the row split, the all-gather layout, and peer
 *     (CUDA IPC) buffers for a GEMM whose epilogue all-gathers over NVLink.
 *  4. W8 sidecar files: the plugin's disk cache of prepared int8 weights.
 *  5. Synthetic K-quant weights for tests and benchmarks (host only).
 */
#ifndef ROCKNPU_B200_H
#define ROCKNPU_B200_H

#include <stddef.h>
#include <stdint.h>

#include "rocknpu.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- 1. ggml plugin rules --------------------------------------------- */

/* ggml type ids used by the rules (ggml's GGML_TYPE_* values). */
enum rocknpu_ggml_type {
    ROCKNPU_GGML_F32 = 0,
    ROCKNPU_GGML_F16 = 1,
    ROCKNPU_GGML_Q4_K = 12,
    ROCKNPU_GGML_Q5_K = 13,
    ROCKNPU_GGML_Q6_K = 14,
};

/* The parts of a ggml MUL_MAT node that supports_op reads: src0 = weights
 * [ne0 = k, ne1 = n, ne2, ne3], src1 = activations [k, m, ...], dst. */
typedef struct rocknpu_mul_mat_desc {
    int32_t is_mul_mat;      /* node->op == GGML_OP_MUL_MAT with both sources */
    int32_t weight_type;     /* src0->type */
    int32_t act_type;        /* src1->type */
    int32_t dst_type;        /* node->type */
    int64_t weight_ne[4];
    int64_t act_ne[4];
    int32_t weight_contiguous;
    int32_t act_contiguous;
    int32_t dst_contiguous;
} rocknpu_mul_mat_desc;

/* Set the plugin's validated default routes (setenv without overwrite),
 * as ggml_backend_rocknpu_reg does on registration
 * (ggml-rocknpu.cpp:1859-1871). */
void rocknpu_apply_default_env(void);

/* 1 when the plugin claims the node, 0 otherwise: the decision of
 * rocknpu_mul_mat_supported (ggml-rocknpu.cpp:614-715), environment
 * switches included. */
int rocknpu_mul_mat_supported(const rocknpu_mul_mat_desc *desc);

/* The plugin's graph_compute dispatch (rocknpu_backend_graph_compute,
 * ggml-rocknpu.cpp:978-1650, with rocknpu_mtile_group :838-976) as a planner:
 * given the nodes of one ggml graph split it returns, in order, the C-ABI
 * calls the plugin makes for them, without making them.  What the plugin
 * carries from split to split and from one graph evaluation to the next --
 * the per-layer QKV stash of prompt batches (:32-53, :506-516, :868-928), the
 * decode triple's weight references and stability count (:1185-1258), the
 * pending FFN composite (:1300-1318) -- lives in a rocknpu_graph_state.
 * Decisions assume every call succeeds (the plugin falls back to the
 * per-node path when a group call fails).  The hybrid CPU/NPU split of
 * ROCKNPU_DECODE=hybrid (:400-489) needs ggml's CPU backend and is not
 * planned: with it set, planned calls are the NPU-only forms. */
enum rocknpu_graph_op {
    ROCKNPU_OP_MUL_MAT = 1,
    ROCKNPU_OP_VIEW = 2,  /* GGML_OP_NONE, RESHAPE, VIEW, PERMUTE, TRANSPOSE: nothing to run */
    ROCKNPU_OP_OTHER = 3, /* anything else: graph_compute fails */
};

typedef struct rocknpu_graph_node {
    int32_t op;                  /* rocknpu_graph_op */
    int32_t compute;             /* GGML_TENSOR_FLAG_COMPUTE is set */
    rocknpu_mul_mat_desc desc;   /* MUL_MAT: src0, src1 and dst as supports_op reads them */
    const char *weight_name;     /* src0->name, e.g. "blk.3.attn_q.weight" */
    const void *weight;          /* src0->data: the weight's identity (the caches key on it) */
    size_t weight_bytes;         /* ggml_nbytes(src0) */
    const void *activation;      /* src1: the activation tensor's identity */
    const void *activation_data; /* src1->data */
    int32_t has_w8;              /* a W8 sidecar exists for the weight (rocknpu_w8_sidecar_get succeeds) */
} rocknpu_graph_node;

enum rocknpu_graph_call {
    ROCKNPU_CALL_CONCAT = 1,            /* rocknpu_matmul_q_concat_f32_f32_mtile over the members */
    ROCKNPU_CALL_STASH = 2,             /* the node's output copied from its layer's QKV stash */
    ROCKNPU_CALL_RELEASE = 3,           /* rocknpu_mtile_release of the members' weights */
    ROCKNPU_CALL_OUTPUT_HEAD_NSPLIT = 4,/* rocknpu_matmul_w8a8_f32_f32_m1_nsplit, chunks of 8192 */
    ROCKNPU_CALL_FFN_DEFER = 5,         /* M=1 gate/up kept for the down node (ROCKNPU_FFN_COMPOSITE) */
    ROCKNPU_CALL_SWIGLU_DOWN = 6,       /* rocknpu_matmul_w8a8_swiglu_down_f32 */
    ROCKNPU_CALL_TRIPLE_M1 = 7,         /* q/v/k: rocknpu_matmul_w8a8_triple_f32_f32_m1 (w8) or _q_triple_ */
    ROCKNPU_CALL_PAIR_M1 = 8,           /* gate/up or v/k: rocknpu_matmul_w8a8_pair_f32_f32_m1 (w8) or _q_pair_ */
    ROCKNPU_CALL_PAIR_MTILE = 9,        /* rocknpu_matmul_q_pair_f32_f32_mtile */
    ROCKNPU_CALL_CHUNKED_M16 = 10,      /* m / 16 single calls of 16 rows each */
    ROCKNPU_CALL_SINGLE = 11,           /* rocknpu_matmul_{q4_k,q5_k,q6_k,f16}_f32_f32, or w8a8_f32_f32_m1 (w8) */
    ROCKNPU_CALL_PREWARM = 12,          /* rocknpu_prewarm_quantized_m16 before a CPU fallback */
    ROCKNPU_CALL_CPU_FALLBACK = 13,     /* the whole split to the CPU backend (ROCKNPU_RUNTIME_M16_ROUTER) */
    ROCKNPU_CALL_FAILED = 14,           /* graph_compute returns GGML_STATUS_FAILED at `node` */
};

typedef struct rocknpu_graph_action {
    int32_t call;            /* rocknpu_graph_call */
    int32_t node;            /* the node being dispatched */
    int32_t count;           /* members (1..4) */
    int32_t members[4];      /* node index per member; -1 for a weight held by the layer state */
    const void *weights[4];  /* each member's weight identity */
    int32_t w8;              /* the call's native W8 (sidecar) form */
    int32_t layer;           /* blk.<layer> of a QKV stash or triple decision, -1 otherwise */
    int64_t m, k, n;         /* rows, depth, total output columns of the call */
} rocknpu_graph_action;

typedef struct rocknpu_graph_state rocknpu_graph_state;
/* cpu_fallback: the backend was created with ROCKNPU_RUNTIME_M16_ROUTER set
 * (rocknpu_device_init, ggml-rocknpu.cpp:1687-1703).  NULL on failure. */
rocknpu_graph_state *rocknpu_graph_state_create(int32_t cpu_fallback);
void rocknpu_graph_state_destroy(rocknpu_graph_state *state);
/* Plan one split: writes the calls, in order, into actions[0..capacity) and
 * returns their number; -1 for a NULL argument or too small a capacity
 * (4 * count + 4 always suffices).  Environment switches are read on each
 * call, as the plugin reads them. */
int rocknpu_graph_plan(rocknpu_graph_state *state, const rocknpu_graph_node *nodes, size_t count,
                       rocknpu_graph_action *actions, size_t capacity);

/* ---- 2. device-pointer entry points ------------------------------------ */

/* Opaque CUDA stream (cudaStream_t). */
typedef void *rocknpu_stream;

/* The context's own stream. */
rocknpu_stream rocknpu_b200_context_stream(rocknpu_context *context);

/* 1 when the host-pointer entry points of include/rocknpu.h access the host
 * range [ptr, ptr + bytes) in place instead of copying it: the range lies in
 * one page-locked allocation mapped into the device's address space at its
 * host address (cudaHostAlloc / cudaMallocHost memory).  Then the quantiser
 * (or the FP16 conversion) reads the activations over PCIe and the GEMM
 * epilogue stores the outputs there, overlapping the transfers with the
 * tiles -- when ROCKNPU_B200_ZERO_COPY is "1" (both), "in" or "out"; unset or
 * "0", every host buffer takes the chunked copy pipeline, which measured
 * faster on B200.  0 for pageable memory, which is always copied.  The
 * results are the same bits either way.  An output accessed in place
 * stays untouched when the call is rejected (a non-finite activation), as
 * a copied one does. */
int rocknpu_b200_host_mapped(const void *ptr, size_t bytes);

/* Page-locked host memory for the host-pointer entry points' activations and
 * outputs: `bytes` rounded up to 2 MB, 2 MB-aligned, backed by transparent
 * huge pages where the kernel provides them, registered with CUDA (portable,
 * device-mapped).  Host-to-device copies out of it run at the link rate at
 * every size, where copies out of 4 KB-page pinned memory vary widely.
 * NULL when the memory cannot be mapped or registered (e.g. no GPU). */
void *rocknpu_b200_host_alloc(size_t bytes);

/* Release a rocknpu_b200_host_alloc buffer; INVALID_ARGUMENT for any other
 * pointer.  No copy from or to it may still be in flight. */
int rocknpu_b200_host_free(void *ptr);

/* Wait for the context's stream and turn its device status word (written by
 * rocknpu_b200_matmul_w8a8) into a status code, clearing it. */
int rocknpu_b200_context_check(rocknpu_context *context);

/* Prompt-path (M > 1) weight caches of a context: resident single
 * projections and concatenated groups, the calls that found their prepared
 * weights resident (hits) or prepared them (misses), and the bytes held.  The
 * reference keeps the same caches (decode_mtile_weights,
 * decode_mtile_concat_weights, capi/src/lib.rs:198-236) and counts them in its
 * prompt-path profile (:3900-3996); this exposes them to callers and tests. */
typedef struct rocknpu_b200_prompt_cache_stats {
    size_t single_entries;
    size_t group_entries;
    size_t hits;
    size_t misses;
    size_t resident_bytes;
} rocknpu_b200_prompt_cache_stats;
int rocknpu_b200_context_prompt_cache_stats(const rocknpu_context *context, rocknpu_b200_prompt_cache_stats *out);

/* The status code of a device status word, as the host-pointer entry points
 * return it: 0 -> ROCKNPU_STATUS_OK, 1 (non-finite input) ->
 * ROCKNPU_STATUS_INVALID_ARGUMENT, any other value (a device-side wait that
 * ran out) -> ROCKNPU_STATUS_EXECUTION_ERROR. */
int rocknpu_b200_status_code(int device_status);

/* K1: Q4_K/Q5_K/Q6_K rows (kind 4/5/6, n rows of k values, k % 256 == 0) ->
 * int8 rows w_i8[n][k] + scales[n], bit-identical to the reference's
 * prepare_q*_k_w8a8 (capi/src/lib.rs:711-757, 974-994).  `blocks` must be
 * 4-byte aligned (INVALID_ARGUMENT otherwise); Q4_K blocks at a 16-byte
 * boundary take the faster one-thread-per-sub-block kernel. */
int rocknpu_b200_prepare_w8(uint32_t kind, const uint8_t *blocks, size_t k, size_t n, int8_t *w_i8, float *scales,
                            int *status, rocknpu_stream stream);

/* K2: per-token int8 a_i8[m][ld_i8] + scales[m]
 * (quantize_symmetric_into per row, capi/src/lib.rs:614-654). */
int rocknpu_b200_quantize_rows(const float *a, size_t m, size_t k, int8_t *a_i8, size_t ld_i8, float *scales,
                               int *status, rocknpu_stream stream);

/* Bytes of split-K workspace the W8A8 GEMM of this shape can use (0: the
 * shape runs without K splits). */
size_t rocknpu_b200_gemm_workspace_bytes(size_t m, size_t n, size_t k);

/* K3: out[m][ldo] = (f32(acc) * a_scales[m]) * w_scales[n], acc = exact int32
 * sum_k a_i8[m][k] * w_i8[n][k]; acc_out (optional, [m][n]) receives acc.
 * `workspace` (optional, device memory, all-zero before its first use; every
 * launch leaves it all-zero) lets short-M shapes split K across CTAs; NULL or
 * fewer than rocknpu_b200_gemm_workspace_bytes bytes runs without splits.
 * Launches that share a workspace must not overlap on the GPU.
 * The GEMM is a programmatic dependent launch: it starts streaming the
 * weights (w_i8) before the preceding kernel on `stream` has finished, and
 * reads everything else only after it.  So the weights must already be
 * complete when the GEMM is queued (prepared in an earlier, synchronised
 * step, as the context's caches do), not written by the kernel just before. */
int rocknpu_b200_gemm_w8a8(const int8_t *a_i8, size_t ld_a, const float *a_scales, const int8_t *w_i8,
                           size_t ld_w, const float *w_scales, float *out, size_t ldo, int32_t *acc_out, size_t m,
                           size_t k, size_t n, void *workspace, size_t workspace_bytes, int *status,
                           rocknpu_stream stream);

/* K2 + K3 (+ K5 for m == 1) through the context's workspace: the whole
 * W8A8 MUL_MAT on resident f32 activations and resident prepared weights
 * (complete before the call: see rocknpu_b200_gemm_w8a8).  A NULL `stream`
 * queues the work on the context's own stream (not the legacy default
 * stream); rocknpu_b200_context_check waits for that stream and returns the
 * status word.  Device errors (a non-finite activation) go to the context's
 * status word; `out` is unspecified when it is not 0. */
int rocknpu_b200_matmul_w8a8(rocknpu_context *context, const float *a, const int8_t *w_i8, const float *w_scales,
                             float *out, size_t m, size_t k, size_t n, rocknpu_stream stream);

/* The same W8A8 MUL_MAT as rocknpu_b200_matmul_w8a8, for callers that may not
 * allocate GPU memory once they are running: a runtime whose memory plan is
 * fixed at start-up (a serving loop or an embedded deployment with a static
 * budget), or a framework whose own allocator must own every byte.  This entry point has no counterpart in the
 * reference interface.  It needs no context and calls no cudaMalloc,
 * cudaFree or allocating library routine: the int8 activations, per-token
 * scales and split-K sums live in a 16 MiB array inside the library's device
 * memory, which every GPU that loads the library holds until the process
 * exits.  Limits: k must be a multiple of 16, and m * k + 4 * m (each
 * rounded up to 256 bytes) must fit in those 16 MiB, e.g. m = 2047 at
 * k = 8192; other calls return ROCKNPU_STATUS_INVALID_ARGUMENT before any
 * work is queued (oversized ones also print the sizes to stderr).
 * All pointers are device pointers on the current device; `status` (device,
 * one int) is cleared by the call and set by the kernels like the other
 * device entry points' status words.  When *status is non-zero after the
 * work has run (a non-finite activation, a device wait that ran out), the
 * contents of `out` are unspecified: they may come from another call's
 * leftovers in the shared array.  Work is queued on `stream` and the
 * call returns without waiting.  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress) with that device current;
 * make that first call before any stream capture.  Every call on a device
 * shares the one array, which keeps the last call's contents: calls whose
 * work overlaps on the GPU (other streams, other host threads) race and must
 * be serialised by the caller. */
int rocknpu_b200_matmul_w8a8_noalloc(const float *a, const int8_t *w_i8, const float *w_scales, float *out,
                                     size_t m, size_t k, size_t n, int *status, rocknpu_stream stream);

/* The FP16 executor's activation conversion (Fp16MatmulExecutor::execute_f32,
 * rocknpu-matmul/src/lib.rs:251): f32 a[m][lda] -> f16 out[m][ldo], round to
 * nearest even; columns k..ldo of out are left as they are. */
int rocknpu_b200_convert_f16(const float *a, size_t m, size_t k, size_t lda, uint16_t *out, size_t ldo,
                             rocknpu_stream stream);

/* K4: out[m][ldo] = sum_k f16(a)[m][k] * w_f16[n][k] in f32 on tcgen05;
 * a_f16 row pitch ld_a elements (multiple of 8). */
int rocknpu_b200_gemm_f16(const uint16_t *a_f16, size_t ld_a, const uint16_t *w_f16, size_t ld_w, float *out,
                          size_t ldo, size_t m, size_t k, size_t n, int *status, rocknpu_stream stream);

/* K5: M=1 W8A8 GEMV: out[n] = (f32(acc) * a_scale[0]) * w_scales[n]. */
int rocknpu_b200_gemv_w8a8(const int8_t *a_i8, const float *a_scale, const int8_t *w_i8, const float *w_scales,
                           float *out, size_t k, size_t n, rocknpu_stream stream);

/* K5b: the decode GEMV that reads K-quant blocks directly (Q4_K: kind 4,
 * Q6_K: kind 6; k % 256 == 0): y[n] = sum_k W[n][k] * x[k] with the weights'
 * codes and sub-block scales applied in registers, no tensor cores and no
 * int8 copy of the weight -- a decode step moves 0.5625 (Q4_K) or 0.8203
 * (Q6_K) bytes per weight, the property for which the reference keeps M=1
 * on llama.cpp's K-quant kernels by default (ggml-rocknpu.cpp:305-312).
 * Numerics: each weight is ggml's f32 dequantisation, x is held as 16-bit
 * fixed point per block of 64 (Q4_K: one sub-block pair) or 32 (Q6_K) values
 * (scale = block max / 32767), the code products are exact int32 sums; outputs are within 1e-3 relative (and about
 * 1e-6 of sum |w x|) of the exact dot product of the f32 weights, not
 * bit-identical to a particular summation order.  A non-finite x sets
 * *status to 1 and leaves y unspecified.  `layout` is the weight's decode
 * layout (16-byte aligned, rocknpu_b200_kq_layout); x is 16-byte aligned;
 * k up to 24576 (longer rows return ROCKNPU_STATUS_INVALID_ARGUMENT). */
size_t rocknpu_b200_kq_layout_bytes(uint32_t kind, size_t k, size_t n);
/* Write the decode layout of n rows of ggml blocks (device pointers; the
 * layout 16-byte aligned, Q4_K blocks 16-byte and Q6_K blocks 2-byte
 * aligned): Q4_K two planes, the 128 * k/256 qs bytes of every row [n] --
 * regrouped per step of 8 blocks (nbs blocks in a short last step): 16-byte
 * chunk j of the step's block i at slot (j % 2) * 4 nbs + 4 i + j / 2 --
 * then a 16-byte header per block (the f16 d and dmin, then the 8 scales and
 * 8 mins regrouped per sub-block pair g as the 24-bit value sc[2g] |
 * sc[2g+1] << 6 | m[2g] << 12 | m[2g+1] << 18 at bytes 4 + 3g); Q6_K 208
 * bytes per block [n][k/256] -- four 48-byte groups G = 2h + c holding
 * ql[64h + 16c ..+16], ql[64h + 32 + 16c ..+16], qh[32h + 16c ..+16], then the
 * 16 scales regrouped so that word G holds sc[8h + c + 2t] in byte t -- then
 * the f16 d of every block and 16 bytes of padding.  Same bytes per block as
 * ggml (plus the padding), arranged for 16-byte copies. */
int rocknpu_b200_kq_layout(uint32_t kind, const uint8_t *blocks, size_t k, size_t n, uint8_t *layout,
                           rocknpu_stream stream);
int rocknpu_b200_gemv_kq(uint32_t kind, const uint8_t *layout, size_t k, size_t n, const float *x, float *y,
                         int *status, rocknpu_stream stream);

/* ---- 3. multi-GPU N-sharding (one process per GPU, one node) ----------- */

#define ROCKNPU_B200_MAX_RANKS 16
#define ROCKNPU_B200_IPC_HANDLE_BYTES 64

/* Weight rows (output columns) of rank r: [starts[r], starts[r] + widths[r]).
 * n / 32 blocks of 32 rows split evenly over `world` ranks, remainder blocks
 * to the first ranks (the reference's N split over NPU cores,
 * rocknpu-matmul/src/int8_decode_pool.rs:1484-1491, split_blocks :1505-1522).
 * Ranks beyond the block count get width 0.  Returns the ranks with work. */
size_t rocknpu_b200_shard_rows(size_t n, size_t world, size_t *starts, size_t *widths);

/* All-gather route: rank-major src[world][m][shard_ld] (shard r at
 * src + r * shard_elems, e.g. the output of an NCCL all-gather) ->
 * row-major out[m][ldo] with shard r at columns [starts[r], +widths[r]). */
int rocknpu_b200_gather_shards(const float *src, size_t shard_elems, size_t shard_ld, size_t m, size_t world,
                               const size_t *starts, const size_t *widths, float *out, size_t ldo,
                               rocknpu_stream stream);

/* Peer route.  A peer buffer is `bytes` of device memory on the current GPU
 * that the other ranks of the node map through CUDA IPC.  create() writes
 * this rank's 64-byte handle; the caller exchanges the handles over any host
 * transport (torch.distributed, a file, a socket) and passes all `world` of
 * them, in rank order, to open(). */
typedef struct rocknpu_b200_peer_buffer rocknpu_b200_peer_buffer;
int rocknpu_b200_peer_buffer_create(size_t bytes, int rank, int world, void *handle_out,
                                    rocknpu_b200_peer_buffer **out);
int rocknpu_b200_peer_buffer_open(rocknpu_b200_peer_buffer *buffer, const void *handles);
/* Rank r's data region as mapped in this process (NULL before open()). */
void *rocknpu_b200_peer_buffer_ptr(rocknpu_b200_peer_buffer *buffer, int r);
/* Device-side barrier of all ranks on `stream`: every rank's writes queued
 * before it (peer stores included) are visible to every rank's work queued
 * after it.  Waits are bounded (2 s); a rank that never arrives leaves
 * status 6 in *status. */
int rocknpu_b200_peer_barrier(rocknpu_b200_peer_buffer *buffer, int *status, rocknpu_stream stream);
/* Wait limit of the peer barrier's flag spin for the barriers queued after
 * this call, in milliseconds (1 .. 600000; 0 restores the 2 s default).  The
 * reference bounds its NPU completion wait the same way
 * (rocknpu-matmul/src/int8_decode.rs:13).  A short limit lets a caller (or a
 * test) learn quickly that a rank will not arrive. */
int rocknpu_b200_set_peer_wait_limit_ms(uint32_t ms);
void rocknpu_b200_peer_buffer_destroy(rocknpu_b200_peer_buffer *buffer);

/* K3 with the all-gather fused into the epilogue: this rank's n_local weight
 * rows produce output columns [col0, col0 + n_local), and every element is
 * stored into outs[0..copies) (device pointers, typically every rank's peer
 * buffer data region: [m][ldo] f32) -- the tiles cross NVLink while the
 * tensor cores work on the next ones.  Follow with rocknpu_b200_peer_barrier
 * before reading the outputs. */
int rocknpu_b200_gemm_w8a8_gather(const int8_t *a_i8, size_t ld_a, const float *a_scales, const int8_t *w_i8,
                                  size_t ld_w, const float *w_scales, float *const *outs, size_t copies, size_t col0,
                                  size_t ldo, size_t m, size_t k, size_t n_local, int *status, rocknpu_stream stream);

/* ---- 4. W8 sidecar files (host) ---------------------------------------- */

/* The plugin's disk cache of prepared weights (ggml-rocknpu.cpp:115-259,
 * written by scripts/make_tinyllama_w8_sidecar_gguf.py): <dir>/<name>.w8
 * (int8 [n][k]), <name>.scale.f32 (f32 [n]) and <name>.source.fnv1a64 (16 hex
 * digits, the fingerprint below of the tensor's source bytes). */

/* rocknpu_source_sample_fingerprint (ggml-rocknpu.cpp:123-146): FNV-1a 64
 * over the source length (8 little-endian bytes), then the whole source when
 * it is at most 12288 bytes, else three 4096-byte samples (start, middle,
 * end). */
uint64_t rocknpu_b200_source_fingerprint(const uint8_t *data, size_t bytes);

/* Load a sidecar into host buffers (w8: k * n bytes, scales: n floats), as
 * rocknpu_w8_sidecar_get does (ggml-rocknpu.cpp:212-243): OK when the
 * fingerprint file matches `source`, both data files have exactly the
 * expected size and every scale is finite and positive; otherwise
 * ROCKNPU_STATUS_INVALID_ARGUMENT (the caller prepares the weight instead). */
int rocknpu_b200_w8_sidecar_read(const char *dir, const char *name, const uint8_t *source, size_t source_bytes,
                                 size_t k, size_t n, int8_t *w8, float *scales);

/* Write the three sidecar files for prepared weights of `source` (creating
 * `dir` if needed), byte-compatible with the reference script's output. */
int rocknpu_b200_w8_sidecar_write(const char *dir, const char *name, const uint8_t *source, size_t source_bytes,
                                  size_t k, size_t n, const int8_t *w8, const float *scales);

/* ---- 5. synthetic K-quant weights (host) ------------------------------- */

/* Deterministic N(0, sigma^2) f32 values (counter-based: value i depends only
 * on seed and i, so any slice can be generated independently). */
void rocknpu_synth_normal(uint64_t seed, uint64_t first, size_t count, float sigma, float *out);

/* Encode rows of f32 values (n rows of k, k % 256 == 0) as Q4_K (4), Q5_K (5)
 * or Q6_K (6) superblocks: a simple min/max encoder producing valid blocks
 * (any valid encoding is a valid input; parity starts at the block bytes). */
int rocknpu_synth_encode(uint32_t kind, const float *values, size_t k, size_t n, uint8_t *blocks);

#ifdef __cplusplus
}
#endif

#endif

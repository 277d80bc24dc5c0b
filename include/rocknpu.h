/*
 * rocknpu.h -- the C ABI of the RockNPU MUL_MAT offload, implemented for
 * NVIDIA B200 (sm_100a) by librocknpu.so.
 *
 * Every declaration below keeps the name, argument order, argument meaning
 * and status codes of the reference interface it replaces, so a caller built
 * against the reference header (the ggml plugin adapters/ggml-rocknpu) links
 * against this library unchanged.  Citations are file:line in the
 * darkautism/RockNPU tree (crates/rocknpu-capi/include/rocknpu.h is "H",
 * crates/rocknpu-capi/src/lib.rs is "L").
 *
 * Calls are synchronous: every pointer is a caller-owned HOST pointer that
 * only needs to stay valid for the call, and the output is written when the
 * call returns.  Weights are cached on the GPU keyed by (address, bytes, k,
 * n, kind), so weight buffers must stay immutable for the context's
 * lifetime.  A context is not re-entrant: one caller thread at a time.
 */
#ifndef ROCKNPU_H
#define ROCKNPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Opaque per-device state: CUDA stream, workspaces, resident weights.
 * Replaces H:11 (RockNpuContext, L:198-236). */
typedef struct RockNpuContext rocknpu_context;

/* Decode (M=1) cache counters.  Replaces H:13-25 (L:241-254).  On B200 there
 * is one device per context, so every M=1 call counts as worker1_calls and
 * ksplit_calls stays 0; tuned_shapes counts distinct (k, n) M=1 shapes. */
typedef struct rocknpu_decode_cache_stats {
    size_t hits;
    size_t misses;
    size_t entries;
    size_t resident_bytes;
    uint64_t hit_ns;
    uint64_t miss_ns;
    size_t tuned_shapes;
    size_t worker1_calls;
    size_t worker2_calls;
    size_t worker3_calls;
    size_t ksplit_calls;
} rocknpu_decode_cache_stats;

/* Status codes, H:27-32 (L:22-24).  INVALID_ARGUMENT covers bad pointers and
 * shapes and non-finite activations / dequantised weights; EXECUTION_ERROR a
 * failed CUDA call or a device-side wait that ran out; DEVICE_ERROR no usable
 * GPU. */
enum rocknpu_status {
    ROCKNPU_STATUS_OK = 0,
    ROCKNPU_STATUS_INVALID_ARGUMENT = -1,
    ROCKNPU_STATUS_DEVICE_ERROR = -2,
    ROCKNPU_STATUS_EXECUTION_ERROR = -3,
};

/* Number of usable sm_100 GPUs (H:34, L:3725-3727). */
size_t rocknpu_device_count(void);

/* New context on the current CUDA device; NULL without a GPU (H:35,
 * L:3730-3777). */
rocknpu_context *rocknpu_context_create(void);

/* Copy the decode-cache counters (H:36-38, L:3785-3848). */
int rocknpu_context_decode_cache_stats(const rocknpu_context *context, rocknpu_decode_cache_stats *out);

/* Free all GPU state of a context; NULL is a no-op (H:39, L:3880-3999). */
void rocknpu_context_destroy(rocknpu_context *context);

/* One-shot host callback run after the next M=1 W8 projection (single, pair
 * or triple) has been queued on the GPU and before the call waits for it;
 * NULL clears it (H:41-45, L:3860-3878). */
typedef void (*rocknpu_overlap_fn)(void *user_data);
int rocknpu_context_set_overlap(rocknpu_context *context, rocknpu_overlap_fn callback, void *user_data);

/* 1..4 same-input Q4_K/Q6_K projections (kinds 4/6) as ONE concatenated-N
 * W8A8 GEMM launch; outputs[i] receives [m, ns[i]] (H:46-53,
 * L:2457-2614).  Same limits as the reference: every ns[i] % 32 == 0,
 * 96 <= sum(ns) <= 24576, k % 512 == 0, k <= 4096 (<= 2048 for row tiles
 * taller than 64 rows -- such tiles run as 64-row halves). */
int rocknpu_matmul_q_concat_f32_f32_mtile(rocknpu_context *context, size_t count, const uint8_t *const *weights,
                                          const size_t *bytes, const uint32_t *kinds, const size_t *ns,
                                          const float *activations_mk_f32, float *const *outputs, size_t m,
                                          size_t k);

/* Drop the prompt-path copies of these weights and of every concatenated
 * group that contains one of them, except the group of exactly these weights
 * in this order; decode (M=1) copies are kept (H:55-60, L:2426-2445). */
int rocknpu_mtile_release(rocknpu_context *context, size_t count, const uint8_t *const *weights);

/* Prepare the resident int8 form of a Q4_K (4) / Q6_K (6) weight for the
 * shapes the reference pre-warms, without running a matmul (H:62-68,
 * L:4001-4121). */
int rocknpu_prewarm_quantized_m16(rocknpu_context *context, const uint8_t *weights, size_t weights_bytes,
                                  uint32_t quant_kind, size_t k, size_t n);

/* FP16 executor: out[m, n] = f16(a)[m, k] . w[n, k]^T with f32 accumulation
 * (H:70-77, L:4134-4196). */
int rocknpu_matmul_f16_f32_f32(rocknpu_context *context, const uint16_t *weights_nk_f16_bits,
                               const float *activations_mk_f32, float *output_mn_f32, size_t m, size_t k,
                               size_t n);

/* M=1 W8A8 over caller-prepared int8 rows + scales (H:79-86, L:4207-4251). */
int rocknpu_matmul_w8a8_f32_f32_m1(rocknpu_context *context, const int8_t *weights_nk_i8,
                                   const float *weight_scales_n_f32, const float *activations_k_f32,
                                   float *output_n_f32, size_t k, size_t n);

/* M=16 W8A8 over caller-prepared int8 rows + scales (H:88-95, L:4395-4447). */
int rocknpu_matmul_w8a8_f32_f32_m16(rocknpu_context *context, const int8_t *weights_nk_i8,
                                    const float *weight_scales_n_f32, const float *activations_mk_f32,
                                    float *output_mn_f32, size_t k, size_t n);

/* Wide M=1 W8A8 run as chunk_n-row pieces (H:97-105, L:4259-4300). */
int rocknpu_matmul_w8a8_f32_f32_m1_nsplit(rocknpu_context *context, const int8_t *weights_nk_i8,
                                          const float *weight_scales_n_f32, const float *activations_k_f32,
                                          float *output_n_f32, size_t k, size_t n, size_t chunk_n);

/* M=1 gate/up W8A8, f32 SwiGLU, down W8A8 (H:107-119, L:4308-4389). */
int rocknpu_matmul_w8a8_swiglu_down_f32(rocknpu_context *context, const int8_t *gate_weights_nk_i8,
                                        const float *gate_scales_n_f32, const int8_t *up_weights_nk_i8,
                                        const float *up_scales_n_f32, const int8_t *down_weights_nk_i8,
                                        const float *down_scales_n_f32, const float *activations_k_f32,
                                        float *output_n_f32, size_t projection_k, size_t ffn_n,
                                        size_t output_n);

/* Two M=1 W8A8 projections sharing one activation, one launch (H:121-132,
 * L:4449-4527). */
int rocknpu_matmul_w8a8_pair_f32_f32_m1(rocknpu_context *context, const int8_t *first_weights_nk_i8,
                                        const float *first_scales_n_f32, size_t first_n,
                                        const int8_t *second_weights_nk_i8, const float *second_scales_n_f32,
                                        size_t second_n, const float *activations_k_f32, float *first_output_f32,
                                        float *second_output_f32, size_t k);

/* Two same-input Q projections, equal n in [2048, 8192] (H:134-148,
 * L:4719-4821, L:2616-2781). */
int rocknpu_matmul_q_pair_f32_f32_mtile(rocknpu_context *context, const uint8_t *first_weights, size_t first_bytes,
                                        uint32_t first_kind, size_t first_n, const uint8_t *second_weights,
                                        size_t second_bytes, uint32_t second_kind, size_t second_n,
                                        const float *activations_mk_f32, float *first_output_mn_f32,
                                        float *second_output_mn_f32, size_t m, size_t k);

/* Three M=1 W8A8 projections sharing one activation (H:150-157,
 * L:4529-4631). */
int rocknpu_matmul_w8a8_triple_f32_f32_m1(rocknpu_context *context, const int8_t *first_weights_nk_i8,
                                          const float *first_scales_n_f32, size_t first_n,
                                          const int8_t *second_weights_nk_i8, const float *second_scales_n_f32,
                                          size_t second_n, const int8_t *third_weights_nk_i8,
                                          const float *third_scales_n_f32, size_t third_n,
                                          const float *activations_k_f32, float *first_output_f32,
                                          float *second_output_f32, float *third_output_f32, size_t k);

/* Two M=1 Q projections (kinds 4/6) sharing one activation (H:159-172,
 * L:4633-4717).  B200 option: with ROCKNPU_B200_DECODE_KQ set when the
 * context is created, the M=1 K-quant calls (this one, the triple, and the
 * Q4_K / Q6_K entries at m == 1, k <= 24576) run the K-quant decode GEMV on
 * cached decode layouts: f32 results within 1e-3 relative of the exact
 * product instead of the W8A8 bits. */
int rocknpu_matmul_q_pair_f32_f32_m1(rocknpu_context *context, const uint8_t *first_weights, size_t first_bytes,
                                     uint32_t first_kind, size_t first_n, const uint8_t *second_weights,
                                     size_t second_bytes, uint32_t second_kind, size_t second_n,
                                     const float *activations_k_f32, float *first_output_f32,
                                     float *second_output_f32, size_t k);

/* Three M=1 Q projections sharing one activation (H:174-192, L:4823-4931). */
int rocknpu_matmul_q_triple_f32_f32_m1(rocknpu_context *context, const uint8_t *first_weights, size_t first_bytes,
                                       uint32_t first_kind, size_t first_n, const uint8_t *second_weights,
                                       size_t second_bytes, uint32_t second_kind, size_t second_n,
                                       const uint8_t *third_weights, size_t third_bytes, uint32_t third_kind,
                                       size_t third_n, const float *activations_k_f32, float *first_output_f32,
                                       float *second_output_f32, float *third_output_f32, size_t k);

/* ggml MUL_MAT with Q4_K weights: out[m, n] = a[m, k] . W[n, k]^T
 * (H:194-202, L:4933-5256).  Under the plugin's default routes the W8A8
 * semantics apply (per-row int8 weights, per-token int8 activations, exact
 * int32 sums, f32 rescale); shapes outside those routes use the FP16 route
 * (f16 weights and activations, f32 accumulation); M=1 requires k % 512 == 0,
 * n % 32 == 0 and n <= 8192. */
int rocknpu_matmul_q4_k_f32_f32(rocknpu_context *context, const uint8_t *weights_nk_q4_k, size_t weights_bytes,
                                const float *activations_mk_f32, float *output_mn_f32, size_t m, size_t k,
                                size_t n);

/* Same for Q5_K; prompt batches only (H:204-212, L:5270-5378). */
int rocknpu_matmul_q5_k_f32_f32(rocknpu_context *context, const uint8_t *weights_nk_q5_k, size_t weights_bytes,
                                const float *activations_mk_f32, float *output_mn_f32, size_t m, size_t k,
                                size_t n);

/* Same for Q6_K (H:214-222, L:5380-5671). */
int rocknpu_matmul_q6_k_f32_f32(rocknpu_context *context, const uint8_t *weights_nk_q6_k, size_t weights_bytes,
                                const float *activations_mk_f32, float *output_mn_f32, size_t m, size_t k,
                                size_t n);

#ifdef __cplusplus
}
#endif

#endif

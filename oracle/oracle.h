/*
 * CPU oracle for the RockNPU ggml MUL_MAT offload path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or
 * calls this code; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg do, and there only as the checker / the timed CPU reference.
 *
 * Each function restates the reference's CPU semantics (the RockNPU C ABI is
 * Rust; no Rust toolchain exists here, so the reference cannot be compiled).
 * Citations are relative to the darkautism/RockNPU source tree.
 *
 * Parity pins: the K-quant dequantisation is checked against the installed
 * gguf-py 0.19.0 `quants.py` dequantisers and the W8 preparation against the
 * reference's own `scripts/make_tinyllama_w8_sidecar_gguf.py::quantize_rows`,
 * both through committed golden fixtures (tests/golden/).
 */
#ifndef ROCKNPU_ORACLE_H
#define ROCKNPU_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes of crates/rocknpu-capi/include/rocknpu.h:27-32. */
#define ORC_OK 0
#define ORC_INVALID_ARGUMENT (-1)

/* Q-kinds as the concat entry point encodes them (capi/src/lib.rs:2567-2570),
 * plus 5 for Q5_K. */
#define ORC_Q4_K 4
#define ORC_Q5_K 5
#define ORC_Q6_K 6

size_t orc_block_bytes(uint32_t kind);

float orc_f16_to_f32(uint16_t bits);
uint16_t orc_f32_to_f16(float value);

void orc_dequant_q4_k(const uint8_t *blocks, size_t nblocks, float *out);
void orc_dequant_q5_k(const uint8_t *blocks, size_t nblocks, float *out);
void orc_dequant_q6_k(const uint8_t *blocks, size_t nblocks, float *out);

int orc_quantize_symmetric_into(const float *values, size_t len, int8_t *out, float *scale);

int orc_prepare_w8a8(uint32_t kind, const uint8_t *bytes, size_t nbytes, size_t k, size_t n,
                     int8_t *w_out, float *scales_out);

/* 2: AMX tiles, 1: AVX-512 VNNI, 0: plain loops (the path orc_gemm_i8_i32
 * takes for this shape on this CPU). */
int orc_gemm_path(size_t m, size_t k, size_t n);
void orc_gemm_i8_i32(const int8_t *a, const int8_t *w, int32_t *c, size_t m, size_t k, size_t n);

void orc_rescale_i32_row(const int32_t *values, const float *w_scales, float a_scale, float *out,
                         size_t n);

int orc_quantize_rows(const float *a, size_t m, size_t k, int8_t *a_i8, float *a_scales);

int orc_matmul_w8a8(const int8_t *w, const float *w_scales, const float *a, float *out,
                    int32_t *acc_out, size_t m, size_t k, size_t n);

int orc_matmul_q(uint32_t kind, const uint8_t *bytes, size_t nbytes, const float *a, float *out,
                 int32_t *acc_out, size_t m, size_t k, size_t n);

void orc_matmul_f16(const uint16_t *w_bits, const float *a, float *out, size_t m, size_t k,
                    size_t n);

void orc_swiglu(const float *gate, const float *up, float *out, size_t n);

uint64_t orc_source_fingerprint(const uint8_t *data, size_t bytes);

int orc_hilo_stack(const float *a, size_t m, size_t k, float *stacked);
void orc_hilo_sum(const float *stacked, size_t len, float *out);

size_t orc_split_blocks(size_t blocks, size_t block_width, size_t workers, size_t *starts,
                        size_t *widths);

int orc_threads(void);
/* OpenMP threads for the calls that follow (threads > 0). */
void orc_set_threads(int threads);

/* Synthetic workload inputs (synth.c): N(0, sigma^2) values (value i of a
 * seed depends only on first + i) and min/max K-quant encoders, byte for byte
 * the library's rocknpu_synth_normal / rocknpu_synth_encode. */
void orc_synth_normal(uint64_t seed, uint64_t first, size_t count, float sigma, float *out);
int orc_synth_encode(uint32_t kind, const float *values, size_t k, size_t n, uint8_t *blocks);

#ifdef __cplusplus
}
#endif

#endif

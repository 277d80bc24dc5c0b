// The ggml plugin's host rules (adapters/ggml-rocknpu/src/ggml-rocknpu.cpp),
// restated over a plain node description so they run without ggml.
#include <cstdlib>
#include <cstring>

#include "../../include/rocknpu_b200.h"

namespace {

// rocknpu_env_enabled (ggml-rocknpu.cpp:261-264): set, non-empty, first
// character not '0'.
bool env_on(const char* name) {
    const char* v = std::getenv(name);
    return v != nullptr && v[0] != '\0' && v[0] != '0';
}

// rocknpu_w8_mtile_shape_enabled (ggml-rocknpu.cpp:274-288).
bool w8_shape(long long k, long long n) {
    if (!env_on("ROCKNPU_W8_MTILE")) return false;
    const char* scope = std::getenv("ROCKNPU_W8_MTILE_SCOPE");
    if (scope == nullptr || scope[0] == '\0' || !std::strcmp(scope, "all")) return true;
    if (!std::strcmp(scope, "kv")) return k == 2048 && n == 256;
    if (!std::strcmp(scope, "qo")) return k == 2048 && n == 2048;
    if (!std::strcmp(scope, "ffn")) return (k == 2048 && n == 5632) || (k == 5632 && n == 2048);
    if (!std::strcmp(scope, "attn")) return k == 2048 && (n == 256 || n == 2048);
    if (!std::strcmp(scope, "safe")) return k == 2048 && (n == 256 || n == 5632);
    return false;
}

// rocknpu_native_mtile_routes (ggml-rocknpu.cpp:351-354).
bool native_routes() {
    return env_on("ROCKNPU_NATIVE_MTILE") && env_on("ROCKNPU_MTILE_PERSIST") && env_on("ROCKNPU_W8_MTILE") &&
           env_on("ROCKNPU_MTILE_MC");
}

// rocknpu_small_native_mtile_supported (ggml-rocknpu.cpp:290-303).
bool small_native(long long m, long long k, long long n) {
    if (!(m == 4 || m == 8 || m == 12) || !env_on("ROCKNPU_NATIVE_MTILE") || !env_on("ROCKNPU_MTILE_PERSIST") ||
        !w8_shape(k, n))
        return false;
    if (k == 5632 && n == 2048) return env_on("ROCKNPU_NATIVE_MTILE_DOWN") && env_on("ROCKNPU_MTILE_MC");
    return k > 0 && k <= 4096 && k % 512 == 0 && n > 0 && n <= 8192 && n % 32 == 0;
}

// rocknpu_decode_mode (ggml-rocknpu.cpp:313-322): decode on the CPU unless
// ROCKNPU_DECODE is "npu", "1" or "hybrid".
bool decode_on_cpu() {
    const char* v = std::getenv("ROCKNPU_DECODE");
    if (v == nullptr || v[0] == '\0') return true;
    return !(std::strcmp(v, "npu") == 0 || std::strcmp(v, "1") == 0 || std::strcmp(v, "hybrid") == 0);
}

}  // namespace

extern "C" {

void rocknpu_apply_default_env(void) {
    static const char* const defaults[] = {
        "ROCKNPU_W8_DIRECT_SUBMIT", "ROCKNPU_EXPERIMENT_DIRECT_SCRATCH", "ROCKNPU_PREFILL_CACHE",
        "ROCKNPU_NATIVE_MTILE",     "ROCKNPU_W8_MTILE",                  "ROCKNPU_MTILE_PERSIST",
        "ROCKNPU_MTILE_MC",         "ROCKNPU_NATIVE_MTILE_DOWN",
    };
    for (const char* name : defaults) setenv(name, "1", 0);
}

int rocknpu_mul_mat_supported(const rocknpu_mul_mat_desc* d) {
    if (d == nullptr || !d->is_mul_mat) return 0;
    const int wt = d->weight_type;
    if ((wt != ROCKNPU_GGML_F16 && wt != ROCKNPU_GGML_Q4_K && wt != ROCKNPU_GGML_Q5_K && wt != ROCKNPU_GGML_Q6_K) ||
        d->act_type != ROCKNPU_GGML_F32 || d->dst_type != ROCKNPU_GGML_F32)
        return 0;
    if (!d->weight_contiguous || !d->act_contiguous || !d->dst_contiguous) return 0;
    if (d->weight_ne[2] != 1 || d->weight_ne[3] != 1 || d->act_ne[2] != 1 || d->act_ne[3] != 1) return 0;
    if (d->weight_ne[0] != d->act_ne[0]) return 0;
    const long long k = d->weight_ne[0], n = d->weight_ne[1], m = d->act_ne[1];
    const bool quantized = wt == ROCKNPU_GGML_Q4_K || wt == ROCKNPU_GGML_Q5_K || wt == ROCKNPU_GGML_Q6_K;
    const bool native = native_routes();
    if (wt == ROCKNPU_GGML_Q5_K && !(m > 1 && k <= 4096 && k % 512 == 0 && n % 32 == 0 && n <= 8192 && native))
        return 0;
    if (quantized && m > 1 && n > (native ? 3 * 8192 : 8192)) return 0;
    if (quantized && m > 128 && !env_on("ROCKNPU_PREFILL_CACHE")) return 0;
    if (quantized && m > 1 && env_on("ROCKNPU_SCHED_FFN_ONLY")) {
        const bool gate_up = k == 2048 && n == 5632;
        const bool down = k == 5632 && n == 2048;
        const char* part = std::getenv("ROCKNPU_SCHED_FFN_PART");
        const bool ffn = part != nullptr && !std::strcmp(part, "gateup") ? gate_up
                         : part != nullptr && !std::strcmp(part, "down") ? down
                                                                         : gate_up || down;
        if (!ffn) return 0;
    }
    if (env_on("ROCKNPU_SCHED_CPU_QO") && quantized && m == 16 && k == 2048 && n == 2048) return 0;
    if (env_on("ROCKNPU_M16_ONLY") && m != 16) return 0;
    if (m == 1) {
        if (decode_on_cpu()) return 0;
        if (quantized && n > 8192)
            return env_on("ROCKNPU_NPU_OUTPUT_HEAD") && k > 0 && k % 512 == 0 && n % 32 == 0 && n <= 32768;
        if (env_on("ROCKNPU_SCHED_CPU_QO") && k == 2048 && n == 2048) return 0;
        if (env_on("ROCKNPU_SCHED_CPU_KV") && k == 2048 && n == 256) return 0;
        if (env_on("ROCKNPU_SCHED_CPU_GATEUP") && k == 2048 && n == 5632) return 0;
        if (env_on("ROCKNPU_SCHED_CPU_FFN") && ((k == 2048 && n == 5632) || (k == 5632 && n == 2048))) return 0;
        if (env_on("ROCKNPU_SCHED_CPU_DOWN") && k == 5632 && n == 2048) return 0;
        return quantized && k > 0 && n > 0 && k % 512 == 0 && n % 32 == 0 && n <= 8192;
    }
    if (quantized && native) return k % 256 == 0 && (k + 511) / 512 * 512 <= 3 * 4096 && n % 32 == 0 && n <= 3 * 8192;
    if (quantized && (m == 4 || m == 8 || m == 12)) return small_native(m, k, n);
    const long long k_align = quantized ? 256 : 32;
    return m > 0 && k > 0 && n > 0 && m % 4 == 0 && k % k_align == 0 && n % 16 == 0;
}

}  // extern "C"

// W8 sidecar files: a disk cache of prepared int8 weights.
//
// The ggml plugin can load a weight's int8 rows and per-row scales from
// `<dir>/<tensor name>.w8` and `.scale.f32` instead of preparing them, when
// `<name>.source.fnv1a64` (16 lowercase hex digits) equals a sampled FNV-1a-64
// fingerprint of the tensor's source bytes (ggml-rocknpu.cpp:115-259; written
// by scripts/make_tinyllama_w8_sidecar_gguf.py).  The prepared values are the
// same either way, so the sidecar only saves the preparation time.
//
// Fingerprint: FNV-1a 64 over the 8 little-endian bytes of the source length,
// then over the whole source if it is at most 3 x 4096 bytes, else over three
// 4096-byte samples at the start, the middle ((len - 4096) / 2) and the end.
#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <sys/stat.h>

#include "../../include/rocknpu_b200.h"

namespace {

constexpr uint64_t kFnvOffset = 14695981039346656037ull;
constexpr uint64_t kFnvPrime = 1099511628211ull;
constexpr size_t kSample = 4096;

uint64_t fnv_bytes(uint64_t h, const uint8_t* p, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        h ^= p[i];
        h *= kFnvPrime;
    }
    return h;
}

// Whole file of exactly `bytes` bytes into dst.
bool read_exact(const std::string& path, void* dst, size_t bytes) {
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) return false;
    bool ok = std::fseek(f, 0, SEEK_END) == 0 && std::ftell(f) == static_cast<long>(bytes) &&
              std::fseek(f, 0, SEEK_SET) == 0;
    if (ok && bytes) ok = std::fread(dst, 1, bytes, f) == bytes;
    std::fclose(f);
    return ok;
}

bool write_all(const std::string& path, const void* src, size_t bytes) {
    FILE* f = std::fopen(path.c_str(), "wb");
    if (!f) return false;
    bool ok = bytes == 0 || std::fwrite(src, 1, bytes, f) == bytes;
    ok = (std::fclose(f) == 0) && ok;
    return ok;
}

bool read_fingerprint(const std::string& path, uint64_t* value) {
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) return false;
    char buf[64] = {};
    const size_t got = std::fread(buf, 1, sizeof(buf) - 1, f);
    std::fclose(f);
    // one whitespace-delimited token of exactly 16 hex digits
    size_t a = 0;
    while (a < got && (buf[a] == ' ' || buf[a] == '\n' || buf[a] == '\t' || buf[a] == '\r')) ++a;
    size_t b = a;
    while (b < got && buf[b] != ' ' && buf[b] != '\n' && buf[b] != '\t' && buf[b] != '\r') ++b;
    if (b - a != 16) return false;
    uint64_t v = 0;
    for (size_t i = a; i < b; ++i) {
        const char c = buf[i];
        const int d = c >= '0' && c <= '9' ? c - '0' : c >= 'a' && c <= 'f' ? c - 'a' + 10
                                                   : c >= 'A' && c <= 'F' ? c - 'A' + 10 : -1;
        if (d < 0) return false;
        v = (v << 4) | static_cast<uint64_t>(d);
    }
    *value = v;
    return true;
}

bool scales_ok(const float* s, size_t n) {
    for (size_t i = 0; i < n; ++i)
        if (!std::isfinite(s[i]) || s[i] <= 0.0f) return false;
    return true;
}

std::string base_path(const char* dir, const char* name) { return std::string(dir) + "/" + name; }

}  // namespace

extern "C" {

uint64_t rocknpu_b200_source_fingerprint(const uint8_t* data, size_t bytes) {
    uint64_t h = kFnvOffset;
    const uint64_t count = bytes;
    for (unsigned shift = 0; shift < 64; shift += 8) {
        h ^= static_cast<uint8_t>(count >> shift);
        h *= kFnvPrime;
    }
    if (bytes == 0 || data == nullptr) return h;
    if (bytes <= 3 * kSample) return fnv_bytes(h, data, bytes);
    h = fnv_bytes(h, data, kSample);
    h = fnv_bytes(h, data + (bytes - kSample) / 2, kSample);
    return fnv_bytes(h, data + bytes - kSample, kSample);
}

int rocknpu_b200_w8_sidecar_read(const char* dir, const char* name, const uint8_t* source, size_t source_bytes,
                                 size_t k, size_t n, int8_t* w8, float* scales) {
    if (!dir || !dir[0] || !name || !name[0] || !source || source_bytes == 0 || k == 0 || n == 0 || !w8 || !scales)
        return ROCKNPU_STATUS_INVALID_ARGUMENT;
    const std::string base = base_path(dir, name);
    uint64_t expected = 0;
    if (!read_fingerprint(base + ".source.fnv1a64", &expected) ||
        expected != rocknpu_b200_source_fingerprint(source, source_bytes))
        return ROCKNPU_STATUS_INVALID_ARGUMENT;  // missing or stale for this source
    if (!read_exact(base + ".w8", w8, k * n) || !read_exact(base + ".scale.f32", scales, n * sizeof(float)) ||
        !scales_ok(scales, n))
        return ROCKNPU_STATUS_INVALID_ARGUMENT;
    return ROCKNPU_STATUS_OK;
}

int rocknpu_b200_w8_sidecar_write(const char* dir, const char* name, const uint8_t* source, size_t source_bytes,
                                  size_t k, size_t n, const int8_t* w8, const float* scales) {
    if (!dir || !dir[0] || !name || !name[0] || !source || source_bytes == 0 || k == 0 || n == 0 || !w8 ||
        !scales || !scales_ok(scales, n))
        return ROCKNPU_STATUS_INVALID_ARGUMENT;
    if (std::strchr(name, '/') != nullptr) return ROCKNPU_STATUS_INVALID_ARGUMENT;
    if (mkdir(dir, 0755) != 0 && errno != EEXIST) return ROCKNPU_STATUS_EXECUTION_ERROR;
    const std::string base = base_path(dir, name);
    char hex[18];
    std::snprintf(hex, sizeof(hex), "%016llx\n",
                  static_cast<unsigned long long>(rocknpu_b200_source_fingerprint(source, source_bytes)));
    if (!write_all(base + ".w8", w8, k * n) || !write_all(base + ".scale.f32", scales, n * sizeof(float)) ||
        !write_all(base + ".source.fnv1a64", hex, 17))
        return ROCKNPU_STATUS_EXECUTION_ERROR;
    return ROCKNPU_STATUS_OK;
}

}  // extern "C"

// Synthetic K-quant weights for tests and benchmarks (host only): a
// counter-based normal generator and simple min/max encoders that emit valid
// Q4_K / Q5_K / Q6_K superblocks in ggml's block layout.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/rocknpu_b200.h"

namespace {

uint64_t mix64(uint64_t x) {  // splitmix64 finaliser
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

uint16_t to_half(float f) {  // round to nearest even, finite inputs
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const int e = static_cast<int>((x >> 23) & 0xFF) - 127 + 15;
    uint32_t man = x & 0x7FFFFFu;
    if (e >= 31) return static_cast<uint16_t>(sign | 0x7BFFu);  // clamp to max finite
    if (e <= 0) {
        if (e < -10) return static_cast<uint16_t>(sign);
        man |= 0x800000u;
        const int shift = 14 - e;
        uint32_t h = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1))) ++h;
        return static_cast<uint16_t>(sign | h);
    }
    uint32_t h = sign | (static_cast<uint32_t>(e) << 10) | (man >> 13);
    const uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) ++h;
    return static_cast<uint16_t>(h);
}

float from_half(uint16_t h) {
    const uint32_t sign = (h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1F, man = h & 0x3FF, bits;
    if (e == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            int s = -1;
            do {
                man <<= 1;
                ++s;
            } while (!(man & 0x400));
            bits = sign | (static_cast<uint32_t>(127 - 15 - s) << 23) | ((man & 0x3FF) << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((e + 112) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

void put_half(uint8_t* p, float v) {
    const uint16_t h = to_half(v);
    p[0] = static_cast<uint8_t>(h & 0xFF);
    p[1] = static_cast<uint8_t>(h >> 8);
}

int clampi(long v, int lo, int hi) { return static_cast<int>(std::min<long>(hi, std::max<long>(lo, v))); }

// Q4_K (levels = 15) and Q5_K (levels = 31): 8 sub-blocks of 32 with an
// unsigned code, a 6-bit scale and a 6-bit min per sub-block.
void encode_qk_asym(const float* x, uint8_t* blk, int levels) {
    float scale[8], minv[8];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; ++j) {
        float lo = 0.0f, hi = 0.0f;
        for (int l = 0; l < 32; ++l) {
            lo = std::min(lo, x[32 * j + l]);
            hi = std::max(hi, x[32 * j + l]);
        }
        scale[j] = (hi - lo) / static_cast<float>(levels);
        minv[j] = -lo;
        max_scale = std::max(max_scale, scale[j]);
        max_min = std::max(max_min, minv[j]);
    }
    const uint16_t dh = to_half(max_scale / 63.0f), mh = to_half(max_min / 63.0f);
    const float d = from_half(dh), dmin = from_half(mh);
    int sc[8], mn[8];
    for (int j = 0; j < 8; ++j) {
        sc[j] = d > 0 ? clampi(std::lround(scale[j] / d), 0, 63) : 0;
        mn[j] = dmin > 0 ? clampi(std::lround(minv[j] / dmin), 0, 63) : 0;
    }
    blk[0] = static_cast<uint8_t>(dh & 0xFF);
    blk[1] = static_cast<uint8_t>(dh >> 8);
    blk[2] = static_cast<uint8_t>(mh & 0xFF);
    blk[3] = static_cast<uint8_t>(mh >> 8);
    uint8_t* s = blk + 4;
    for (int j = 0; j < 4; ++j) {
        s[j] = static_cast<uint8_t>((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = static_cast<uint8_t>((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
        s[j + 8] = static_cast<uint8_t>((sc[j + 4] & 0xF) | ((mn[j + 4] & 0xF) << 4));
    }
    int q[256];
    for (int j = 0; j < 8; ++j) {
        const float dj = d * static_cast<float>(sc[j]), mj = dmin * static_cast<float>(mn[j]);
        for (int l = 0; l < 32; ++l)
            q[32 * j + l] = dj > 0 ? clampi(std::lround((x[32 * j + l] + mj) / dj), 0, levels) : 0;
    }
    if (levels == 15) {
        uint8_t* qs = blk + 16;
        for (int g = 0; g < 4; ++g)
            for (int l = 0; l < 32; ++l) qs[32 * g + l] = static_cast<uint8_t>(q[64 * g + l] | (q[64 * g + 32 + l] << 4));
    } else {
        uint8_t* qh = blk + 16;
        uint8_t* qs = blk + 48;
        std::memset(qh, 0, 32);
        for (int g = 0; g < 4; ++g)
            for (int l = 0; l < 32; ++l) {
                const int lo = q[64 * g + l], hi = q[64 * g + 32 + l];
                qs[32 * g + l] = static_cast<uint8_t>((lo & 0xF) | ((hi & 0xF) << 4));
                qh[l] |= static_cast<uint8_t>(((lo >> 4) & 1) << (2 * g));
                qh[l] |= static_cast<uint8_t>(((hi >> 4) & 1) << (2 * g + 1));
            }
    }
}

// Q6_K: 16 sub-blocks of 16 with a signed 6-bit code and an int8 scale.
void encode_q6k(const float* x, uint8_t* blk) {
    float scale[16], max_scale = 0.0f;
    for (int j = 0; j < 16; ++j) {
        float amax = 0.0f;
        for (int l = 0; l < 16; ++l) amax = std::max(amax, std::fabs(x[16 * j + l]));
        scale[j] = amax / 31.0f;
        max_scale = std::max(max_scale, scale[j]);
    }
    const uint16_t dh = to_half(max_scale / 127.0f);
    const float d = from_half(dh);
    int8_t sc[16];
    for (int j = 0; j < 16; ++j) sc[j] = static_cast<int8_t>(d > 0 ? clampi(std::lround(scale[j] / d), -128, 127) : 0);
    int q[256];
    for (int v = 0; v < 256; ++v) {
        const float dj = d * static_cast<float>(sc[v / 16]);
        q[v] = (dj != 0 ? clampi(std::lround(x[v] / dj), -32, 31) : 0) + 32;
    }
    uint8_t* ql = blk;
    uint8_t* qh = blk + 128;
    std::memset(ql, 0, 128);
    std::memset(qh, 0, 64);
    for (int v = 0; v < 256; ++v) {
        const int h = v >> 7, t = (v >> 5) & 3, l = v & 31;
        ql[64 * h + 32 * (t & 1) + l] |= static_cast<uint8_t>((q[v] & 0xF) << (4 * (t >> 1)));
        qh[32 * h + l] |= static_cast<uint8_t>(((q[v] >> 4) & 3) << (2 * t));
    }
    std::memcpy(blk + 192, sc, 16);
    blk[208] = static_cast<uint8_t>(dh & 0xFF);
    blk[209] = static_cast<uint8_t>(dh >> 8);
}

template <class F>
void parallel_for(size_t n, F&& f) {
    const size_t workers = std::max<size_t>(1, std::min<size_t>(std::thread::hardware_concurrency(), 64));
    if (n < 1024 || workers == 1) {
        f(0, n);
        return;
    }
    std::vector<std::thread> ts;
    const size_t per = (n + workers - 1) / workers;
    for (size_t w = 0; w < workers; ++w) {
        const size_t a = w * per, b = std::min(n, a + per);
        if (a < b) ts.emplace_back([&f, a, b] { f(a, b); });
    }
    for (auto& t : ts) t.join();
}

}  // namespace

extern "C" {

void rocknpu_synth_normal(uint64_t seed, uint64_t first, size_t count, float sigma, float* out) {
    parallel_for(count, [&](size_t a, size_t b) {
        for (size_t i = a; i < b; ++i) {
            const uint64_t r = mix64(seed * 0xD1B54A32D192ED03ull ^ mix64(first + i));
            const double u1 = (static_cast<double>(r >> 11) + 0.5) * (1.0 / 9007199254740992.0);
            const double u2 = static_cast<double>(mix64(r) >> 11) * (1.0 / 9007199254740992.0);
            out[i] = static_cast<float>(sigma * std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2));
        }
    });
}

int rocknpu_synth_encode(uint32_t kind, const float* values, size_t k, size_t n, uint8_t* blocks) {
    if (!values || !blocks || k == 0 || k % 256 != 0 || (kind != 4 && kind != 5 && kind != 6)) return -1;
    const size_t bb = kind == 4 ? 144 : kind == 5 ? 176 : 210;
    const size_t nblocks = n * (k / 256);
    parallel_for(nblocks, [&](size_t a, size_t b) {
        for (size_t i = a; i < b; ++i) {
            const float* x = values + i * 256;
            uint8_t* blk = blocks + i * bb;
            if (kind == 6)
                encode_q6k(x, blk);
            else
                encode_qk_asym(x, blk, kind == 4 ? 15 : 31);
        }
    });
    return 0;
}

}  // extern "C"

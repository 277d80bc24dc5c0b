/*
 * Synthetic workload inputs for the CPU reference arm.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).  bench.py's `--impl reference`
 * run builds its K-quant weights and activations here, so that the timed
 * reference process loads only liboracle.so.  The values and block bytes are
 * the same as the library's own generator (the counter-based normal sampler
 * and the min/max K-quant encoders behind rocknpu_synth_normal /
 * rocknpu_synth_encode); tests/test_oracle.py checks that both produce
 * identical bytes.  The arithmetic is spelled out below:
 *
 *  - value i of seed s: r = mix(s * 0xD1B54A32D192ED03 ^ mix(first + i)) with
 *    the splitmix64 finaliser `mix`; u1 = ((r >> 11) + 0.5) / 2^53,
 *    u2 = (mix(r) >> 11) / 2^53; x = (float)(sigma * sqrt(-2 ln u1) *
 *    cos(2 pi u2)) (Box-Muller in double);
 *  - Q4_K / Q5_K: per 32-value sub-block scale = (max - min) / levels and
 *    min = -lo (lo = min(0, values)); d = f16(max scale / 63), dmin =
 *    f16(max min / 63); 6-bit codes round(scale / d), round(min / dmin);
 *    q = round((x + dmin * m) / (d * sc)) clamped to [0, levels];
 *  - Q6_K: per 16-value sub-block scale = absmax / 31; d = f16(max / 127);
 *    int8 sub-scales round(scale / d); q = round(x / (d * sc)) clamped to
 *    [-32, 31], stored + 32.
 * Blocks are laid out as ggml's block_q4_K / block_q5_K / block_q6_K.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <omp.h>

#include "oracle.h"

static uint64_t syn_mix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

static int syn_clamp(long v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : (int)v; }

/* f32 -> f16 bits, round to nearest even; finite values beyond the f16
 * range clamp to the largest finite f16 (the library generator's rule). */
static uint16_t syn_to_half(float v) {
    const uint16_t h = orc_f32_to_f16(v);
    if ((h & 0x7FFFu) == 0x7C00u && isfinite(v)) return (uint16_t)((h & 0x8000u) | 0x7BFFu);
    return h;
}

static void syn_put_half(uint8_t *p, uint16_t h) {
    p[0] = (uint8_t)(h & 0xFF);
    p[1] = (uint8_t)(h >> 8);
}

void orc_synth_normal(uint64_t seed, uint64_t first, size_t count, float sigma, float *out) {
    const long long cnt = (long long)count;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < cnt; ++i) {
        const uint64_t r = syn_mix64(seed * 0xD1B54A32D192ED03ull ^ syn_mix64(first + (uint64_t)i));
        const double u1 = ((double)(r >> 11) + 0.5) * (1.0 / 9007199254740992.0);
        const double u2 = (double)(syn_mix64(r) >> 11) * (1.0 / 9007199254740992.0);
        out[i] = (float)(sigma * sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
    }
}

/* Q4_K (levels 15) and Q5_K (levels 31): 8 sub-blocks of 32. */
static void syn_encode_asym(const float *x, uint8_t *blk, int levels) {
    float scale[8], minv[8];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; ++j) {
        float lo = 0.0f, hi = 0.0f;
        for (int l = 0; l < 32; ++l) {
            const float v = x[32 * j + l];
            lo = v < lo ? v : lo;
            hi = v > hi ? v : hi;
        }
        scale[j] = (hi - lo) / (float)levels;
        minv[j] = -lo;
        max_scale = scale[j] > max_scale ? scale[j] : max_scale;
        max_min = minv[j] > max_min ? minv[j] : max_min;
    }
    const uint16_t dh = syn_to_half(max_scale / 63.0f), mh = syn_to_half(max_min / 63.0f);
    const float d = orc_f16_to_f32(dh), dmin = orc_f16_to_f32(mh);
    int sc[8], mn[8];
    for (int j = 0; j < 8; ++j) {
        sc[j] = d > 0 ? syn_clamp(lroundf(scale[j] / d), 0, 63) : 0;
        mn[j] = dmin > 0 ? syn_clamp(lroundf(minv[j] / dmin), 0, 63) : 0;
    }
    syn_put_half(blk, dh);
    syn_put_half(blk + 2, mh);
    uint8_t *s = blk + 4;
    for (int j = 0; j < 4; ++j) {
        s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((mn[j + 4] & 0xF) << 4));
    }
    int q[256];
    for (int j = 0; j < 8; ++j) {
        const float dj = d * (float)sc[j], mj = dmin * (float)mn[j];
        for (int l = 0; l < 32; ++l)
            q[32 * j + l] = dj > 0 ? syn_clamp(lroundf((x[32 * j + l] + mj) / dj), 0, levels) : 0;
    }
    if (levels == 15) {
        uint8_t *qs = blk + 16;
        for (int g = 0; g < 4; ++g)
            for (int l = 0; l < 32; ++l) qs[32 * g + l] = (uint8_t)(q[64 * g + l] | (q[64 * g + 32 + l] << 4));
    } else {
        uint8_t *qh = blk + 16;
        uint8_t *qs = blk + 48;
        memset(qh, 0, 32);
        for (int g = 0; g < 4; ++g)
            for (int l = 0; l < 32; ++l) {
                const int lo = q[64 * g + l], hi = q[64 * g + 32 + l];
                qs[32 * g + l] = (uint8_t)((lo & 0xF) | ((hi & 0xF) << 4));
                qh[l] |= (uint8_t)(((lo >> 4) & 1) << (2 * g));
                qh[l] |= (uint8_t)(((hi >> 4) & 1) << (2 * g + 1));
            }
    }
}

/* Q6_K: 16 sub-blocks of 16, signed 6-bit codes, int8 sub-scales. */
static void syn_encode_q6k(const float *x, uint8_t *blk) {
    float scale[16], max_scale = 0.0f;
    for (int j = 0; j < 16; ++j) {
        float amax = 0.0f;
        for (int l = 0; l < 16; ++l) {
            const float a = fabsf(x[16 * j + l]);
            amax = a > amax ? a : amax;
        }
        scale[j] = amax / 31.0f;
        max_scale = scale[j] > max_scale ? scale[j] : max_scale;
    }
    const uint16_t dh = syn_to_half(max_scale / 127.0f);
    const float d = orc_f16_to_f32(dh);
    int8_t sc[16];
    for (int j = 0; j < 16; ++j) sc[j] = (int8_t)(d > 0 ? syn_clamp(lroundf(scale[j] / d), -128, 127) : 0);
    int q[256];
    for (int v = 0; v < 256; ++v) {
        const float dj = d * (float)sc[v / 16];
        q[v] = (dj != 0 ? syn_clamp(lroundf(x[v] / dj), -32, 31) : 0) + 32;
    }
    uint8_t *ql = blk;
    uint8_t *qh = blk + 128;
    memset(ql, 0, 128);
    memset(qh, 0, 64);
    for (int v = 0; v < 256; ++v) {
        const int h = v >> 7, t = (v >> 5) & 3, l = v & 31;
        ql[64 * h + 32 * (t & 1) + l] |= (uint8_t)((q[v] & 0xF) << (4 * (t >> 1)));
        qh[32 * h + l] |= (uint8_t)(((q[v] >> 4) & 3) << (2 * t));
    }
    memcpy(blk + 192, sc, 16);
    syn_put_half(blk + 208, dh);
}

int orc_synth_encode(uint32_t kind, const float *values, size_t k, size_t n, uint8_t *blocks) {
    if (!values || !blocks || k == 0 || k % 256 != 0 || (kind != 4 && kind != 5 && kind != 6)) return ORC_INVALID_ARGUMENT;
    const size_t bb = orc_block_bytes(kind);
    const long long nblocks = (long long)(n * (k / 256));
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < nblocks; ++i) {
        const float *x = values + (size_t)i * 256;
        uint8_t *blk = blocks + (size_t)i * bb;
        if (kind == 6)
            syn_encode_q6k(x, blk);
        else
            syn_encode_asym(x, blk, kind == 4 ? 15 : 31);
    }
    return ORC_OK;
}

void orc_set_threads(int threads) {
    if (threads > 0) omp_set_num_threads(threads);
}

/*
 * CPU oracle for the RockNPU ggml MUL_MAT offload path.
 *
 * TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and the
 * CPU-baseline leg of bench.py as the checker and the timed CPU reference,
 * never by the shipped library.  Compiled with -ffp-contract=off so that every
 * f32 expression rounds after each operation, as Rust (the reference's host
 * language) evaluates it.
 *
 * Citations are file:line inside the darkautism/RockNPU tree.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif


/* Grow-only per-thread scratch for the oracle's large temporaries: fresh
 * multi-MB allocations fault in page by page on every call, which on some
 * hosts costs more than the arithmetic being measured.  Each calling thread
 * keeps its own buffers, so the oracle stays reentrant across threads. */
static void *orc_scratch(void **slot, size_t *cap, size_t bytes) {
    if (bytes > *cap) {
        free(*slot);
        *slot = malloc(bytes);
        *cap = *slot ? bytes : 0;
    }
    return *slot;
}

#define QK_K 256

int orc_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ggml block sizes, pinned by capi/src/lib.rs:5729-5736 (144, 210); Q5_K is
 * d, dmin, 12 scale bytes, 32 high-bit bytes and 128 nibble bytes. */
size_t orc_block_bytes(uint32_t kind) {
    switch (kind) {
    case ORC_Q4_K: return 144;
    case ORC_Q5_K: return 176;
    case ORC_Q6_K: return 210;
    default: return 0;
    }
}

/* IEEE binary16 -> binary32, exact (the `half` crate's f16::to_f32). */
float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            /* subnormal: normalise */
            int e = -1;
            do {
                man <<= 1;
                e++;
            } while ((man & 0x400u) == 0);
            man &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* IEEE binary32 -> binary16 with round-to-nearest-even (f16::from_f32, used
 * for the activations at capi/src/lib.rs:4180-4184). */
uint16_t orc_f32_to_f16(float value) {
    uint32_t x;
    memcpy(&x, &value, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp == 0xff) {
        if (man == 0) return (uint16_t)(sign | 0x7c00u);
        return (uint16_t)(sign | 0x7e00u | (man >> 13));
    }
    int e = (int)exp - 127 + 15;
    if (e >= 0x1f) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        /* subnormal result */
        uint32_t full = man | 0x800000u;
        int shift = 14 - e;
        uint32_t half_man = full >> shift;
        uint32_t rem = full & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (half_man & 1u))) half_man++;
        return (uint16_t)(sign | half_man);
    }
    uint32_t half_man = man >> 13;
    uint32_t rem = man & 0x1fffu;
    uint32_t out = sign | ((uint32_t)e << 10) | half_man;
    if (rem > 0x1000u || (rem == 0x1000u && (half_man & 1u))) out++;
    return (uint16_t)out;
}

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* The 6-bit scale/min pair j of a Q4_K/Q5_K superblock (ggml's K-quant block
 * format, as gguf-py quants.py Q4_K.get_scale_min unpacks it). */
static inline void scale_min_k4(int j, const uint8_t *s, uint8_t *sc, uint8_t *m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (uint8_t)((s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4));
        *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

/* Q4_K dequantisation (third-party llama-gguf 0.14.0 `dequantize_q4_k`,
 * called at capi/src/lib.rs:732-733): value = (d*sc)*q - (dmin*m), f32. */
void orc_dequant_q4_k(const uint8_t *blocks, size_t nblocks, float *out) {
    for (size_t b = 0; b < nblocks; ++b) {
        const uint8_t *blk = blocks + b * 144;
        const float d = orc_f16_to_f32(rd16(blk));
        const float dmin = orc_f16_to_f32(rd16(blk + 2));
        const uint8_t *scales = blk + 4;
        const uint8_t *qs = blk + 16;
        float *y = out + b * QK_K;
        for (int g = 0; g < 4; ++g) {
            uint8_t sc, m;
            scale_min_k4(2 * g, scales, &sc, &m);
            const float d1 = d * (float)sc, m1 = dmin * (float)m;
            scale_min_k4(2 * g + 1, scales, &sc, &m);
            const float d2 = d * (float)sc, m2 = dmin * (float)m;
            for (int l = 0; l < 32; ++l) y[64 * g + l] = d1 * (float)(qs[32 * g + l] & 0x0f) - m1;
            for (int l = 0; l < 32; ++l) y[64 * g + 32 + l] = d2 * (float)(qs[32 * g + l] >> 4) - m2;
        }
    }
}

/* Q5_K dequantisation (llama-gguf `dequantize_q5_k`, capi/src/lib.rs:759-806). */
void orc_dequant_q5_k(const uint8_t *blocks, size_t nblocks, float *out) {
    for (size_t b = 0; b < nblocks; ++b) {
        const uint8_t *blk = blocks + b * 176;
        const float d = orc_f16_to_f32(rd16(blk));
        const float dmin = orc_f16_to_f32(rd16(blk + 2));
        const uint8_t *scales = blk + 4;
        const uint8_t *qh = blk + 16;
        const uint8_t *qs = blk + 48;
        float *y = out + b * QK_K;
        for (int s = 0; s < 8; ++s) {
            uint8_t sc, m;
            scale_min_k4(s, scales, &sc, &m);
            const float ds = d * (float)sc, ms = dmin * (float)m;
            const int g = s >> 1, shift = (s & 1) * 4;
            for (int l = 0; l < 32; ++l) {
                int q = ((qs[32 * g + l] >> shift) & 0x0f) | (((qh[l] >> s) & 1) << 4);
                y[32 * s + l] = ds * (float)q - ms;
            }
        }
    }
}

/* Q6_K dequantisation (llama-gguf `dequantize_q6_k`, capi/src/lib.rs:986-988):
 * value = (d*sc[v/16])*q, q = 6-bit - 32. */
void orc_dequant_q6_k(const uint8_t *blocks, size_t nblocks, float *out) {
    for (size_t b = 0; b < nblocks; ++b) {
        const uint8_t *blk = blocks + b * 210;
        const uint8_t *ql = blk;
        const uint8_t *qh = blk + 128;
        const int8_t *sc = (const int8_t *)(blk + 192);
        const float d = orc_f16_to_f32(rd16(blk + 208));
        float *y = out + b * QK_K;
        for (int v = 0; v < QK_K; ++v) {
            const int h = v >> 7, t = (v >> 5) & 3, l = v & 31;
            const int lo = (ql[64 * h + 32 * (t & 1) + l] >> (4 * (t >> 1))) & 0x0f;
            const int hi = (qh[32 * h + l] >> (2 * t)) & 3;
            const int q = (lo | (hi << 4)) - 32;
            y[v] = (d * (float)sc[v >> 4]) * (float)q;
        }
    }
}

/* quantize_symmetric_into, scalar branch (capi/src/lib.rs:614-654): reject
 * non-finite, scale = max|x|/127 (1.0 for an all-zero row),
 * q = round_half_away(x/scale) clamped to +-127. */
int orc_quantize_symmetric_into(const float *values, size_t len, int8_t *out, float *scale) {
    float max_abs = 0.0f;
    for (size_t i = 0; i < len; ++i) {
        if (!isfinite(values[i])) return ORC_INVALID_ARGUMENT;
        float a = fabsf(values[i]);
        if (a > max_abs) max_abs = a;
    }
    const float s = max_abs == 0.0f ? 1.0f : max_abs / 127.0f;
    for (size_t i = 0; i < len; ++i) {
        float q = roundf(values[i] / s);
        if (q < -127.0f) q = -127.0f;
        if (q > 127.0f) q = 127.0f;
        out[i] = (int8_t)q;
    }
    *scale = s;
    return ORC_OK;
}

/* prepare_q4_k_w8a8 / prepare_q5_k_w8a8 / prepare_q6_k_w8a8
 * (capi/src/lib.rs:711-757, 759-806, 974-994): dequantise each weight row,
 * then quantize_symmetric_into over the full row. */
int orc_prepare_w8a8(uint32_t kind, const uint8_t *bytes, size_t nbytes, size_t k, size_t n,
                     int8_t *w_out, float *scales_out) {
    const size_t bb = orc_block_bytes(kind);
    if (bb == 0 || k == 0 || n == 0 || k % QK_K != 0) return ORC_INVALID_ARGUMENT;
    const size_t row_bytes = (k / QK_K) * bb;
    if (nbytes != n * row_bytes) return ORC_INVALID_ARGUMENT;
    int status = ORC_OK;
#pragma omp parallel
    {
        float *row = (float *)malloc(k * sizeof(float));
#pragma omp for schedule(static)
        for (long r = 0; r < (long)n; ++r) {
            const uint8_t *src = bytes + (size_t)r * row_bytes;
            if (kind == ORC_Q4_K) orc_dequant_q4_k(src, k / QK_K, row);
            else if (kind == ORC_Q5_K) orc_dequant_q5_k(src, k / QK_K, row);
            else orc_dequant_q6_k(src, k / QK_K, row);
            if (orc_quantize_symmetric_into(row, k, w_out + (size_t)r * k, scales_out + r) != ORC_OK) {
#pragma omp atomic write
                status = ORC_INVALID_ARGUMENT;
            }
        }
        free(row);
    }
    return status;
}

/* Exact int8 x int8 -> int32 product C[M,N] = A[M,K] . W[N,K]^T, the NPU
 * M-tile's arithmetic (rocknpu-matmul/src/int8_decode.rs:221-516, oracle form
 * of rocket-smoke/src/bin/int8_decode_m1.rs:38-45).  Sums use wrapping int32
 * like the K-split host accumulation (capi/src/lib.rs:1906-1914); for
 * |x| <= 127 and K <= 2^17 no wrap occurs. */
#if defined(__x86_64__)
#include <cpuid.h>
#include <immintrin.h>
#include <sys/syscall.h>
#include <unistd.h>

/* The same exact product with AVX-512 VNNI (the CPU baseline's fast path):
 * vpdpbusd multiplies unsigned by signed bytes, so A is offset to a + 128
 * (a ^ 0x80) and 128 * sum_k w[j][k] is subtracted afterwards -- exact in
 * int32 for |values| <= 127 and k <= 2^17.  4 x 4 output tiles, 64 bytes of
 * K per step; masked loads cover the K tail (masked W bytes are zero, so the
 * offset A bytes there multiply to zero). */
__attribute__((target("avx512f,avx512bw,avx512vnni")))
static void gemm_vnni(const int8_t *a, const int8_t *w, int32_t *c, size_t m, size_t k, size_t n) {
    int32_t *wsum = (int32_t *)malloc(n * sizeof(int32_t));
#pragma omp parallel for schedule(static)
    for (long j = 0; j < (long)n; ++j) {
        int32_t t = 0;
        for (size_t kk = 0; kk < k; ++kk) t += w[(size_t)j * k + kk];
        wsum[j] = t;
    }
    const long rb = (long)((m + 3) / 4), cb = (long)((n + 3) / 4);
    const __m512i flip = _mm512_set1_epi8((char)0x80);
#pragma omp parallel for schedule(dynamic, 4) collapse(2)
    for (long jb = 0; jb < cb; ++jb) {
        for (long ib = 0; ib < rb; ++ib) {
            const int8_t *ar[4], *wr[4];
            for (int t = 0; t < 4; ++t) {
                size_t i = (size_t)ib * 4 + t, j = (size_t)jb * 4 + t;
                ar[t] = a + (i < m ? i : m - 1) * k;
                wr[t] = w + (j < n ? j : n - 1) * k;
            }
            __m512i acc[4][4];
            for (int x = 0; x < 4; ++x)
                for (int y = 0; y < 4; ++y) acc[x][y] = _mm512_setzero_si512();
            for (size_t kk = 0; kk < k; kk += 64) {
                const size_t left = k - kk;
                const __mmask64 mask = left >= 64 ? ~(__mmask64)0 : (((__mmask64)1 << left) - 1);
                __m512i va[4], vw[4];
                for (int t = 0; t < 4; ++t) {
                    va[t] = _mm512_xor_si512(_mm512_maskz_loadu_epi8(mask, ar[t] + kk), flip);
                    vw[t] = _mm512_maskz_loadu_epi8(mask, wr[t] + kk);
                }
                for (int x = 0; x < 4; ++x)
                    for (int y = 0; y < 4; ++y) acc[x][y] = _mm512_dpbusd_epi32(acc[x][y], va[x], vw[y]);
            }
            for (int x = 0; x < 4; ++x) {
                const size_t i = (size_t)ib * 4 + x;
                if (i >= m) continue;
                for (int y = 0; y < 4; ++y) {
                    const size_t j = (size_t)jb * 4 + y;
                    if (j >= n) continue;
                    c[i * n + j] = _mm512_reduce_add_epi32(acc[x][y]) - 128 * wsum[j];
                }
            }
        }
    }
    free(wsum);
}
#endif

/* The same exact product on AMX tiles (tdpbssd: signed x signed bytes, four
 * per int32 lane, exact int32 accumulation).  A is copied zero-padded to
 * 32-row / 64-byte blocks; W is packed once per call into the tile layout of
 * the B operand (row r of a 16-column, 64-byte-deep block holds, for each of
 * the 16 columns, its 4 bytes at depth 4r..4r+3).  Each thread computes 32 x 32
 * blocks of C in four accumulator tiles. */
#define ORC_ARCH_REQ_XCOMP_PERM 0x1023
#define ORC_XFEATURE_XTILEDATA 18

static int amx_ready(void) {
    static int state = -1;
    if (state >= 0) return state;
    unsigned eax = 0, ebx = 0, ecx = 0, edx = 0;
    state = 0;
    if (!__get_cpuid_count(7, 0, &eax, &ebx, &ecx, &edx)) return state;
    if (!((edx >> 24) & 1) || !((edx >> 25) & 1)) return state; /* AMX-TILE, AMX-INT8 */
    if (syscall(SYS_arch_prctl, ORC_ARCH_REQ_XCOMP_PERM, ORC_XFEATURE_XTILEDATA) != 0) return state;
    state = 1;
    return state;
}

struct orc_tilecfg {
    uint8_t palette_id;
    uint8_t start_row;
    uint8_t reserved[14];
    uint16_t colsb[16];
    uint8_t rows[16];
};

__attribute__((target("amx-tile,amx-int8")))
static void gemm_amx(const int8_t *a, const int8_t *w, int32_t *c, size_t m, size_t k, size_t n) {
    const size_t kp = (k + 63) / 64 * 64, mp = (m + 31) / 32 * 32, np = (n + 31) / 32 * 32;
    const size_t kb = kp / 64;
    static __thread void *ap_buf, *wp_buf;
    static __thread size_t ap_cap, wp_cap;
    int8_t *ap = (int8_t *)orc_scratch(&ap_buf, &ap_cap, mp * kp);
    int8_t *wp = (int8_t *)orc_scratch(&wp_buf, &wp_cap, np * kp);
    if (!ap || !wp) abort();
    /* zero padding: A's rows past m and columns past k, W's packed bytes past n or k */
#pragma omp parallel for schedule(static)
    for (long i = 0; i < (long)mp; ++i) {
        if (i < (long)m) {
            memcpy(ap + (size_t)i * kp, a + (size_t)i * k, k);
            memset(ap + (size_t)i * kp + k, 0, kp - k);
        } else {
            memset(ap + (size_t)i * kp, 0, kp);
        }
    }
    if (np != n || kp != k) memset(wp, 0, np * kp);
    /* wp[(t * kb + b) * 1024 + r * 64 + q * 4 + e] = w[t*16 + q][b*64 + 4r + e] */
#pragma omp parallel for schedule(static) collapse(2)
    for (long t = 0; t < (long)(np / 16); ++t) {
        for (long b = 0; b < (long)kb; ++b) {
            int8_t *blk = wp + ((size_t)t * kb + (size_t)b) * 1024;
            const size_t k0 = (size_t)b * 64;
            for (int q = 0; q < 16; ++q) {
                const size_t col = (size_t)t * 16 + q;
                if (col >= n) continue;
                const int8_t *src = w + col * k + k0;
                if (k - k0 >= 64) {
                    for (int r = 0; r < 16; ++r) memcpy(blk + r * 64 + q * 4, src + 4 * r, 4);
                } else {
                    for (size_t kk = 0; kk < k - k0; ++kk) blk[(kk / 4) * 64 + q * 4 + kk % 4] = src[kk];
                }
            }
        }
    }
    struct orc_tilecfg cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.palette_id = 1;
    for (int t = 0; t < 8; ++t) {
        cfg.rows[t] = 16;
        cfg.colsb[t] = 64;
    }
    const long mblocks = (long)(mp / 32), nblocks = (long)(np / 32);
#pragma omp parallel
    {
        _tile_loadconfig(&cfg);
        int32_t out[32 * 32];
#pragma omp for schedule(dynamic, 2) collapse(2)
        for (long mb = 0; mb < mblocks; ++mb) {
            for (long nb = 0; nb < nblocks; ++nb) {
                _tile_zero(0);
                _tile_zero(1);
                _tile_zero(2);
                _tile_zero(3);
                const int8_t *a0 = ap + (size_t)mb * 32 * kp;
                const int8_t *b0 = wp + (size_t)(nb * 2) * kb * 1024;
                const int8_t *b1 = wp + (size_t)(nb * 2 + 1) * kb * 1024;
                for (size_t b = 0; b < kb; ++b) {
                    _tile_loadd(4, a0 + b * 64, kp);
                    _tile_loadd(5, a0 + 16 * kp + b * 64, kp);
                    _tile_loadd(6, b0 + b * 1024, 64);
                    _tile_loadd(7, b1 + b * 1024, 64);
                    _tile_dpbssd(0, 4, 6);
                    _tile_dpbssd(1, 4, 7);
                    _tile_dpbssd(2, 5, 6);
                    _tile_dpbssd(3, 5, 7);
                }
                _tile_stored(0, out, 128);
                _tile_stored(1, out + 16, 128);
                _tile_stored(2, out + 16 * 32, 128);
                _tile_stored(3, out + 16 * 32 + 16, 128);
                for (int i = 0; i < 32; ++i) {
                    const size_t row = (size_t)mb * 32 + i;
                    if (row >= m) break;
                    const size_t col0 = (size_t)nb * 32;
                    const size_t cols = n - col0 < 32 ? n - col0 : 32;
                    memcpy(c + row * n + col0, out + i * 32, cols * sizeof(int32_t));
                }
            }
        }
        _tile_release();
    }
}

/* Which path orc_gemm_i8_i32 takes for this shape: 2 AMX, 1 AVX-512 VNNI,
 * 0 the plain loops. */
int orc_gemm_path(size_t m, size_t k, size_t n) {
#if defined(__x86_64__)
    const char *force = getenv("ORACLE_SCALAR_GEMM");
    const char *path = getenv("ORACLE_GEMM_PATH");
    const int scalar = (force && force[0] == '1') || (path && !strcmp(path, "scalar"));
    const int want_vnni = path && !strcmp(path, "vnni");
    const int want_amx = path && !strcmp(path, "amx");
    if (!scalar && !want_vnni && k <= ((size_t)1 << 17) && (want_amx || (m >= 16 && n >= 16)) && amx_ready())
        return 2;
    if (!scalar && k <= ((size_t)1 << 17) && __builtin_cpu_supports("avx512f") &&
        __builtin_cpu_supports("avx512bw") && __builtin_cpu_supports("avx512vnni"))
        return 1;
#endif
    (void)m, (void)k, (void)n;
    return 0;
}

/* ORACLE_GEMM_PATH = amx | vnni | scalar forces one path (all give the same
 * exact int32 results); ORACLE_SCALAR_GEMM=1 is the same as "scalar". */
void orc_gemm_i8_i32(const int8_t *a, const int8_t *w, int32_t *c, size_t m, size_t k, size_t n) {
#if defined(__x86_64__)
    const int path = orc_gemm_path(m, k, n);
    if (path == 2) {
        gemm_amx(a, w, c, m, k, n);
        return;
    }
    if (path == 1) {
        gemm_vnni(a, w, c, m, k, n);
        return;
    }
#endif
    const size_t NB = 16;
#pragma omp parallel for schedule(dynamic, 1) collapse(2)
    for (long nb = 0; nb < (long)((n + NB - 1) / NB); ++nb) {
        for (long row = 0; row < (long)m; ++row) {
            const int8_t *ar = a + (size_t)row * k;
            const size_t n0 = (size_t)nb * NB;
            const size_t n1 = n0 + NB < n ? n0 + NB : n;
            for (size_t col = n0; col < n1; ++col) {
                const int8_t *wr = w + col * k;
                int32_t acc = 0;
                for (size_t kk = 0; kk < k; ++kk) acc += (int32_t)((int16_t)ar[kk] * (int16_t)wr[kk]);
                c[(size_t)row * n + col] = acc;
            }
        }
    }
}

/* rescale_i32_row, scalar branch (capi/src/lib.rs:692-709):
 * out = (f32)acc * a_scale * w_scale, evaluated left to right. */
void orc_rescale_i32_row(const int32_t *values, const float *w_scales, float a_scale, float *out,
                         size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = (float)values[i] * a_scale * w_scales[i];
}

/* Per-token quantisation of an [M,K] activation block
 * (capi/src/lib.rs:1776-1791). */
int orc_quantize_rows(const float *a, size_t m, size_t k, int8_t *a_i8, float *a_scales) {
    int status = ORC_OK;
#pragma omp parallel for schedule(static)
    for (long r = 0; r < (long)m; ++r) {
        if (orc_quantize_symmetric_into(a + (size_t)r * k, k, a_i8 + (size_t)r * k, a_scales + r) != ORC_OK) {
#pragma omp atomic write
            status = ORC_INVALID_ARGUMENT;
        }
    }
    return status;
}

/* W8A8 with prepared int8 weights: quantise rows, int32 GEMM, rescale
 * (execute_cached_w8a8_mtile_pool_padded, capi/src/lib.rs:1731-1989, and
 * execute_cached_w8a8_m1, capi/src/lib.rs:1567-1701). */
int orc_matmul_w8a8(const int8_t *w, const float *w_scales, const float *a, float *out,
                    int32_t *acc_out, size_t m, size_t k, size_t n) {
    static __thread void *a8_buf, *as_buf, *acc_buf;
    static __thread size_t a8_cap, as_cap, acc_cap;
    int8_t *a8 = (int8_t *)orc_scratch(&a8_buf, &a8_cap, m * k);
    float *as = (float *)orc_scratch(&as_buf, &as_cap, m * sizeof(float));
    int32_t *acc = acc_out ? acc_out : (int32_t *)orc_scratch(&acc_buf, &acc_cap, m * n * sizeof(int32_t));
    if (!a8 || !as || !acc) abort();
    int status = orc_quantize_rows(a, m, k, a8, as);
    if (status == ORC_OK) {
        orc_gemm_i8_i32(a8, w, acc, m, k, n);
#pragma omp parallel for schedule(static)
        for (long r = 0; r < (long)m; ++r)
            orc_rescale_i32_row(acc + (size_t)r * n, w_scales, as[r], out + (size_t)r * n, n);
    }
    return status;
}

/* rocknpu_matmul_q{4,5,6}_k_f32_f32 (capi/src/lib.rs:4933-5256, 5270, 5380-5671)
 * with the plugin's default routes: argument validation, then the W8A8
 * semantics every M-tile route shares (row chunking, K padding and N/K splits
 * leave the per-element result unchanged: padded rows/columns are zero and
 * discarded, K partials are exact int32). */
int orc_matmul_q(uint32_t kind, const uint8_t *bytes, size_t nbytes, const float *a, float *out,
                 int32_t *acc_out, size_t m, size_t k, size_t n) {
    const size_t bb = orc_block_bytes(kind);
    if (bb == 0 || !bytes || !a || !out || m == 0 || k == 0 || n == 0 || k % QK_K != 0)
        return ORC_INVALID_ARGUMENT;
    if (nbytes != n * (k / QK_K) * bb) return ORC_INVALID_ARGUMENT;
    int8_t *w = (int8_t *)malloc(n * k);
    float *ws = (float *)malloc(n * sizeof(float));
    int status = orc_prepare_w8a8(kind, bytes, nbytes, k, n, w, ws);
    if (status == ORC_OK) status = orc_matmul_w8a8(w, ws, a, out, acc_out, m, k, n);
    free(w);
    free(ws);
    return status;
}

/* cpu_reference_fp32 (rocknpu-matmul/src/lib.rs:1680-1699) behind
 * rocknpu_matmul_f16_f32_f32 (capi/src/lib.rs:4134-4196): activations are
 * rounded to f16 (round-nearest-even), products are exact in f64 and the
 * K-sum is accumulated in f64, then narrowed to f32. */
void orc_matmul_f16(const uint16_t *w_bits, const float *a, float *out, size_t m, size_t k,
                    size_t n) {
    double *ad = (double *)malloc(m * k * sizeof(double));
#pragma omp parallel for schedule(static)
    for (long i = 0; i < (long)(m * k); ++i) ad[i] = (double)orc_f16_to_f32(orc_f32_to_f16(a[i]));
#pragma omp parallel
    {
        double *wrow = (double *)malloc(k * sizeof(double));
#pragma omp for schedule(dynamic, 4)
        for (long col = 0; col < (long)n; ++col) {
            for (size_t kk = 0; kk < k; ++kk) wrow[kk] = (double)orc_f16_to_f32(w_bits[(size_t)col * k + kk]);
            for (size_t row = 0; row < m; ++row) {
                const double *ar = ad + row * k;
                double acc = 0.0;
                for (size_t kk = 0; kk < k; ++kk) acc += ar[kk] * wrow[kk];
                out[row * n + (size_t)col] = (float)acc;
            }
        }
        free(wrow);
    }
    free(ad);
}

/* F32 SwiGLU between the gate/up and down projections of
 * rocknpu_matmul_w8a8_swiglu_down_f32 (capi/src/lib.rs:4368-4373). */
void orc_swiglu(const float *gate, const float *up, float *out, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        const float g = gate[i];
        const float sig = 1.0f / (1.0f + expf(-g));
        out[i] = g * sig * up[i];
    }
}

/* hilo_stack (capi/src/lib.rs:2045-2070): rows [x; residual(x)] of the
 * two-part activation encoding, residual = x - f32(q) * scale with q, scale
 * from quantize_symmetric_into (two f32 roundings, no fused multiply-add).
 * `stacked` is [2m][k]; returns ORC_INVALID_ARGUMENT when a row does not
 * quantise (non-finite), where the reference takes its normal path. */
int orc_hilo_stack(const float *a, size_t m, size_t k, float *stacked) {
    int status = ORC_OK;
    memcpy(stacked, a, m * k * sizeof(float));
#pragma omp parallel
    {
        int8_t *q = (int8_t *)malloc(k);
#pragma omp for schedule(static)
        for (long r = 0; r < (long)m; ++r) {
            const float *x = a + (size_t)r * k;
            float *res = stacked + (m + (size_t)r) * k;
            float scale;
            if (orc_quantize_symmetric_into(x, k, q, &scale) != ORC_OK) {
#pragma omp atomic write
                status = ORC_INVALID_ARGUMENT;
                continue;
            }
            for (size_t i = 0; i < k; ++i) {
                const float back = (float)q[i] * scale;
                res[i] = x[i] - back;
            }
        }
        free(q);
    }
    return status;
}

/* hilo_sum (capi/src/lib.rs:2073-2083): out[i] = hi[i] + lo[i] over the two
 * halves of the stacked output [2][len]. */
void orc_hilo_sum(const float *stacked, size_t len, float *out) {
    for (size_t i = 0; i < len; ++i) out[i] = stacked[i] + stacked[len + i];
}

/* rocknpu_source_sample_fingerprint (adapters/ggml-rocknpu/src/
 * ggml-rocknpu.cpp:123-146; the sidecar script's source_sample_fnv1a64):
 * FNV-1a 64 over the length's 8 little-endian bytes, then all bytes up to
 * 3 * 4096, else 4096-byte samples at 0, (len - 4096) / 2 and len - 4096. */
uint64_t orc_source_fingerprint(const uint8_t *data, size_t bytes) {
    const uint64_t prime = 1099511628211ULL;
    uint64_t h = 14695981039346656037ULL;
    for (unsigned shift = 0; shift < 64; shift += 8) {
        h ^= (uint8_t)((uint64_t)bytes >> shift);
        h *= prime;
    }
    size_t starts[3], counts[3], parts;
    if (bytes <= 3 * 4096) {
        starts[0] = 0; counts[0] = bytes; parts = 1;
    } else {
        starts[0] = 0; counts[0] = 4096;
        starts[1] = (bytes - 4096) / 2; counts[1] = 4096;
        starts[2] = bytes - 4096; counts[2] = 4096;
        parts = 3;
    }
    for (size_t p = 0; p < parts; ++p)
        for (size_t i = 0; i < counts[p]; ++i) {
            h ^= data[starts[p] + i];
            h *= prime;
        }
    return h;
}

/* split_blocks (rocknpu-matmul/src/int8_decode_pool.rs:1505-1522): an even
 * split of `blocks` blocks over `workers`, remainder to the first workers. */
size_t orc_split_blocks(size_t blocks, size_t block_width, size_t workers, size_t *starts,
                        size_t *widths) {
    if (workers == 0 || blocks == 0) return 0;
    const size_t active = workers < blocks ? workers : blocks;
    const size_t base = blocks / active, extra = blocks % active;
    size_t start = 0;
    for (size_t w = 0; w < active; ++w) {
        const size_t width = (base + (w < extra ? 1 : 0)) * block_width;
        starts[w] = start;
        widths[w] = width;
        start += width;
    }
    return active;
}

/*
 * CPU oracle for the prefill MUL_MAT path: TEST INFRASTRUCTURE ONLY (see
 * zest_oracle.h). Compiled with -ffp-contract=off so that every float
 * expression rounds exactly where the C source says it does.
 */
#include "zest_oracle.h"

#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ------------------------------------------------------------------------ */
/* bfp16 codec                                                              */
/* ------------------------------------------------------------------------ */

/* x86 cvtps2dq under the default rounding mode: round to nearest even, and
 * the "integer indefinite" 0x80000000 for NaN or anything outside int32. */
static int32_t cvt_rne_i32(float v) {
    if (v != v) return INT32_MIN;
    if (v >= 2147483648.0f || v < -2147483648.0f) return INT32_MIN;
    return (int32_t) nearbyintf(v);
}

/* bfp16_encode_block, AVX2 path (src/npu/bfp16_pack.cpp:85-114), which is
 * what the reference's Linux and Windows builds compile (-mavx2): the block
 * exponent is the largest biased exponent byte of the eight; when the scale
 * 2^(133-maxe) is a normal float every value is multiplied by it (exact) and
 * rounded to nearest even, NaN/Inf giving 0x80000000, then clamped to
 * [-128,127]. Blocks of (signed) zeros are nine zero bytes (:108-112). Tiny
 * exponents (maxe <= 5) take the scalar path (:115-126). */
void zo_encode_block(const float *x, uint8_t *out) {
    uint32_t mx = 0;
    for (int i = 0; i < 8; i++) {
        uint32_t e = (f2u(x[i]) >> 23) & 0xffu;
        if (e > mx) mx = e;
    }
    const int sexp = 133 - (int) mx + 127;
    if (sexp >= 1 && sexp <= 254) {
        out[0] = (uint8_t) mx;
        const float scale = u2f((uint32_t) sexp << 23);
        for (int i = 0; i < 8; i++) {
            int32_t q = cvt_rne_i32(x[i] * scale);
            if (q < -128) q = -128;
            if (q > 127) q = 127;
            out[1 + i] = (uint8_t) (int8_t) q;
        }
        return;
    }
    uint32_t any = 0;
    for (int i = 0; i < 8; i++) any |= f2u(x[i]) & 0x7fffffffu;
    if (!any) {
        memset(out, 0, ZO_BLOCK_BYTES);
        return;
    }
    out[0] = (uint8_t) mx;
    const int sh = 133 - (int) mx;
    for (int i = 0; i < 8; i++) {
        float q = nearbyintf(ldexpf(x[i], sh));
        /* std::min(127, std::max(-128, q)) */
        q = (-128.0f < q) ? q : -128.0f;
        q = (q < 127.0f) ? q : 127.0f;
        out[1 + i] = (uint8_t) (int8_t) q;
    }
}

/* bfp16_decode_block (src/npu/bfp16_pack.cpp:129-144): mantissa * 2^(e-133) */
void zo_decode_block(const uint8_t *in, float *x) {
    if (in[0] >= 7) {
        const float scale = u2f((uint32_t) ((int) in[0] - 133 + 127) << 23);
        for (int i = 0; i < 8; i++) x[i] = (float) (int8_t) in[1 + i] * scale;
        return;
    }
    const int sh = (int) in[0] - 133;
    for (int i = 0; i < 8; i++) x[i] = ldexpf((float) (int8_t) in[1 + i], sh);
}

void zo_encode_blocks(const float *x, int64_t n, uint8_t *out) {
    for (int64_t b = 0; b < n; b++) zo_encode_block(x + 8 * b, out + ZO_BLOCK_BYTES * b);
}

void zo_decode_blocks(const uint8_t *in, int64_t n, float *x) {
    for (int64_t b = 0; b < n; b++) zo_decode_block(in + ZO_BLOCK_BYTES * b, x + 8 * b);
}

/* ------------------------------------------------------------------------ */
/* tile layouts                                                             */
/* ------------------------------------------------------------------------ */

/* Position of block column cb of tile row rr inside one tile: 16-row pairs,
 * then block columns, then the 16 rows (src/npu/bfp16_pack.cpp:29-36,172-175). */
static int64_t in_tile(int64_t rr, int64_t cb, const zo_tiling *t) {
    const int64_t tkb = t->k / 8;
    return ((rr / 16) * tkb + cb % tkb) * 16 + rr % 16;
}

/* bfp16_a_offset (src/npu/bfp16_pack.cpp:177-180): A is m-row blocks, each a
 * run of K/k tiles of m x k. */
size_t zo_a_offset(int64_t r, int64_t cb, int64_t K, const zo_tiling *t) {
    const int64_t nk = K / t->k;
    const int64_t tile = (r / t->m) * nk + cb / (t->k / 8);
    return (size_t) (tile * t->m * (t->k / 8) + in_tile(r % t->m, cb, t)) * ZO_BLOCK_BYTES;
}

/* bfp16_b_offset (src/npu/bfp16_pack.cpp:182-186): B is, per array column c,
 * its n-row groups (rows (c + cols*t)*n onward), each a run of K/k tiles. */
size_t zo_b_offset(int64_t r, int64_t cb, int64_t N, int64_t K, const zo_tiling *t) {
    const int64_t per_col = N / t->n / t->cols, nk = K / t->k, g = r / t->n;
    const int64_t tile = ((g % t->cols) * per_col + g / t->cols) * nk + cb / (t->k / 8);
    return (size_t) (tile * t->n * (t->k / 8) + in_tile(r % t->n, cb, t)) * ZO_BLOCK_BYTES;
}

/* bfp16_pack_a / bfp16_pack_b (src/npu/bfp16_pack.cpp:146-163) */
void zo_pack_a(const float *x, int64_t M, int64_t K, const zo_tiling *t, uint8_t *out) {
    for (int64_t r = 0; r < M; r++)
        for (int64_t cb = 0; cb < K / 8; cb++) zo_encode_block(x + r * K + cb * 8, out + zo_a_offset(r, cb, K, t));
}

void zo_pack_b(const float *w, int64_t N, int64_t K, const zo_tiling *t, uint8_t *out) {
    for (int64_t r = 0; r < N; r++)
        for (int64_t cb = 0; cb < K / 8; cb++) zo_encode_block(w + r * K + cb * 8, out + zo_b_offset(r, cb, N, K, t));
}

/* bfp16_unpack_a / bfp16_unpack_b (src/npu/bfp16_pack.cpp:239-245) */
void zo_unpack_a(const uint8_t *in, int64_t M, int64_t K, const zo_tiling *t, float *x) {
    for (int64_t r = 0; r < M; r++)
        for (int64_t cb = 0; cb < K / 8; cb++) zo_decode_block(in + zo_a_offset(r, cb, K, t), x + r * K + cb * 8);
}

void zo_unpack_b(const uint8_t *in, int64_t N, int64_t K, const zo_tiling *t, float *w) {
    for (int64_t r = 0; r < N; r++)
        for (int64_t cb = 0; cb < K / 8; cb++) zo_decode_block(in + zo_b_offset(r, cb, N, K, t), w + r * K + cb * 8);
}

/* bfp16_interleave_gate_up (src/npu/bfp16_pack.cpp:231-237): 8 gate rows,
 * then the 8 up rows that pair with them. */
void zo_interleave_gate_up(const float *gate, const float *up, int64_t F, int64_t K, float *out) {
    for (int64_t i = 0; i < F; i++) {
        const int64_t at = (i / 8) * 16 + i % 8;
        memcpy(out + at * K, gate + i * K, (size_t) K * sizeof(float));
        memcpy(out + (at + 8) * K, up + i * K, (size_t) K * sizeof(float));
    }
}

/* ------------------------------------------------------------------------ */
/* GGUF block formats                                                       */
/* ------------------------------------------------------------------------ */

float zo_fp16_to_fp32(uint16_t h) {
    const uint32_t s = (uint32_t) (h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    if (e == 0) {
        const float v = (float) m * (1.0f / 16777216.0f); /* m * 2^-24, exact */
        return s ? -v : v;
    }
    if (e == 31) return u2f(s | 0x7f800000u | (m << 13));
    return u2f(s | ((e + 112) << 23) | (m << 13));
}

/* round to nearest even, for the synthetic quantisers */
uint16_t zo_fp32_to_fp16(float f) {
    const uint32_t u = f2u(f);
    const uint16_t s = (uint16_t) ((u >> 16) & 0x8000u);
    const float a = fabsf(f);
    if (a != a) return (uint16_t) (s | 0x7e00u);
    if (a >= 65520.0f) return (uint16_t) (s | 0x7c00u);
    if (a < 6.103515625e-05f) { /* subnormal half: multiples of 2^-24 */
        const float q = nearbyintf(a * 16777216.0f);
        return (uint16_t) (s | (uint16_t) q);
    }
    const uint32_t au = f2u(a);
    uint32_t e = (au >> 23) - 112, m = au & 0x7fffffu;
    uint32_t hm = m >> 13, rest = m & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (hm & 1u))) {
        hm++;
        if (hm == 0x400u) { hm = 0; e++; }
    }
    return (uint16_t) (s | (e << 10) | hm);
}

static const int64_t QK8_0 = 32, QK_K = 256;

int64_t zo_row_bytes(int type, int64_t k) {
    switch (type) {
        case ZO_TYPE_F32: return k * 4;
        case ZO_TYPE_F16: return k * 2;
        case ZO_TYPE_Q8_0: return k / QK8_0 * 34;
        case ZO_TYPE_Q4_K: return k / QK_K * 144;
        case ZO_TYPE_Q6_K: return k / QK_K * 210;
        case ZO_TYPE_IQ3_S: return k / QK_K * 110;
        default: return -1;
    }
}

static uint16_t rd16(const uint8_t *p) { return (uint16_t) (p[0] | (p[1] << 8)); }

/* Q8_0: {fp16 d; int8 qs[32]}, y = qs * d */
static void dq_q8_0(const uint8_t *x, float *y, int64_t k) {
    for (int64_t i = 0; i < k / QK8_0; i++, x += 34) {
        const float d = zo_fp16_to_fp32(rd16(x));
        for (int j = 0; j < 32; j++) y[i * 32 + j] = (float) (int8_t) x[2 + j] * d;
    }
}

/* The 6-bit scale and min of sub-block j of a Q4_K super-block, from its
 * 12 packed scale bytes. */
static void q4k_scale_min(int j, const uint8_t *q, uint8_t *d, uint8_t *m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (uint8_t) ((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t) ((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* Q4_K: {fp16 d, dmin; u8 scales[12]; u8 qs[128]}; sub-block j of 32:
 * y = (d*sc_j) * q - (dmin*m_j), q a nibble (low nibbles: even sub-blocks). */
static void dq_q4_k(const uint8_t *x, float *y, int64_t k) {
    for (int64_t i = 0; i < k / QK_K; i++, x += 144) {
        const float d = zo_fp16_to_fp32(rd16(x)), mn = zo_fp16_to_fp32(rd16(x + 2));
        const uint8_t *sc = x + 4, *q = x + 16;
        for (int j = 0; j < 4; j++) {
            uint8_t s0, m0, s1, m1;
            q4k_scale_min(2 * j, sc, &s0, &m0);
            q4k_scale_min(2 * j + 1, sc, &s1, &m1);
            const float d1 = d * (float) s0, mm1 = mn * (float) m0;
            const float d2 = d * (float) s1, mm2 = mn * (float) m1;
            for (int l = 0; l < 32; l++) *y++ = d1 * (float) (q[l] & 0xF) - mm1;
            for (int l = 0; l < 32; l++) *y++ = d2 * (float) (q[l] >> 4) - mm2;
            q += 32;
        }
    }
}

/* Q6_K: {u8 ql[128]; u8 qh[64]; i8 scales[16]; fp16 d}; y = (d*sc) * (q6 - 32) */
static void dq_q6_k(const uint8_t *x, float *y, int64_t k) {
    for (int64_t i = 0; i < k / QK_K; i++, x += 210) {
        const float d = zo_fp16_to_fp32(rd16(x + 208));
        const uint8_t *ql = x, *qh = x + 128;
        const int8_t *sc = (const int8_t *) (x + 192);
        for (int n = 0; n < 2; n++) {
            for (int l = 0; l < 32; l++) {
                const int is = l / 16;
                const int q1 = (int) ((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                const int q2 = (int) ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                const int q3 = (int) ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                const int q4 = (int) ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                y[l + 0] = d * (float) sc[is + 0] * (float) q1;
                y[l + 32] = d * (float) sc[is + 2] * (float) q2;
                y[l + 64] = d * (float) sc[is + 4] * (float) q3;
                y[l + 96] = d * (float) sc[is + 6] * (float) q4;
            }
            y += 128;
            ql += 64;
            qh += 32;
            sc += 8;
        }
    }
}

static uint32_t g_iq3s_grid[512];
static int g_iq3s_ready = 0;

void zo_set_iq3s_grid(const uint32_t *grid512) {
    memcpy(g_iq3s_grid, grid512, sizeof(g_iq3s_grid));
    g_iq3s_ready = 1;
}

/* IQ3_S: {fp16 d; u8 qs[64]; u8 qh[8]; u8 signs[32]; u8 scales[4]}. Each run
 * of 32 values has scale db = d * (1 + 2*s) (s a nibble); each 8 values are two
 * 4-entry codebook rows picked by 9-bit indices (8 bits in qs, the ninth in
 * qh) with one sign bit per value; y = db * grid * sign. */
static void dq_iq3_s(const uint8_t *x, float *y, int64_t k) {
    for (int64_t i = 0; i < k / QK_K; i++, x += 110) {
        const float d = zo_fp16_to_fp32(rd16(x));
        const uint8_t *qs = x + 2, *qh = x + 66, *signs = x + 74, *scales = x + 106;
        for (int ib32 = 0; ib32 < 8; ib32++) {
            const int s = ib32 & 1 ? scales[ib32 / 2] >> 4 : scales[ib32 / 2] & 0xf;
            const float db = d * (float) (1 + 2 * s);
            for (int l = 0; l < 4; l++) {
                const int i1 = qs[2 * l + 0] | (((qh[ib32] >> (2 * l + 0)) & 1) << 8);
                const int i2 = qs[2 * l + 1] | (((qh[ib32] >> (2 * l + 1)) & 1) << 8);
                const uint8_t *g1 = (const uint8_t *) &g_iq3s_grid[i1], *g2 = (const uint8_t *) &g_iq3s_grid[i2];
                for (int j = 0; j < 4; j++) {
                    y[j + 0] = db * (float) g1[j] * ((signs[l] >> (j + 0)) & 1 ? -1.0f : 1.0f);
                    y[j + 4] = db * (float) g2[j] * ((signs[l] >> (j + 4)) & 1 ? -1.0f : 1.0f);
                }
                y += 8;
            }
            qs += 8;
            signs += 4;
        }
    }
}

int zo_dequant_row(int type, const void *raw, float *y, int64_t k) {
    const uint8_t *x = (const uint8_t *) raw;
    switch (type) {
        case ZO_TYPE_F32: memcpy(y, raw, (size_t) k * 4); return 0;
        case ZO_TYPE_F16:
            for (int64_t i = 0; i < k; i++) y[i] = zo_fp16_to_fp32(rd16(x + 2 * i));
            return 0;
        case ZO_TYPE_Q8_0: if (k % QK8_0) return -1; dq_q8_0(x, y, k); return 0;
        case ZO_TYPE_Q4_K: if (k % QK_K) return -1; dq_q4_k(x, y, k); return 0;
        case ZO_TYPE_Q6_K: if (k % QK_K) return -1; dq_q6_k(x, y, k); return 0;
        case ZO_TYPE_IQ3_S:
            if (k % QK_K || !g_iq3s_ready) return -1;
            dq_iq3_s(x, y, k);
            return 0;
        default: return -1;
    }
}

int zo_dequant(int type, const void *raw, int64_t rows, int64_t k, float *y) {
    const int64_t rb = zo_row_bytes(type, k);
    if (rb < 0) return -1;
    for (int64_t r = 0; r < rows; r++)
        if (zo_dequant_row(type, (const uint8_t *) raw + r * rb, y + r * k, k)) return -1;
    return 0;
}

/* ------------------------------------------------------------------------ */
/* quantisers (synthetic weights; not the reference's and need not be)      */
/* ------------------------------------------------------------------------ */

static int clampi(int v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : v; }

static void q_q8_0(const float *x, uint8_t *o, int64_t k) {
    for (int64_t i = 0; i < k / QK8_0; i++, x += 32, o += 34) {
        float amax = 0;
        for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(x[j]));
        const uint16_t dh = zo_fp32_to_fp16(amax / 127.0f);
        const float d = zo_fp16_to_fp32(dh), id = d ? 1.0f / d : 0.0f;
        o[0] = (uint8_t) dh;
        o[1] = (uint8_t) (dh >> 8);
        for (int j = 0; j < 32; j++) o[2 + j] = (uint8_t) (int8_t) clampi((int) nearbyintf(x[j] * id), -128, 127);
    }
}

static void q_q4_k(const float *x, uint8_t *o, int64_t k) {
    for (int64_t i = 0; i < k / QK_K; i++, x += QK_K, o += 144) {
        float sc[8], mn[8], smax = 0, mmax = 0;
        for (int j = 0; j < 8; j++) {
            float lo = 0, hi = 0;
            for (int l = 0; l < 32; l++) {
                lo = fminf(lo, x[j * 32 + l]);
                hi = fmaxf(hi, x[j * 32 + l]);
            }
            sc[j] = (hi - lo) / 15.0f;
            mn[j] = -lo;
            smax = fmaxf(smax, sc[j]);
            mmax = fmaxf(mmax, mn[j]);
        }
        const uint16_t dh = zo_fp32_to_fp16(smax / 63.0f), mh = zo_fp32_to_fp16(mmax / 63.0f);
        const float d = zo_fp16_to_fp32(dh), dm = zo_fp16_to_fp32(mh);
        uint8_t isc[8], imn[8];
        for (int j = 0; j < 8; j++) {
            isc[j] = (uint8_t) clampi(d > 0 ? (int) nearbyintf(sc[j] / d) : 0, 0, 63);
            imn[j] = (uint8_t) clampi(dm > 0 ? (int) nearbyintf(mn[j] / dm) : 0, 0, 63);
        }
        memset(o, 0, 144);
        o[0] = (uint8_t) dh; o[1] = (uint8_t) (dh >> 8);
        o[2] = (uint8_t) mh; o[3] = (uint8_t) (mh >> 8);
        uint8_t *s = o + 4;
        for (int j = 0; j < 4; j++) {
            s[j] = (uint8_t) (isc[j] & 63);
            s[j + 4] = (uint8_t) (imn[j] & 63);
        }
        for (int j = 4; j < 8; j++) {
            s[j + 4] = (uint8_t) ((isc[j] & 0xF) | ((imn[j] & 0xF) << 4));
            s[j - 4] |= (uint8_t) ((isc[j] >> 4) << 6);
            s[j] |= (uint8_t) ((imn[j] >> 4) << 6);
        }
        uint8_t *q = o + 16;
        for (int j = 0; j < 8; j++) {
            const float dd = d * (float) isc[j], mm = dm * (float) imn[j];
            for (int l = 0; l < 32; l++) {
                const int v = dd > 0 ? clampi((int) nearbyintf((x[j * 32 + l] + mm) / dd), 0, 15) : 0;
                q[(j / 2) * 32 + l] |= (uint8_t) (j & 1 ? v << 4 : v);
            }
        }
    }
}

static void q_q6_k(const float *x, uint8_t *o, int64_t k) {
    for (int64_t i = 0; i < k / QK_K; i++, x += QK_K, o += 210) {
        float ss[16], smax = 0;
        for (int j = 0; j < 16; j++) {
            float amax = 0;
            for (int l = 0; l < 16; l++) amax = fmaxf(amax, fabsf(x[j * 16 + l]));
            ss[j] = amax / 31.0f;
            smax = fmaxf(smax, ss[j]);
        }
        const uint16_t dh = zo_fp32_to_fp16(smax / 127.0f);
        const float d = zo_fp16_to_fp32(dh);
        memset(o, 0, 210);
        int8_t *sc = (int8_t *) (o + 192);
        for (int j = 0; j < 16; j++) sc[j] = (int8_t) clampi(d > 0 ? (int) nearbyintf(ss[j] / d) : 0, 0, 127);
        o[208] = (uint8_t) dh;
        o[209] = (uint8_t) (dh >> 8);
        uint8_t *ql = o, *qh = o + 128;
        for (int idx = 0; idx < QK_K; idx++) {
            const float dd = d * (float) sc[idx / 16];
            const int v = (dd > 0 ? clampi((int) nearbyintf(x[idx] / dd), -32, 31) : 0) + 32;
            /* inverse of dq_q6_k's placement */
            const int n = idx / 128, r = idx % 128, quarter = r / 32, l = r % 32;
            uint8_t *qln = ql + n * 64, *qhn = qh + n * 32;
            const int lq = (quarter == 1 || quarter == 3) ? l + 32 : l;
            if (quarter < 2) qln[lq] |= (uint8_t) (v & 0xF);
            else qln[lq] |= (uint8_t) ((v & 0xF) << 4);
            qhn[l] |= (uint8_t) (((v >> 4) & 3) << (2 * quarter));
        }
    }
}

static void q_iq3_s(const float *x, uint8_t *o, int64_t k) {
    for (int64_t i = 0; i < k / QK_K; i++, x += QK_K, o += 110) {
        float want[8], top = 0;
        for (int j = 0; j < 8; j++) {
            float amax = 0;
            for (int l = 0; l < 32; l++) amax = fmaxf(amax, fabsf(x[j * 32 + l]));
            want[j] = amax / 15.0f; /* codebook magnitudes reach 15 */
            top = fmaxf(top, want[j]);
        }
        const uint16_t dh = zo_fp32_to_fp16(top / 31.0f);
        const float d = zo_fp16_to_fp32(dh);
        memset(o, 0, 110);
        o[0] = (uint8_t) dh;
        o[1] = (uint8_t) (dh >> 8);
        uint8_t *qs = o + 2, *qh = o + 66, *signs = o + 74, *scales = o + 106;
        for (int j = 0; j < 8; j++) {
            const int s = d > 0 ? clampi((int) nearbyintf((want[j] / d - 1.0f) / 2.0f), 0, 15) : 0;
            scales[j / 2] |= (uint8_t) (j & 1 ? s << 4 : s);
            const float db = d * (float) (1 + 2 * s);
            for (int g = 0; g < 8; g++) { /* 8 four-value groups in 32 */
                const float *v = x + j * 32 + g * 4;
                int best = 0;
                float berr = INFINITY;
                for (int e = 0; e < 512; e++) {
                    const uint8_t *gv = (const uint8_t *) &g_iq3s_grid[e];
                    float err = 0;
                    for (int t = 0; t < 4; t++) {
                        const float diff = fabsf(v[t]) - db * (float) gv[t];
                        err += diff * diff;
                    }
                    if (err < berr) { berr = err; best = e; }
                }
                qs[j * 8 + g] = (uint8_t) (best & 0xff);
                qh[j] |= (uint8_t) (((best >> 8) & 1) << g);
                for (int t = 0; t < 4; t++)
                    if (v[t] < 0) signs[j * 4 + g / 2] |= (uint8_t) (1u << ((g & 1) * 4 + t));
            }
        }
    }
}

int zo_quantize(int type, const float *x, int64_t rows, int64_t k, void *raw) {
    const int64_t rb = zo_row_bytes(type, k);
    if (rb < 0) return -1;
    for (int64_t r = 0; r < rows; r++) {
        const float *xr = x + r * k;
        uint8_t *o = (uint8_t *) raw + r * rb;
        switch (type) {
            case ZO_TYPE_F32: memcpy(o, xr, (size_t) k * 4); break;
            case ZO_TYPE_F16:
                for (int64_t i = 0; i < k; i++) {
                    const uint16_t h = zo_fp32_to_fp16(xr[i]);
                    o[2 * i] = (uint8_t) h;
                    o[2 * i + 1] = (uint8_t) (h >> 8);
                }
                break;
            case ZO_TYPE_Q8_0: if (k % QK8_0) return -1; q_q8_0(xr, o, k); break;
            case ZO_TYPE_Q4_K: if (k % QK_K) return -1; q_q4_k(xr, o, k); break;
            case ZO_TYPE_Q6_K: if (k % QK_K) return -1; q_q6_k(xr, o, k); break;
            case ZO_TYPE_IQ3_S: if (k % QK_K || !g_iq3s_ready) return -1; q_iq3_s(xr, o, k); break;
            default: return -1;
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* reference matmul                                                         */
/* ------------------------------------------------------------------------ */

typedef struct {
    const float *W, *X;
    int64_t N, M, K, n0, n1;
    float *Y;
    double *Yd;
} mm_job;

static void *mm_rows(void *p) {
    const mm_job *j = (const mm_job *) p;
    for (int64_t n = j->n0; n < j->n1; n++) {
        const float *w = j->W + n * j->K;
        for (int64_t m = 0; m < j->M; m++) {
            const float *x = j->X + m * j->K;
            if (j->Y) {
                float acc = 0.0f;
                for (int64_t k = 0; k < j->K; k++) acc += w[k] * x[k];
                j->Y[m * j->N + n] = acc;
            } else {
                double acc = 0.0;
                for (int64_t k = 0; k < j->K; k++) acc += (double) w[k] * (double) x[k];
                j->Yd[m * j->N + n] = acc;
            }
        }
    }
    return NULL;
}

static void mm_run(const float *W, int64_t N, const float *X, int64_t M, int64_t K, float *Y, double *Yd, int nth) {
    if (nth < 1) nth = 1;
    if (nth > 64) nth = 64;
    if (nth > N) nth = (int) (N > 0 ? N : 1);
    pthread_t th[64];
    mm_job jobs[64];
    const int64_t chunk = (N + nth - 1) / nth;
    for (int t = 0; t < nth; t++) {
        jobs[t] = (mm_job){ W, X, N, M, K, t * chunk, (t + 1) * chunk < N ? (t + 1) * chunk : N, Y, Yd };
        if (t) pthread_create(&th[t], NULL, mm_rows, &jobs[t]);
    }
    mm_rows(&jobs[0]);
    for (int t = 1; t < nth; t++) pthread_join(th[t], NULL);
}

/* xdna_ref_mul_mat's mul_mat_rows (src/xdna-ref.cpp:10-60): per weight row,
 * a float dot with every token row, acc += row[k] * s1[k] in k order. */
void zo_mul_mat(const float *W, int64_t N, const float *X, int64_t M, int64_t K, float *Y, int n_threads) {
    mm_run(W, N, X, M, K, Y, NULL, n_threads);
}

void zo_mul_mat_f64(const float *W, int64_t N, const float *X, int64_t M, int64_t K, double *Y, int n_threads) {
    mm_run(W, N, X, M, K, NULL, Y, n_threads);
}

/* ------------------------------------------------------------------------ */
/* output epilogues                                                         */
/* ------------------------------------------------------------------------ */

/* out_epilogue mode 1 (mm_bfp_acc.cc:258-264): fp32 -> bf16, nearest even */
float zo_round_bf16(float x) {
    uint32_t u = f2u(x);
    if ((u & 0x7fffffffu) > 0x7f800000u) return u2f(u | 0x00400000u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return u2f(u & 0xffff0000u);
}

/* out_epilogue mode 2 (mm_bfp_acc.cc:207-247,265-276): SiLU(g) * u, one
 * rounding to bf16. The NPU evaluates it in bf16 pairs to ~2^-15; this is
 * the double-precision value it approximates. */
float zo_swiglu_bf16(float g, float u) {
    const double s = 1.0 / (1.0 + exp(-(double) g));
    return zo_round_bf16((float) ((double) g * s * (double) u));
}

/* npu_self_test's operands (src/xdna-npu.cpp:142-152): an LCG from seed 1,
 * activations in [-2,2], weights in [-3,3]. */
void zo_selftest_operands(int64_t M, int64_t K, int64_t N, int8_t *a, int8_t *w) {
    uint32_t seed = 1;
    for (int64_t i = 0; i < M * K; i++) {
        seed = seed * 1664525u + 1013904223u;
        a[i] = (int8_t) ((int) (seed >> 24) % 5 - 5 / 2);
    }
    for (int64_t i = 0; i < N * K; i++) {
        seed = seed * 1664525u + 1013904223u;
        w[i] = (int8_t) ((int) (seed >> 24) % 7 - 7 / 2);
    }
}

/* ------------------------------------------------------------------------ */
/* the block executor's small ops (src/xdna-exec.cpp:253-346)               */
/* ------------------------------------------------------------------------ */

void zo_rms_norm(const float *x, int64_t rows, int64_t d, float eps, float *y) {
    for (int64_t r = 0; r < rows; r++) {
        const float *xr = x + r * d;
        float ss = 0.0f;
        for (int64_t j = 0; j < d; j++) ss += xr[j] * xr[j];
        const float sc = 1.0f / sqrtf(ss / (float) d + eps);
        for (int64_t j = 0; j < d; j++) y[r * d + j] = xr[j] * sc;
    }
}

void zo_mul_row(const float *x, const float *w, int64_t rows, int64_t d, float *y) {
    for (int64_t r = 0; r < rows; r++)
        for (int64_t j = 0; j < d; j++) y[r * d + j] = x[r * d + j] * w[j];
}

void zo_add(const float *x, const float *b, int bias_row, int64_t rows, int64_t d, float *y) {
    for (int64_t r = 0; r < rows; r++)
        for (int64_t j = 0; j < d; j++) y[r * d + j] = x[r * d + j] + (bias_row ? b[j] : b[r * d + j]);
}

void zo_scale(const float *x, int64_t n, float s, float bias, float *y) {
    for (int64_t i = 0; i < n; i++) y[i] = x[i] * s + bias;
}

/* the activations, in float (src/xdna-exec.cpp:54-58) */
static float zo_silu(float x) { return x / (1.0f + expf(-x)); }
static float zo_gelu(float x) { return 0.5f * x * (1.0f + tanhf(0.7978845608f * x * (1.0f + 0.044715f * x * x))); }
static float zo_gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.7071067812f)); }
static float zo_gelu_quick(float x) { return x / (1.0f + expf(-1.702f * x)); }

void zo_glu(int kind, const float *g, int64_t g_stride, const float *u, int64_t u_stride, int64_t rows, int64_t f,
            float *y) {
    for (int64_t r = 0; r < rows; r++) {
        const float *gr = g + r * g_stride, *ur = u + r * u_stride;
        float *o = y + r * f;
        for (int64_t j = 0; j < f; j++) {
            switch (kind) {
                case ZO_GLU_SWIGLU: o[j] = zo_silu(gr[j]) * ur[j]; break;
                case ZO_GLU_GEGLU: o[j] = zo_gelu(gr[j]) * ur[j]; break;
                case ZO_GLU_GEGLU_ERF: o[j] = zo_gelu_erf(gr[j]) * ur[j]; break;
                case ZO_GLU_GEGLU_QUICK: o[j] = zo_gelu_quick(gr[j]) * ur[j]; break;
                default: o[j] = gr[j] > 0.0f ? gr[j] * ur[j] : 0.0f; break; /* REGLU */
            }
        }
    }
}

static float zo_corr_dim(int n_dims, int n_ctx_orig, float n_rot, float base) {
    return (float) n_dims * logf((float) n_ctx_orig / (n_rot * 2.0f * (float) M_PI)) / (2.0f * logf(base));
}

void zo_rope_corr_dims(int n_dims, int n_ctx_orig, float freq_base, float beta_fast, float beta_slow, float dims[2]) {
    const float start = floorf(zo_corr_dim(n_dims, n_ctx_orig, beta_fast, freq_base));
    const float end = ceilf(zo_corr_dim(n_dims, n_ctx_orig, beta_slow, freq_base));
    dims[0] = start > 0.0f ? start : 0.0f;
    dims[1] = end < (float) (n_dims - 1) ? end : (float) (n_dims - 1);
}

/* ggml's YaRN rotary for one pair (src/xdna-exec.cpp:65-77) */
static void zo_rope_yarn(float theta_extrap, float freq_scale, const float corr[2], int64_t pair, float ext_factor,
                         float mscale, float *c, float *s) {
    float theta = freq_scale * theta_extrap;
    if (ext_factor != 0.0f) {
        const float lim = corr[1] - corr[0] > 0.001f ? corr[1] - corr[0] : 0.001f;
        const float y = ((float) pair - corr[0]) / lim;
        const float cl = y < 0.0f ? 0.0f : (y > 1.0f ? 1.0f : y);
        const float ramp_mix = (1.0f - cl) * ext_factor;
        theta = theta * (1.0f - ramp_mix) + theta_extrap * ramp_mix;
        mscale *= 1.0f + 0.1f * logf(1.0f / freq_scale);
    }
    *c = cosf(theta) * mscale;
    *s = sinf(theta) * mscale;
}

void zo_rope_table(const int32_t *pos, int64_t T, int n_dims, int n_ctx_orig, const float *par, const float *ff,
                   float *table) {
    const float freq_base = par[0], freq_scale = par[1], ext_factor = par[2], attn_factor = par[3];
    float corr[2];
    zo_rope_corr_dims(n_dims, n_ctx_orig, freq_base, par[4], par[5], corr);
    const float theta_scale = powf(freq_base, -2.0f / (float) n_dims);
    for (int64_t t = 0; t < T; t++) {
        float theta = (float) pos[t];
        float *cs = table + t * n_dims;
        for (int p = 0; p < n_dims / 2; p++) {
            zo_rope_yarn(ff ? theta / ff[p] : theta, freq_scale, corr, p, ext_factor, attn_factor, &cs[2 * p],
                         &cs[2 * p + 1]);
            theta *= theta_scale;
        }
    }
}

void zo_rope(const float *x, int64_t T, int64_t heads, int64_t d, int n_dims, int mode, const float *table, float *y) {
    const int64_t off_n = mode == ZO_ROPE_NEOX ? n_dims / 2 : 1;
    for (int64_t t = 0; t < T; t++) {
        const float *cs = table + t * n_dims;
        for (int64_t h = 0; h < heads; h++) {
            const float *src = x + (t * heads + h) * d;
            float *dst = y + (t * heads + h) * d;
            for (int64_t i = 0; i < n_dims; i += 2) {
                const int64_t ic = mode == ZO_ROPE_NEOX ? i / 2 : i;
                const float c = cs[i], sn = cs[i + 1];
                const float x0 = src[ic], x1 = src[ic + off_n];
                dst[ic] = x0 * c - x1 * sn;
                dst[ic + off_n] = x0 * sn + x1 * c;
            }
            for (int64_t i = n_dims; i < d; i++) dst[i] = src[i];
        }
    }
}

/* CPU oracle for the quantized-weight hot path — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's scalar quantization kernels, used by tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg as the checker. Nothing in the
 * product (sardyne_b200/) links or calls this file.
 *
 * Pinned: tests/test_oracle_golden.py checks every function here against golden vectors
 * produced by the reference itself (tests/golden/make_golden.py: the reference C library
 * built from its own sources plus its NumPy module sardyne/quant.py).
 *
 * Byte layouts (reference csrc/quant.h:16-49):
 *   Q8_0  34 B / 32   : f16 d, int8 qs[32]
 *   Q4_0  18 B / 32   : f16 d, qs[16] low nibble = elt j, high = elt j+16, value q-8
 *   Q5_0  22 B / 32   : f16 d, u32 qh (bit e = 5th bit of elt e), qs[16] as Q4_0, value q-16
 *   Q4_K 144 B / 256  : f16 d, f16 dmin, 12 B packed 6-bit scales/mins, qs[128]
 *   Q6_K 210 B / 256  : ql[128], qh[64], int8 scales[16], f16 d
 *   Q8_K 292 B / 256  : f32 d, int8 qs[256], int16 bsums[16]
 * Built with -ffp-contract=off like the reference (Makefile:15) so every fp32 expression
 * rounds after each operation, in the same order.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

enum { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q5_0 = 6, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14, T_Q8_K = 15 };

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static void wr16(uint8_t *p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }
static float rdf32(const uint8_t *p) { float f; memcpy(&f, p, 4); return f; }

/* IEEE binary16 -> binary32, exact (reference ops.c:15-41). */
float oq_f16_to_f32(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023, bits;
    if (e == 31) {
        bits = s | 0x7F800000u | (m << 13);
    } else if (e) {
        bits = s | ((e + 112) << 23) | (m << 13);
    } else if (!m) {
        bits = s;
    } else { /* subnormal: value m * 2^-24, renormalise */
        int sh = 0;
        while (!(m & 0x400)) { m <<= 1; sh++; }
        bits = s | ((uint32_t)(113 - sh) << 23) | ((m & 1023) << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* binary32 -> binary16, round to nearest even, overflow to inf (reference ops.c:43-62). */
uint16_t oq_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t s = (x >> 16) & 0x8000, a = x & 0x7FFFFFFF;
    if (a > 0x7F800000) return (uint16_t)(s | 0x7E00); /* NaN */
    if (a == 0x7F800000) return (uint16_t)(s | 0x7C00);
    if ((a >> 23) == 0) return (uint16_t)s;             /* f32 subnormal: far below f16 range */
    int e = (int)(a >> 23) - 127;
    uint32_t m = (a & 0x7FFFFF) | 0x800000;             /* value = m * 2^(e-23) */
    /* f16 normal keeps 11 significand bits (drop 13); below 2^-14 count units of 2^-24. */
    int drop = e >= -14 ? 13 : -e - 1;
    if (drop > 25) return (uint16_t)s;
    uint32_t q = m >> drop, rem = m & ((1u << drop) - 1), half = 1u << (drop - 1);
    if (rem > half || (rem == half && (q & 1))) q++;
    if (e < -14) return (uint16_t)(s | q); /* q == 1024 is the smallest normal: still right */
    uint32_t r = ((uint32_t)(e + 15) << 10) + (q - 1024); /* q == 2048 carries into the exponent */
    return (uint16_t)(s | (r >= 0x7C00 ? 0x7C00 : r));
}

/* ------------------------------------------------------------ dequantization (quant.c:13-94) */

/* The 6-bit scale and min of sub-block j of a Q4_K superblock (quant.h:72-80). */
static void k4_scale_min(int j, const uint8_t *p, int *sc, int *mn) {
    if (j < 4) { *sc = p[j] & 63; *mn = p[j + 4] & 63; }
    else { *sc = (p[j + 4] & 15) | ((p[j - 4] >> 6) << 4); *mn = (p[j + 4] >> 4) | ((p[j] >> 6) << 4); }
}

/* Element e (0..255) of a Q6_K superblock as 0..63 (quant.c:62-74). */
static int k6_raw(const uint8_t *b, int e) {
    int half = e >> 7, w = e & 127, quarter = w >> 5, l = w & 31;
    const uint8_t *ql = b + 64 * half, *qh = b + 128 + 32 * half;
    int lo = (quarter & 1) ? ql[l + 32] : ql[l];
    lo = (quarter >> 1) ? (lo >> 4) : (lo & 15);
    return lo | (((qh[l] >> (2 * quarter)) & 3) << 4);
}

static int q5_0_value(const uint8_t *b, int e) {
    uint32_t qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) | ((uint32_t)b[5] << 24);
    int nib = e < 16 ? (b[6 + e] & 15) : (b[6 + e - 16] >> 4);
    return (nib | (int)(((qh >> e) & 1) << 4)) - 16;
}

void oq_dequant_row(int type, const uint8_t *src, float *dst, int n) {
    if (type == T_Q8_0 || type == T_Q4_0 || type == T_Q5_0) {
        int bb = type == T_Q8_0 ? 34 : type == T_Q4_0 ? 18 : 22;
        for (int i = 0; i < n / 32; i++) {
            const uint8_t *b = src + (size_t)i * bb;
            float d = oq_f16_to_f32(rd16(b));
            for (int e = 0; e < 32; e++) {
                int v;
                if (type == T_Q8_0) v = (int8_t)b[2 + e];
                else if (type == T_Q4_0) v = (e < 16 ? (b[2 + e] & 15) : (b[2 + e - 16] >> 4)) - 8;
                else v = q5_0_value(b, e);
                dst[i * 32 + e] = (float)v * d;
            }
        }
    } else if (type == T_Q4_K) {
        for (int i = 0; i < n / 256; i++) {
            const uint8_t *b = src + (size_t)i * 144;
            float d = oq_f16_to_f32(rd16(b)), dmin = oq_f16_to_f32(rd16(b + 2));
            for (int j = 0; j < 8; j++) {
                int sc, mn;
                k4_scale_min(j, b + 4, &sc, &mn);
                float d1 = d * (float)sc, m1 = dmin * (float)mn; /* quant.c:41-44 */
                const uint8_t *q = b + 16 + 32 * (j >> 1);
                for (int l = 0; l < 32; l++) {
                    int v = (j & 1) ? (q[l] >> 4) : (q[l] & 15);
                    dst[i * 256 + j * 32 + l] = d1 * (float)v - m1;
                }
            }
        }
    } else if (type == T_Q6_K) {
        for (int i = 0; i < n / 256; i++) {
            const uint8_t *b = src + (size_t)i * 210;
            float d = oq_f16_to_f32(rd16(b + 208));
            for (int e = 0; e < 256; e++) {
                float dsc = d * (float)(int8_t)b[192 + e / 16]; /* (d*sc)*q, quant.c:81 */
                dst[i * 256 + e] = dsc * (float)(k6_raw(b, e) - 32);
            }
        }
    } else if (type == T_F16) {
        for (int i = 0; i < n; i++) dst[i] = oq_f16_to_f32(rd16(src + 2 * i));
    } else if (type == T_F32) {
        memcpy(dst, src, (size_t)n * 4);
    }
}

/* ------------------------------------------------------------ activation quantization (quant.c:98-144) */

void oq_quant_q8_0(const float *x, uint8_t *dst, int n) {
    for (int i = 0; i < n / 32; i++) {
        const float *v = x + 32 * i;
        uint8_t *b = dst + 34 * i;
        float amax = 0.0f;
        for (int e = 0; e < 32; e++) amax = fmaxf(amax, fabsf(v[e]));
        float d = amax / 127.0f;
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        wr16(b, oq_f32_to_f16(d));
        for (int e = 0; e < 32; e++) b[2 + e] = (uint8_t)(int8_t)roundf(v[e] * id);
    }
}

/* Round half to even for |v| < 2^22 (quant.c:111-116), written with rint under the default mode. */
static int round_even(float v) { return (int)rintf(v); }

void oq_quant_q8_K(const float *x, uint8_t *dst, int n) {
    for (int i = 0; i < n / 256; i++) {
        const float *v = x + 256 * i;
        uint8_t *b = dst + 292 * i;
        float amax = 0.0f, vmax = 0.0f;
        for (int e = 0; e < 256; e++) /* first index of the largest magnitude keeps its sign */
            if (fabsf(v[e]) > amax) { amax = fabsf(v[e]); vmax = v[e]; }
        memset(b, 0, 292);
        if (amax == 0.0f) continue;
        float iscale = -127.0f / vmax;
        int8_t *qs = (int8_t *)(b + 4);
        for (int e = 0; e < 256; e++) {
            int q = round_even(iscale * v[e]);
            qs[e] = (int8_t)(q < 127 ? q : 127);
        }
        for (int g = 0; g < 16; g++) {
            int s = 0;
            for (int k = 0; k < 16; k++) s += qs[16 * g + k];
            wr16(b + 260 + 2 * g, (uint16_t)(int16_t)s);
        }
        float d = 1.0f / iscale;
        memcpy(b, &d, 4);
    }
}

/* ------------------------------------------------------------ dot products (quant.c:148-235) */

/* One weight row (n elements) against one quantized activation row, in the reference's scalar
 * order: an exact integer sum per block, then one fp32 combine per block in block order. */
float oq_vec_dot(int type, const uint8_t *w, const uint8_t *x, int n) {
    float acc = 0.0f;
    if (type == T_Q8_0 || type == T_Q4_0 || type == T_Q5_0) {
        int bb = type == T_Q8_0 ? 34 : type == T_Q4_0 ? 18 : 22;
        for (int i = 0; i < n / 32; i++) {
            const uint8_t *a = w + (size_t)i * bb, *y = x + (size_t)i * 34;
            int32_t s = 0;
            for (int e = 0; e < 32; e++) {
                int v = type == T_Q8_0 ? (int8_t)a[2 + e]
                      : type == T_Q4_0 ? (e < 16 ? (a[2 + e] & 15) : (a[2 + e - 16] >> 4)) - 8
                                       : q5_0_value(a, e);
                s += v * (int8_t)y[2 + e];
            }
            float scale = oq_f16_to_f32(rd16(a)) * oq_f16_to_f32(rd16(y));
            acc = acc + (float)s * scale; /* quant.c:160 */
        }
    } else if (type == T_Q4_K) {
        for (int i = 0; i < n / 256; i++) {
            const uint8_t *a = w + (size_t)i * 144, *y = x + (size_t)i * 292;
            const int8_t *yq = (const int8_t *)(y + 4);
            int32_t isum = 0, msum = 0;
            for (int j = 0; j < 8; j++) {
                int sc, mn;
                k4_scale_min(j, a + 4, &sc, &mn);
                const uint8_t *q = a + 16 + 32 * (j >> 1);
                int32_t s = 0;
                for (int l = 0; l < 32; l++) s += ((j & 1) ? (q[l] >> 4) : (q[l] & 15)) * yq[32 * j + l];
                isum += sc * s;
                int16_t b0, b1;
                memcpy(&b0, y + 260 + 4 * j, 2);
                memcpy(&b1, y + 262 + 4 * j, 2);
                msum += mn * (b0 + b1);
            }
            /* q4k_combine (quant.h:84-87) */
            float yd = rdf32(y), d = oq_f16_to_f32(rd16(a)), dmin = oq_f16_to_f32(rd16(a + 2));
            float dall = yd * d, dmn = yd * dmin;
            acc = acc + (dall * (float)isum - dmn * (float)msum);
        }
    } else if (type == T_Q6_K) {
        for (int i = 0; i < n / 256; i++) {
            const uint8_t *a = w + (size_t)i * 210, *y = x + (size_t)i * 292;
            const int8_t *yq = (const int8_t *)(y + 4);
            int32_t isum = 0;
            for (int g = 0; g < 16; g++) {
                int32_t s = 0;
                for (int k = 0; k < 16; k++) s += (k6_raw(a, 16 * g + k) - 32) * yq[16 * g + k];
                isum += (int8_t)a[192 + g] * s;
            }
            /* q6k_combine (quant.h:89-91) */
            float yd = rdf32(y), d = oq_f16_to_f32(rd16(a + 208));
            acc = acc + (yd * d) * (float)isum;
        }
    }
    return acc;
}

static size_t row_bytes(int type, int n) {
    switch (type) {
    case T_Q8_0: return (size_t)(n / 32) * 34;
    case T_Q4_0: return (size_t)(n / 32) * 18;
    case T_Q5_0: return (size_t)(n / 32) * 22;
    case T_Q4_K: return (size_t)(n / 256) * 144;
    case T_Q6_K: return (size_t)(n / 256) * 210;
    case T_Q8_K: return (size_t)(n / 256) * 292;
    case T_F16: return (size_t)n * 2;
    case T_F32: return (size_t)n * 4;
    default: return 0;
    }
}

size_t oq_row_bytes(int type, int n) { return row_bytes(type, n); }

/* out[t*n_out + j] for rows row0..row1 and every token (ops.c:293-309, rows outer). */
void oq_matmul_q_rows(float *out, const uint8_t *xq, const uint8_t *w, int type, int n_tok, int n_in, int n_out,
                      int row0, int row1) {
    int vt = (type == T_Q4_K || type == T_Q6_K) ? T_Q8_K : T_Q8_0;
    size_t wr = row_bytes(type, n_in), xr = row_bytes(vt, n_in);
    for (int j = row0; j < row1; j++)
        for (int t = 0; t < n_tok; t++)
            out[(size_t)t * n_out + j] = oq_vec_dot(type, w + (size_t)j * wr, xq + (size_t)t * xr, n_in);
}

/* Quantize n_tok rows of n_in floats into the activation type of `type`. */
void oq_quantize_rows(int vtype, const float *x, uint8_t *xq, int n_in, int n_tok) {
    size_t xr = row_bytes(vtype, n_in);
    for (int t = 0; t < n_tok; t++) {
        if (vtype == T_Q8_0) oq_quant_q8_0(x + (size_t)t * n_in, xq + (size_t)t * xr, n_in);
        else oq_quant_q8_K(x + (size_t)t * n_in, xq + (size_t)t * xr, n_in);
    }
}

/* The reference's fp32 parts call libm's expf (softmax ops.c:353-364, SiLU ops.c:366-371); the
 * operation-order models in the tests take it from the same libm, element by element. */
void oq_expf_n(const float *x, float *y, size_t n) {
    for (size_t i = 0; i < n; i++) y[i] = expf(x[i]);
}

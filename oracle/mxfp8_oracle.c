/*
 * mxfp8_oracle.c -- CPU restatement of the reference MXFP8 quantizer recipe.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the CUDA kernels are
 * compared against; it is never part of the product path.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it.
 *
 * Parity pin: the scale rule and the payload rule below were checked against
 * the reference's own torch restatement (`reference_quantize`,
 * MXFP8_quantizer.py:610-641) and its layout decoder (`decode_scale_bytes`,
 * MXFP8_quantizer.py:643-662) on every finite amax bit pattern of both input
 * dtypes and on seeded random matrices; the digests live in tests/golden/.
 * Non-finite blocks follow the reference *kernel* (MXFP8_quantizer.py:170-200
 * and 473-501), whose instructions (fma.rn.f32, mul.rn.f32x2,
 * cvt.rn.satfinite.e4m3x2.f32) are restated here from their PTX ISA
 * definitions with integer arithmetic only, so the quantizer's result does
 * not depend on the host's floating-point environment (rounding mode,
 * DAZ/FTZ).  Only the dequantize restatement (oracle_dequantize) multiplies
 * in float: an E4M3 value times a power of two, exact unless the product
 * falls below the normal f32 range.
 *
 * Everything is plain C99 + pthreads.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_BF16 0
#define ORACLE_FP16 1

/* Constants of the recipe, MXFP8_quantizer.py:57-64 and 172-178.  The
 * reference builds them as Float32(python double), i.e. one double->float
 * rounding: Float32(1.0/448.0) and Float32(1.0e-12). */
#define INV_448_BITS 0x3B124925u
#define EPS_BITS 0x2B8CBCCCu
#define SCALE_VEC 32
#define SCALE_PACK_COLS 4
#define SCALE_ROWS_PER_PACK 128
#define E4M3_NAN 0x7Fu

static float f32_from_bits(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static uint32_t bits_from_f32(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

/* Exact fp16 -> f32 widening (every fp16 value is an f32 value). */
static uint32_t fp16_to_f32_bits(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1F, m = h & 0x3FF;
    if (e == 0x1F) return sign | 0x7F800000u | (m << 13);
    if (e != 0) return sign | ((e + 112u) << 23) | (m << 13);
    if (m == 0) return sign;
    /* subnormal fp16: m * 2^-24, normalise */
    int sh = 0;
    while (!(m & 0x400)) { m <<= 1; ++sh; }
    m &= 0x3FF;
    return sign | ((uint32_t)(113 - sh) << 23) | (m << 13);
}

static uint32_t in_to_f32_bits(uint16_t v, int dtype) {
    return dtype == ORACLE_BF16 ? ((uint32_t)v << 16) : fp16_to_f32_bits(v);
}

/* ------------------------------------------------------------------------
 * Scale rule, MXFP8_quantizer.py:170-200 (ceil_pow2_scale_from_amax) applied
 * to the block amax of MXFP8_quantizer.py:456-468:
 *   amax_bits = max over the block of (bits & 0x7FFF)   (NaN outranks inf)
 *   amax == 0  -> byte 127, inverse scale 1.0
 *   else       -> s = fma.rn(amax, f32(1/448), f32(1e-12)); e = exp(s) + (mant(s) != 0)
 *                 byte = (u8)e ; inverse = f32 bits ((254 - e) << 23), u32 wraparound
 * Returns the byte; *inv_bits receives the inverse-scale bit pattern.
 * ------------------------------------------------------------------------ */
/* Significand and exponent of a finite f32 >= 0: value = *sig * 2^*exp. */
static void f32_split(uint32_t b, uint64_t* sig, int* exp) {
    uint32_t e = (b >> 23) & 0xFF, m = b & 0x7FFFFF;
    if (e == 0) { *sig = m; *exp = -149; }
    else { *sig = (uint64_t)m | 0x800000u; *exp = (int)e - 150; }
}

static int msb64(uint64_t v) { int p = -1; while (v) { v >>= 1; ++p; } return p; }

/* fma.rn.f32(a, c, e) for finite a >= 0 and c, e > 0 whose result is a
 * normal f32 (here s >= e = f32(1e-12) > 2^-126 and a <= the bf16 maximum,
 * so it is), in integer arithmetic: the exact sum a*c + e, then one
 * round-to-nearest-even to 24 significant bits (PTX ISA, fma.rn.f32). */
static uint32_t fma_rn_pos_bits(uint32_t a, uint32_t c, uint32_t e) {
    uint64_t sa, sc, se;
    int xa, xc, xe;
    f32_split(a, &sa, &xa);
    f32_split(c, &sc, &xc);
    f32_split(e, &se, &xe);
    uint64_t s1 = sa * sc, s2 = se;  /* terms s1 * 2^x1 (the product, exact in 48 bits) and s2 * 2^x2 */
    int x1 = xa + xc, x2 = xe;
    if (s1 == 0) return e;
    int p1 = msb64(s1), p2 = msb64(s2);
    s1 <<= 62 - p1; x1 -= 62 - p1;  /* both significands now have bit 62 as their top bit */
    s2 <<= 62 - p2; x2 -= 62 - p2;
    if (x2 > x1) { uint64_t ts = s1; s1 = s2; s2 = ts; int tx = x1; x1 = x2; x2 = tx; }
    const int k = x1 - x2;  /* align the smaller term under the larger one, 64 bits below it */
    unsigned __int128 acc = (unsigned __int128)s1 << 64;
    int sticky = 0;
    if (k <= 64) {
        acc += (unsigned __int128)s2 << (64 - k);
    } else if (k < 127) {
        acc += s2 >> (k - 64);
        sticky = (s2 & ((1ull << (k - 64)) - 1)) != 0;
    } else {
        sticky = 1;
    }
    /* value = acc * 2^(x1 - 64), acc's top bit at 126 or 127 */
    const int top = (acc >> 127) ? 127 : 126;
    const int drop = top - 23;  /* bits below the 24-bit significand */
    uint64_t sig = (uint64_t)(acc >> drop);
    const unsigned __int128 rest = acc & (((unsigned __int128)1 << drop) - 1);
    const unsigned __int128 half = (unsigned __int128)1 << (drop - 1);
    int exp = top + x1 - 64;  /* unbiased exponent of the leading bit */
    if (rest > half || (rest == half && (sticky || (sig & 1))) ) sig += 1;
    if (sig >> 24) { sig >>= 1; exp += 1; }
    return ((uint32_t)(exp + 127) << 23) | ((uint32_t)sig & 0x7FFFFFu);
}

uint8_t oracle_scale_from_amax_bits(uint16_t amax_bits, int dtype, uint32_t* inv_bits) {
    uint32_t e;
    if ((amax_bits & 0x7FFF) == 0) {
        e = 127u;
    } else {
        const uint32_t a = in_to_f32_bits(amax_bits & 0x7FFF, dtype);
        uint32_t b;
        if ((a & 0x7F800000u) == 0x7F800000u)
            b = (a & 0x7FFFFFu) ? 0x7FFFFFFFu : 0x7F800000u;  /* NaN stays NaN, inf * c + e = inf */
        else
            b = fma_rn_pos_bits(a, INV_448_BITS, EPS_BITS);
        e = (b >> 23) & 0xFFu;
        if (b & 0x7FFFFFu) e += 1u;
    }
    if (inv_bits) *inv_bits = (254u - e) << 23;
    return (uint8_t)(e & 0xFFu);
}

/* ------------------------------------------------------------------------
 * f32 product x * inv rounded to nearest-even with subnormals kept (no FTZ),
 * as mul.rn.f32x2 does (MXFP8_quantizer.py:477-486).  Integer-only.
 * ------------------------------------------------------------------------ */
typedef struct { uint32_t sign; int cls; uint64_t sig; int exp; } fval; /* cls: 0 zero, 1 finite, 2 inf, 3 nan */

static fval f32_decode(uint32_t b) {
    fval v; v.sign = b >> 31; v.sig = 0; v.exp = 0;
    uint32_t e = (b >> 23) & 0xFF, m = b & 0x7FFFFF;
    if (e == 0xFF) { v.cls = m ? 3 : 2; return v; }
    if (e == 0) {
        if (m == 0) { v.cls = 0; return v; }
        v.cls = 1; v.sig = m; v.exp = -149; return v;
    }
    v.cls = 1; v.sig = (uint64_t)m | 0x800000u; v.exp = (int)e - 150; return v;
}

/* Round sign * sig * 2^exp (sig != 0) to an f32 bit pattern, RNE. */
static uint32_t f32_round(uint32_t sign, uint64_t sig, int exp) {
    int p = 63 - __builtin_clzll(sig);
    int lead = p + exp;                      /* weight of the leading bit */
    int q = lead >= -126 ? lead - 23 : -149; /* weight of the result's LSB */
    int sh = q - exp;
    uint64_t r;
    if (sh <= 0) {
        r = sig << (-sh);                    /* exact; at most 24 bits */
    } else if (sh >= 64) {
        r = 0;                               /* below half an LSB */
    } else {
        r = sig >> sh;
        uint64_t rem = sig & ((1ull << sh) - 1), half = 1ull << (sh - 1);
        if (rem > half || (rem == half && (r & 1))) ++r;
    }
    if (r < 0x800000u) return (sign << 31) | (uint32_t)r;   /* subnormal or zero */
    if (r == 0x1000000u) { r >>= 1; ++q; }
    int be = q + 150;
    if (be >= 255) return (sign << 31) | 0x7F800000u;
    return (sign << 31) | ((uint32_t)be << 23) | ((uint32_t)r & 0x7FFFFFu);
}

uint32_t oracle_f32_mul_rn(uint32_t a, uint32_t b) {
    fval x = f32_decode(a), y = f32_decode(b);
    uint32_t sign = x.sign ^ y.sign;
    if (x.cls == 3 || y.cls == 3) return 0x7FFFFFFFu;               /* canonical NaN */
    if ((x.cls == 2 && y.cls == 0) || (x.cls == 0 && y.cls == 2)) return 0x7FFFFFFFu;
    if (x.cls == 2 || y.cls == 2) return (sign << 31) | 0x7F800000u;
    if (x.cls == 0 || y.cls == 0) return sign << 31;
    return f32_round(sign, x.sig * y.sig, x.exp + y.exp);
}

/* ------------------------------------------------------------------------
 * cvt.rn.satfinite.e4m3x2.f32 for one lane (MXFP8_quantizer.py:116-137):
 * round-to-nearest-even into E4M3 (bias 7, 3 mantissa bits, subnormals down
 * to 2^-9, max 448 = 0x7E); |v| beyond 448 (inf included) saturates to
 * +-448; NaN gives the E4M3 NaN 0x7F.
 * ------------------------------------------------------------------------ */
uint8_t oracle_e4m3_from_f32_bits(uint32_t b) {
    uint32_t sign = (b >> 24) & 0x80u;
    uint32_t a = b & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return (uint8_t)E4M3_NAN;
    if (a >= 0x43E00000u) return (uint8_t)(sign | 0x7Eu);        /* >= 448, inf */
    uint32_t E = a >> 23, m23 = a & 0x7FFFFFu;
    uint32_t code;
    if (E < 121u) {
        /* below 2^-6: result is a multiple of 2^-9 (E4M3 subnormal step) */
        uint64_t sig = E ? ((uint64_t)m23 | 0x800000u) : (uint64_t)m23;
        int sh = 141 - (int)(E ? E : 1);       /* value / 2^-9 = sig >> sh */
        if (sh >= 64) {
            code = 0;
        } else {
            uint64_t r = sig >> sh, rem = sig & ((1ull << sh) - 1), half = 1ull << (sh - 1);
            if (rem > half || (rem == half && (r & 1))) ++r;
            code = (uint32_t)r;                 /* 8 rolls into the smallest normal */
        }
    } else {
        code = ((E - 120u) << 3) | (m23 >> 20);
        uint32_t rem = m23 & 0xFFFFFu;
        if (rem > 0x80000u || (rem == 0x80000u && (code & 1u))) ++code;
        if (code > 0x7Eu) code = 0x7Eu;
    }
    return (uint8_t)(sign | code);
}

/* Packed scale storage (MXFP8_quantizer.py:531-539): 128-row x 4-column,
 * 512-byte chunks, row-block major. */
int64_t oracle_scale_storage_bytes(int64_t rows, int64_t cols) {
    int64_t scale_cols = (cols + SCALE_VEC - 1) / SCALE_VEC;
    int64_t prow = (rows + SCALE_ROWS_PER_PACK - 1) / SCALE_ROWS_PER_PACK * SCALE_ROWS_PER_PACK;
    int64_t pcol = (scale_cols + SCALE_PACK_COLS - 1) / SCALE_PACK_COLS * SCALE_PACK_COLS;
    return prow * pcol;
}

/* Byte offset of scale (r, c) inside the packed storage
 * (MXFP8_quantizer.py:502-525 and its inverse 643-662). */
int64_t oracle_scale_offset(int64_t r, int64_t c, int64_t scale_cols) {
    int64_t cb = (scale_cols + SCALE_PACK_COLS - 1) / SCALE_PACK_COLS;
    int64_t rr = r % SCALE_ROWS_PER_PACK;
    return ((r / SCALE_ROWS_PER_PACK) * cb + c / SCALE_PACK_COLS) * 512 + (rr % 32) * 16 +
           (rr / 32) * 4 + (c % SCALE_PACK_COLS);
}

/* Per-dtype table of the scale rule over all 32768 amax patterns. */
static uint8_t g_scale_lut[2][32768];
static uint32_t g_inv_lut[2][32768];
static pthread_once_t g_lut_once = PTHREAD_ONCE_INIT;
static void build_luts(void) {
    for (int d = 0; d < 2; ++d)
        for (uint32_t a = 0; a < 32768u; ++a)
            g_scale_lut[d][a] = oracle_scale_from_amax_bits((uint16_t)a, d, &g_inv_lut[d][a]);
}

/* One 32-element block: x points at the first element; `valid` elements are
 * real, the rest are zero padding (MXFP8_quantizer.py:554-562 zero-pads). */
static uint8_t quantize_block(const uint16_t* x, int valid, int dtype, uint8_t* q) {
    uint16_t v[SCALE_VEC];
    uint16_t amax = 0;
    for (int i = 0; i < SCALE_VEC; ++i) {
        v[i] = i < valid ? x[i] : 0;
        uint16_t a = v[i] & 0x7FFF;
        if (a > amax) amax = a;
    }
    uint8_t s = g_scale_lut[dtype][amax];
    uint32_t inv = g_inv_lut[dtype][amax];
    for (int i = 0; i < SCALE_VEC; ++i)
        q[i] = oracle_e4m3_from_f32_bits(oracle_f32_mul_rn(in_to_f32_bits(v[i], dtype), inv));
    return s;
}

/* Quantize rows [r0, r1) of the output geometry.  X is (m, k) with row stride
 * ld_x elements; Q is q_rows x q_cols bytes with row stride ld_q; S is the
 * packed storage for (q_rows, q_cols).  Elements of X outside (m, k) read as
 * zero, so padded columns get scale 127 and payload 0, as in the reference's
 * zero-padded launch.  Scale bytes for rows >= q_rows are left untouched. */
static void quantize_rows(const uint16_t* x, int dtype, int64_t m, int64_t k, int64_t ld_x,
                          uint8_t* q, int64_t q_rows, int64_t q_cols, int64_t ld_q,
                          uint8_t* s, int64_t r0, int64_t r1) {
    int64_t nblk = q_cols / SCALE_VEC;
    static const uint16_t zeros[SCALE_VEC] = {0};
    for (int64_t r = r0; r < r1 && r < q_rows; ++r) {
        for (int64_t b = 0; b < nblk; ++b) {
            int64_t c0 = b * SCALE_VEC;
            int valid = 0;
            const uint16_t* src = zeros;
            if (r < m && c0 < k) {
                valid = (int)((k - c0) < SCALE_VEC ? (k - c0) : SCALE_VEC);
                src = x + r * ld_x + c0;
            }
            uint8_t sb = quantize_block(src, valid, dtype, q + r * ld_q + c0);
            s[oracle_scale_offset(r, b, nblk)] = sb;
        }
    }
}

typedef struct {
    const uint16_t* x; int dtype; int64_t m, k, ld_x;
    uint8_t* q; int64_t q_rows, q_cols, ld_q; uint8_t* s;
    int64_t r0, r1;
} job_t;

static void* job_main(void* p) {
    job_t* j = (job_t*)p;
    quantize_rows(j->x, j->dtype, j->m, j->k, j->ld_x, j->q, j->q_rows, j->q_cols, j->ld_q, j->s,
                  j->r0, j->r1);
    return NULL;
}

/* Returns 0 on success, -1 on bad arguments.  S must hold
 * oracle_scale_storage_bytes(q_rows, q_cols) bytes; bytes of rows >= q_rows
 * and columns >= q_cols/32 are set to zero (never-written storage of the
 * reference's torch.zeros buffer, MXFP8_quantizer.py:567).  Work is split
 * over `nthreads` threads by 128-row chunks. */
int oracle_quantize(const void* x, int dtype, int64_t m, int64_t k, int64_t ld_x,
                    void* q, int64_t q_rows, int64_t q_cols, int64_t ld_q,
                    void* s, int64_t s_bytes, int nthreads) {
    if ((dtype != ORACLE_BF16 && dtype != ORACLE_FP16) || m < 0 || k < 0 || ld_x < k ||
        q_rows < m || q_cols < k || q_cols % SCALE_VEC || ld_q < q_cols ||
        s_bytes < oracle_scale_storage_bytes(q_rows, q_cols))
        return -1;
    pthread_once(&g_lut_once, build_luts);
    memset(s, 0, (size_t)oracle_scale_storage_bytes(q_rows, q_cols));
    if (q_rows == 0 || q_cols == 0) return 0;
    int64_t chunks = (q_rows + SCALE_ROWS_PER_PACK - 1) / SCALE_ROWS_PER_PACK;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > chunks) nthreads = (int)chunks;
    if (nthreads > 256) nthreads = 256;
    job_t jobs[256];
    pthread_t th[256];
    int64_t per = (chunks + nthreads - 1) / nthreads;
    int launched = 0;
    for (int t = 0; t < nthreads; ++t) {
        int64_t c0 = t * per, c1 = c0 + per < chunks ? c0 + per : chunks;
        if (c0 >= c1) break;
        job_t j = {(const uint16_t*)x, dtype, m, k, ld_x, (uint8_t*)q, q_rows, q_cols, ld_q,
                   (uint8_t*)s, c0 * SCALE_ROWS_PER_PACK, c1 * SCALE_ROWS_PER_PACK};
        jobs[t] = j;
        if (t == 0) continue;
        if (pthread_create(&th[t], NULL, job_main, &jobs[t]) != 0) {
            job_main(&jobs[t]);            /* run inline if no thread could be made */
            th[t] = 0;
        }
        launched = t + 1;
    }
    job_main(&jobs[0]);
    for (int t = 1; t < launched; ++t)
        if (th[t]) pthread_join(th[t], NULL);
    return 0;
}

/* Dense (rows, scale_cols) view of packed scales, the inverse layout map of
 * MXFP8_quantizer.py:643-662. */
int oracle_unpack_scales(const void* s, int64_t rows, int64_t scale_cols, void* dense) {
    const uint8_t* sp = (const uint8_t*)s;
    uint8_t* d = (uint8_t*)dense;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < scale_cols; ++c)
            d[r * scale_cols + c] = sp[oracle_scale_offset(r, c, scale_cols)];
    return 0;
}

/* E4M3 byte -> f32 value (exact). */
static float e4m3_to_f32(uint8_t v) {
    uint32_t sign = (uint32_t)(v >> 7) << 31;
    uint32_t e = (v >> 3) & 0xF, m = v & 7;
    if (e == 0xF && m == 7) return f32_from_bits(0x7FC00000u | sign);
    float mag = e ? ldexpf((float)(8 + m), (int)e - 10) : ldexpf((float)m, -9);
    return sign ? -mag : mag;
}

/* Dequantize: out[r, c] = e4m3(Q[r, c]) * 2^(S[r, c/32] - 127), the value
 * the reference's end-to-end check rebuilds (MXFP8_quantizer.py:1179-1187).
 * Scale byte 255 decodes to NaN (UE8M0 NaN). */
int oracle_dequantize(const void* q, int64_t rows, int64_t cols, int64_t ld_q,
                      const void* s, float* out, int64_t ld_out) {
    if (cols % SCALE_VEC) return -1;
    const uint8_t* qp = (const uint8_t*)q;
    const uint8_t* sp = (const uint8_t*)s;
    int64_t scale_cols = cols / SCALE_VEC;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t b = 0; b < scale_cols; ++b) {
            uint8_t sb = sp[oracle_scale_offset(r, b, scale_cols)];
            float scale = sb == 255 ? f32_from_bits(0x7FC00000u)
                                    : (sb == 0 ? ldexpf(1.0f, -127) : f32_from_bits((uint32_t)sb << 23));
            for (int i = 0; i < SCALE_VEC; ++i) {
                int64_t c = b * SCALE_VEC + i;
                out[r * ld_out + c] = e4m3_to_f32(qp[r * ld_q + c]) * scale;
            }
        }
    return 0;
}

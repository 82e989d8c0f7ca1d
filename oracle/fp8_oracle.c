/*
 * TEST INFRASTRUCTURE ONLY — the CPU oracle for the FP8 weight quantizer.
 *
 * This file restates, in plain C, the algorithm of the reference's host
 * quantizer `reng-fp8` (crates/reng-fp8/src/lib.rs).  It is the checker the
 * parity tests compare the CUDA quantizer against, and the CPU baseline that
 * bench.py times beside it.  Nothing in the product path links or calls it:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU legs load it.
 *
 * Parity pin: tests/test_fp8_oracle.py checks this restatement against every
 * case of the reference's golden file crates/reng-fp8/fixtures/fp8_cast.json
 * (copied to tests/golden/fp8_cast.json by tests/golden/make_golden.py)
 * and against the known answers of the reference's unit tests
 * (crates/reng-fp8/src/lib.rs:632-926).
 *
 * Semantics restated (reference line numbers in brackets):
 *   bf16 <-> f32, RNE, NaN -> 0x7fc0                        [lib.rs:33-48]
 *   E4M3: bias 7, max finite 240 (0x77); E5M2: bias 15,
 *   max finite 57344 (0x7b); top exponent field reserved     [lib.rs:53-147]
 *   encode: RNE, saturate to max finite, NaN -> sign|0x7f,
 *   f32 subnormal -> signed zero, carry into next binade    [lib.rs:154-201]
 *   decode: finite exactly, top field inf/NaN               [lib.rs:205-225]
 *   pow2 incl. subnormal powers                              [lib.rs:229-236]
 *   quantize_with: row absmax with '>' (NaN ignored), scale
 *   m/(max_finite*backoff) or 1.0 for a zero row; hw bias
 *   choice; unit; encode(f32(bf16)/s) by division          [lib.rs:519-563]
 *   row split over <= 8 threads (result equals serial)      [lib.rs:565-621]
 *   row_errors: f64 sum of f32 relative errors              [lib.rs:364-388]
 *   choose_exp_bias                                          [lib.rs:464-475]
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_E4M3 0
#define ORC_E5M2 1
#define ORC_PCS 0
#define ORC_HW 1
#define ORC_UNIT 2

static float bits_f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

float orc_bf16_to_f32(uint16_t b) { return bits_f((uint32_t)b << 16); }

uint16_t orc_f32_to_bf16(float x) {
    uint32_t u = f_bits(x);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
    uint32_t rb = 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)((u + rb) >> 16);
}

static int fmt_mbits(int fmt) { return fmt == ORC_E4M3 ? 3 : 2; }
static int fmt_ebits(int fmt) { return 7 - fmt_mbits(fmt); }
static int fmt_bias(int fmt) { return fmt == ORC_E4M3 ? 7 : 15; }

uint8_t orc_max_finite_code(int fmt) {
    int m = fmt_mbits(fmt);
    return (uint8_t)((((1 << fmt_ebits(fmt)) - 2) << m) | ((1 << m) - 1));
}

/* 2^e exactly, e in [-149, 127]. */
static float pow2_exact(int e) {
    if (e >= -126) return bits_f((uint32_t)(e + 127) << 23);
    return bits_f(1u << (e + 149));
}

float orc_fp8_decode(uint8_t code, int fmt) {
    int m = fmt_mbits(fmt), bias = fmt_bias(fmt);
    float sign = (code & 0x80) ? -1.0f : 1.0f;
    uint32_t mant = code & ((1u << m) - 1u);
    uint32_t ef = (uint32_t)(code & 0x7f) >> m;
    if (ef == (1u << fmt_ebits(fmt)) - 1u) return mant == 0 ? sign * INFINITY : NAN;
    float frac = (float)mant / (float)(1u << m);
    if (ef == 0) return sign * frac * pow2_exact(1 - bias);
    return sign * (1.0f + frac) * pow2_exact((int)ef - bias);
}

float orc_max_finite(int fmt) { return orc_fp8_decode(orc_max_finite_code(fmt), fmt); }

uint8_t orc_fp8_encode(float x, int fmt) {
    uint32_t u = f_bits(x);
    uint8_t sign = (u >> 31) ? 0x80 : 0x00;
    if (isnan(x)) return sign | 0x7f;
    uint32_t mag = u & 0x7fffffffu;
    if ((mag >> 23) == 0) return sign;            /* zero or f32 subnormal */
    int m = fmt_mbits(fmt), bias = fmt_bias(fmt);
    int emin = 1 - bias;
    int emax = ((1 << fmt_ebits(fmt)) - 2) - bias;
    int e = (int)(mag >> 23) - 127;
    if (e > emax) return sign | orc_max_finite_code(fmt);
    int eq = (e > emin ? e : emin);
    float a = bits_f(mag);
    /* a / 2^(eq-m) is exact; rintf rounds ties to even in the default mode */
    uint32_t n = (uint32_t)rintf(a / pow2_exact(eq - m));
    int e_eff = eq;
    if (n >= (2u << m)) { n >>= 1; e_eff += 1; }
    if (e_eff > emax) return sign | orc_max_finite_code(fmt);
    uint32_t code;
    if (e < emin) code = n;                       /* subnormal (or rounds up to min normal) */
    else code = ((uint32_t)(e_eff + bias) << m) | (n - (1u << m));
    return sign | (uint8_t)code;
}

uint32_t orc_choose_exp_bias(float absmax, int fmt) {
    static const uint32_t e4[4] = {15, 11, 7, 3};
    static const uint32_t e5[1] = {15};
    const uint32_t *b = fmt == ORC_E4M3 ? e4 : e5;
    int n = fmt == ORC_E4M3 ? 4 : 1;
    int def = fmt_bias(fmt);
    for (int i = 0; i < n; i++)
        if (absmax <= orc_max_finite(fmt) * pow2_exact(def - (int)b[i])) return b[i];
    return b[n - 1];
}

/* Row absmax of rows [r0, r1). */
static void absmax_rows(const uint16_t *w, int64_t cols, int64_t r0, int64_t r1, float *out) {
    for (int64_t r = r0; r < r1; r++) {
        float m = 0.0f;
        const uint16_t *row = w + r * cols;
        for (int64_t c = 0; c < cols; c++) {
            float v = fabsf(orc_bf16_to_f32(row[c]));
            if (v > m) m = v;
        }
        out[r] = m;
    }
}

static void encode_rows(const uint16_t *w, int64_t cols, const float *scales, int fmt,
                        int64_t r0, int64_t r1, uint8_t *codes) {
    for (int64_t r = r0; r < r1; r++) {
        const uint16_t *row = w + r * cols;
        uint8_t *dst = codes + r * cols;
        float s = scales[r];
        for (int64_t c = 0; c < cols; c++) dst[c] = orc_fp8_encode(orc_bf16_to_f32(row[c]) / s, fmt);
    }
}

/* The reference's thread count: up to 8, one per 2^20 elements, <= rows. */
int orc_split(int64_t rows, int64_t cols) {
    int64_t per = (int64_t)1 << 20;
    int64_t by = (rows * cols + per - 1) / per;
    if (by < 1) by = 1;
    if (by > 8) by = 8;
    if (by > rows) by = rows;
    return (int)by;
}

typedef struct {
    const uint16_t *w; int64_t cols; int64_t r0, r1; float *absmax;
    const float *scales; int fmt; uint8_t *codes; int pass;
} job_t;

static void *job_run(void *p) {
    job_t *j = (job_t *)p;
    if (j->pass == 0) absmax_rows(j->w, j->cols, j->r0, j->r1, j->absmax);
    else encode_rows(j->w, j->cols, j->scales, j->fmt, j->r0, j->r1, j->codes);
    return NULL;
}

/* Run one pass over `threads` contiguous row chunks (ceil split, ragged last). */
static void run_pass(int pass, int threads, const uint16_t *w, int64_t rows, int64_t cols,
                     float *absmax, const float *scales, int fmt, uint8_t *codes) {
    if (threads <= 1) {
        job_t j = {w, cols, 0, rows, absmax, scales, fmt, codes, pass};
        job_run(&j);
        return;
    }
    int64_t chunk = (rows + threads - 1) / threads;
    pthread_t tid[64];
    job_t jobs[64];
    int n = 0;
    for (int64_t r0 = 0; r0 < rows && n < 64; r0 += chunk, n++) {
        int64_t r1 = r0 + chunk < rows ? r0 + chunk : rows;
        jobs[n] = (job_t){w, cols, r0, r1, absmax, scales, fmt, codes, pass};
        pthread_create(&tid[n], NULL, job_run, &jobs[n]);
    }
    for (int i = 0; i < n; i++) pthread_join(tid[i], NULL);
}

/*
 * quantize_with.  `threads` <= 0 takes the reference's own split (<= 8);
 * a positive value forces that many threads (the all-cores CPU baseline).
 * Returns 0, or -1 on the reference's panicking preconditions.
 */
int orc_fp8_quantize(const uint16_t *w, int64_t rows, int64_t cols, int fmt, int scaling,
                     float backoff, int threads, uint8_t *codes, float *scales,
                     uint32_t *exp_bias) {
    if (rows <= 0 || cols <= 0) return -1;
    if (!(backoff > 0.0f) || !isfinite(backoff)) return -1;
    if (fmt != ORC_E4M3 && fmt != ORC_E5M2) return -1;
    if (scaling < ORC_PCS || scaling > ORC_UNIT) return -1;
    int t = threads > 0 ? (threads > 64 ? 64 : threads) : orc_split(rows, cols);
    if (t > rows) t = (int)rows;
    float *absmax = (float *)malloc(sizeof(float) * (size_t)rows);
    if (!absmax) return -1;
    run_pass(0, t, w, rows, cols, absmax, NULL, fmt, NULL);
    float full = orc_max_finite(fmt) * backoff;
    if (scaling == ORC_PCS) {
        for (int64_t r = 0; r < rows; r++) scales[r] = absmax[r] > 0.0f ? absmax[r] / full : 1.0f;
        *exp_bias = (uint32_t)fmt_bias(fmt);
    } else if (scaling == ORC_HW) {
        float tm = 0.0f;
        for (int64_t r = 0; r < rows; r++) tm = fmaxf(tm, absmax[r]);
        uint32_t b = orc_choose_exp_bias(tm / backoff, fmt);
        float s = pow2_exact(fmt_bias(fmt) - (int)b);
        for (int64_t r = 0; r < rows; r++) scales[r] = s;
        *exp_bias = b;
    } else {
        for (int64_t r = 0; r < rows; r++) scales[r] = 1.0f;
        *exp_bias = (uint32_t)fmt_bias(fmt);
    }
    free(absmax);
    run_pass(1, t, w, rows, cols, NULL, scales, fmt, codes);
    return 0;
}

/* Row absmax alone (the reference's row_absmax). */
void orc_row_absmax(const uint16_t *w, int64_t rows, int64_t cols, float *out) {
    absmax_rows(w, cols, 0, rows, out);
}

/* Per-row relative error of the round trip: mean (f64 sum) and max. */
void orc_row_errors(const uint16_t *w, int64_t rows, int64_t cols, const uint8_t *codes,
                    const float *scales, int fmt, float *mean_rel, float *max_rel) {
    for (int64_t r = 0; r < rows; r++) {
        double sum = 0.0;
        float mx = 0.0f;
        int64_t n = 0;
        for (int64_t c = 0; c < cols; c++) {
            float want = orc_bf16_to_f32(w[r * cols + c]);
            if (want == 0.0f) continue;
            float got = orc_fp8_decode(codes[r * cols + c], fmt) * scales[r];
            float rel = fabsf((got - want) / want);
            sum += (double)rel;
            mx = fmaxf(mx, rel);
            n++;
        }
        mean_rel[r] = n == 0 ? 0.0f : (float)(sum / (double)n);
        max_rel[r] = mx;
    }
}

/* Dequantize to f32 (decode * scale), row-major. */
void orc_fp8_dequantize(const uint8_t *codes, const float *scales, int64_t rows, int64_t cols,
                        int fmt, float *out) {
    for (int64_t r = 0; r < rows; r++)
        for (int64_t c = 0; c < cols; c++)
            out[r * cols + c] = orc_fp8_decode(codes[r * cols + c], fmt) * scales[r];
}

/*
 * Order-independent checksum of the encoder over every f32 bit pattern u in
 * [lo, hi): sum of code(u) * ((u & 0xffff) + 1).  Used to compare the device
 * encoder with this one over all 2^32 inputs without moving the codes.
 */
#include <omp.h>
uint64_t orc_encode_checksum(uint64_t lo, uint64_t hi, int fmt, int threads) {
    uint64_t sum = 0;
    if (threads > 0) omp_set_num_threads(threads);
    int64_t n = (int64_t)(hi - lo);
#pragma omp parallel for reduction(+ : sum) schedule(static)
    for (int64_t i = 0; i < n; i++) {
        uint32_t u = (uint32_t)(lo + (uint64_t)i);
        sum += (uint64_t)orc_fp8_encode(bits_f(u), fmt) * (uint64_t)((u & 0xffffu) + 1u);
    }
    return sum;
}

/*
 * af2_oracle.c -- CPU restatement of the reference's f32 maths for the
 * Evoformer pair-stack contractions.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker and the CPU
 * baseline; the product library (libaf2cuda.so) never links, loads or calls
 * it.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
 * use it.
 *
 * Rounding model.  The reference CPU code is TypeScript: every intermediate
 * tensor is a Float32Array (so each stored element is rounded to f32) while
 * every scalar expression is a JS number (f64).  The functions below keep the
 * same two rules -- f64 arithmetic, f32 storage at exactly the points where
 * the reference stores into a Float32Array -- and the same loop orders, so
 * sums accumulate in the same sequence.  Compile without -ffast-math and with
 * -ffp-contract=off so the compiler neither reassociates nor fuses.
 *
 * Parity pin: triangle outgoing is checked against the reference's four
 * frozen bundles (tests/golden).  Incoming, outer-product mean and transition
 * have no frozen bundle in the reference; they follow the formulas cited at
 * each function.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define AF2O_EXPORT __attribute__((visibility("default")))

static void set_threads(int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
}

/* ------------------------------------------------------------------------ */
/* f16 <-> f32, restating src/runtime/float16.ts:5-29 (numberToFloat16) and  */
/* src/reference/dtype.ts:28-35 (float16ToNumber).                           */
/* ------------------------------------------------------------------------ */

AF2O_EXPORT uint16_t af2o_f16_bits(float value) {
    uint32_t bits;
    memcpy(&bits, &value, 4);
    uint32_t sign = (bits >> 16) & 0x8000u;
    int32_t exponent = (int32_t)((bits >> 23) & 0xffu) - 127 + 15;
    uint32_t mantissa = bits & 0x7fffffu;
    if (((bits >> 23) & 0xffu) == 0xffu) return (uint16_t)(sign | (mantissa == 0 ? 0x7c00u : 0x7e00u));
    if (exponent >= 0x1f) return (uint16_t)(sign | 0x7c00u);
    if (exponent <= 0) {
        if (exponent < -10) return (uint16_t)sign;
        /* The reference shifts first and rounds the shifted value. */
        mantissa = (mantissa | 0x800000u) >> (uint32_t)(1 - exponent);
        return (uint16_t)(sign | ((mantissa + 0x0fffu + ((mantissa >> 13) & 1u)) >> 13));
    }
    mantissa += 0x0fffu + ((mantissa >> 13) & 1u);
    if (mantissa & 0x800000u) {
        mantissa = 0;
        exponent += 1;
        if (exponent >= 0x1f) return (uint16_t)(sign | 0x7c00u);
    }
    return (uint16_t)(sign | ((uint32_t)exponent << 10) | (mantissa >> 13));
}

AF2O_EXPORT double af2o_f16_value(uint16_t bits) {
    double sign = (bits & 0x8000u) ? -1.0 : 1.0;
    int exponent = (bits >> 10) & 0x1f;
    int fraction = bits & 0x03ff;
    if (exponent == 0) return fraction == 0 ? sign * 0.0 : sign * ldexp(fraction / 1024.0, -14);
    if (exponent == 0x1f) return fraction == 0 ? sign * INFINITY : NAN;
    return sign * ldexp(1.0 + fraction / 1024.0, exponent - 15);
}

/* ------------------------------------------------------------------------ */
/* Mixed-q8 weights.                                                          */
/* ------------------------------------------------------------------------ */

/* JS Math.round: nearest integer, halves toward +infinity. */
static double js_round(double x) { return floor(x + 0.5); }

/*
 * Block-64 symmetric int8 with an f16 scale per block of the flattened tensor,
 * restating tools/quantize-web-model.ts:98-119: scale = f16(max|w|/127), the
 * decoded scale is replaced by 1 when it is 0, code = clamp(round(w/scale)).
 */
AF2O_EXPORT void af2o_quantize_q8_block(const float *w, int64_t n, int64_t block,
                                        int8_t *codes, uint16_t *scales) {
    int64_t blocks = (n + block - 1) / block;
    for (int64_t b = 0; b < blocks; ++b) {
        int64_t start = b * block, end = start + block < n ? start + block : n;
        double maximum = 0;
        for (int64_t i = start; i < end; ++i) maximum = fmax(maximum, fabs((double)w[i]));
        uint16_t bits = af2o_f16_bits((float)(maximum / 127.0));
        double scale = af2o_f16_value(bits);
        if (scale == 0) scale = 1;
        scales[b] = bits;
        for (int64_t i = start; i < end; ++i) {
            double q = js_round((double)w[i] / scale);
            q = q < -127 ? -127 : (q > 127 ? 127 : q);
            codes[i] = (int8_t)q;
        }
    }
}

/* Decode, restating src/reference/dtype.ts:86-97: w = code * f16(scale[i/block]). */
AF2O_EXPORT void af2o_dequant_q8_block(const int8_t *codes, const uint16_t *scales, int64_t n,
                                       int64_t block, float *out) {
    for (int64_t i = 0; i < n; ++i) out[i] = (float)((double)codes[i] * af2o_f16_value(scales[i / block]));
}

/*
 * Per-output-channel symmetric int8 (the format the benchmark configs name):
 * w is [inner, cols] row-major ([in, out], transition.ts:115); the scale of
 * column o is the f32 value max_k |w[k,o]| / 127 (1 when that is 0), and the
 * decoded weight is the f32 product code * scale.
 */
AF2O_EXPORT void af2o_quantize_q8_columns(const float *w, int64_t inner, int64_t cols,
                                          int8_t *codes, float *scales) {
    for (int64_t o = 0; o < cols; ++o) {
        double maximum = 0;
        for (int64_t k = 0; k < inner; ++k) maximum = fmax(maximum, fabs((double)w[k * cols + o]));
        float scale = (float)(maximum / 127.0);
        if (scale == 0) scale = 1;
        scales[o] = scale;
        for (int64_t k = 0; k < inner; ++k) {
            double q = js_round((double)w[k * cols + o] / (double)scale);
            q = q < -127 ? -127 : (q > 127 ? 127 : q);
            codes[k * cols + o] = (int8_t)q;
        }
    }
}

AF2O_EXPORT void af2o_dequant_q8_columns(const int8_t *codes, const float *scales, int64_t inner,
                                         int64_t cols, float *out) {
    for (int64_t k = 0; k < inner; ++k)
        for (int64_t o = 0; o < cols; ++o)
            out[k * cols + o] = (float)codes[k * cols + o] * scales[o];
}

/* ------------------------------------------------------------------------ */
/* Shared pieces of src/triangle/cpu-reference.ts.                           */
/* ------------------------------------------------------------------------ */

static double sigmoid(double v) { return 1.0 / (1.0 + exp(-v)); }

/* normalizeRows, cpu-reference.ts:6-31 (f64 statistics, f32 output). */
static void normalize_rows(const float *in, int64_t rows, int64_t channels, const float *weight,
                           const float *bias, double eps, float *out) {
#pragma omp parallel for schedule(static)
    for (int64_t row = 0; row < rows; ++row) {
        const float *x = in + row * channels;
        double mean = 0;
        for (int64_t c = 0; c < channels; ++c) mean += x[c];
        mean /= (double)channels;
        double variance = 0;
        for (int64_t c = 0; c < channels; ++c) {
            double centered = x[c] - mean;
            variance += centered * centered;
        }
        double inv = 1.0 / sqrt(variance / (double)channels + eps);
        for (int64_t c = 0; c < channels; ++c)
            out[row * channels + c] = (float)((x[c] - mean) * inv * weight[c] + bias[c]);
    }
}

/* project, cpu-reference.ts:33-54: weight is [out, in] row-major. */
static void project(const float *in, int64_t rows, int64_t cin, int64_t cout, const float *weight,
                    const float *bias, float *out) {
#pragma omp parallel for schedule(static)
    for (int64_t row = 0; row < rows; ++row) {
        for (int64_t o = 0; o < cout; ++o) {
            double value = bias[o];
            const float *w = weight + o * cin;
            const float *x = in + row * cin;
            for (int64_t c = 0; c < cin; ++c) value += (double)x[c] * (double)w[c];
            out[row * cout + o] = (float)value;
        }
    }
}

/*
 * Offsets of the 16 tensors in the packed weight array, in the order of
 * src/triangle/weights.ts:4-10 (ORDER): LN-in w/b, AP w/b, AG w/b, BP w/b,
 * BG w/b, LN-out w/b, Z w/b, G w/b.
 */
typedef struct {
    const float *ln_in_w, *ln_in_b, *ap_w, *ap_b, *ag_w, *ag_b, *bp_w, *bp_b, *bg_w, *bg_b;
    const float *ln_out_w, *ln_out_b, *z_w, *z_b, *g_w, *g_b;
} tri_weights;

static tri_weights unpack_triangle(const float *p, int64_t cz, int64_t ch) {
    tri_weights w;
    w.ln_in_w = p; p += cz;
    w.ln_in_b = p; p += cz;
    w.ap_w = p; p += ch * cz;
    w.ap_b = p; p += ch;
    w.ag_w = p; p += ch * cz;
    w.ag_b = p; p += ch;
    w.bp_w = p; p += ch * cz;
    w.bp_b = p; p += ch;
    w.bg_w = p; p += ch * cz;
    w.bg_b = p; p += ch;
    w.ln_out_w = p; p += ch;
    w.ln_out_b = p; p += ch;
    w.z_w = p; p += cz * ch;
    w.z_b = p; p += cz;
    w.g_w = p; p += cz * cz;
    w.g_b = p;
    return w;
}

/* expectedWeightElementCount, src/triangle/weights.ts:36-40. */
AF2O_EXPORT int64_t af2o_triangle_weight_count(int64_t cz, int64_t ch) {
    return 2 * cz + 4 * (ch * cz + ch) + 2 * ch + (cz * ch + cz) + (cz * cz + cz);
}

/*
 * Triangle multiplication.  direction 0 = outgoing, restating
 * src/triangle/cpu-reference.ts:56-100; direction 1 = incoming, the same
 * with the contraction x[i,j,h] = sum_k a[k,j,h] * b[k,i,h]
 * (src/triangle/shaders.ts:452-455; AlphaFold's 'kjc,kic->ijc').
 * z [n,n,cz], mask [n,n], packed weights in ORDER.  Only the output rows i
 * listed in `rows` (count of them) are produced, into out [count,n,cz] (no
 * residual): the projections cover every pair, the contraction, output
 * LayerNorm and output projection only the listed rows.  Every computed
 * element takes the same operations in the same order as in the whole op.
 */
AF2O_EXPORT int af2o_triangle_rows(int direction, int64_t n, int64_t cz, int64_t ch, const float *z,
                                   const float *mask, const float *packed, double eps, const int64_t *rows,
                                   int64_t count, float *out, int threads) {
    if (n <= 0 || cz <= 0 || ch <= 0 || count <= 0 || (direction != 0 && direction != 1)) return 1;
    for (int64_t r = 0; r < count; ++r)
        if (rows[r] < 0 || rows[r] >= n) return 1;
    set_threads(threads);
    tri_weights w = unpack_triangle(packed, cz, ch);
    int64_t pairs = n * n, sel = count * n;
    float *zn = (float *)malloc(sizeof(float) * pairs * cz);
    float *ap = (float *)malloc(sizeof(float) * pairs * ch);
    float *ag = (float *)malloc(sizeof(float) * pairs * ch);
    float *bp = (float *)malloc(sizeof(float) * pairs * ch);
    float *bg = (float *)malloc(sizeof(float) * pairs * ch);
    float *x = (float *)malloc(sizeof(float) * sel * ch);
    float *xn = (float *)malloc(sizeof(float) * sel * ch);
    float *zs = (float *)malloc(sizeof(float) * sel * cz);
    float *gate = (float *)malloc(sizeof(float) * sel * cz);
    if (!zn || !ap || !ag || !bp || !bg || !x || !xn || !zs || !gate) {
        free(zn); free(ap); free(ag); free(bp); free(bg); free(x); free(xn); free(zs); free(gate);
        return 2;
    }
    normalize_rows(z, pairs, cz, w.ln_in_w, w.ln_in_b, eps, zn);
    project(zn, pairs, cz, ch, w.ap_w, w.ap_b, ap);
    project(zn, pairs, cz, ch, w.ag_w, w.ag_b, ag);
    project(zn, pairs, cz, ch, w.bp_w, w.bp_b, bp);
    project(zn, pairs, cz, ch, w.bg_w, w.bg_b, bg);
    /* cpu-reference.ts:68-75: a = ap * sigmoid(ag) * mask, same for b. */
#pragma omp parallel for schedule(static)
    for (int64_t pair = 0; pair < pairs; ++pair) {
        double m = mask[pair];
        for (int64_t h = 0; h < ch; ++h) {
            int64_t idx = pair * ch + h;
            ap[idx] = (float)((double)ap[idx] * sigmoid(ag[idx]) * m);
            bp[idx] = (float)((double)bp[idx] * sigmoid(bg[idx]) * m);
        }
    }
    /* cpu-reference.ts:77-89 (outgoing) and the transposed einsum (incoming). */
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < count; ++r) {
        const int64_t i = rows[r];
        for (int64_t j = 0; j < n; ++j) {
            for (int64_t h = 0; h < ch; ++h) {
                double value = 0;
                if (direction == 0) {
                    for (int64_t k = 0; k < n; ++k)
                        value += (double)ap[(i * n + k) * ch + h] * (double)bp[(j * n + k) * ch + h];
                } else {
                    for (int64_t k = 0; k < n; ++k)
                        value += (double)ap[(k * n + j) * ch + h] * (double)bp[(k * n + i) * ch + h];
                }
                x[(r * n + j) * ch + h] = (float)value;
            }
        }
        memcpy(zs + r * n * cz, zn + i * n * cz, sizeof(float) * n * cz);
    }
    /* cpu-reference.ts:91-99. */
    normalize_rows(x, sel, ch, w.ln_out_w, w.ln_out_b, eps, xn);
    project(xn, sel, ch, cz, w.z_w, w.z_b, out);
    project(zs, sel, cz, cz, w.g_w, w.g_b, gate);
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < sel * cz; ++idx) out[idx] = (float)((double)out[idx] * sigmoid(gate[idx]));
    free(zn); free(ap); free(ag); free(bp); free(bg); free(x); free(xn); free(zs); free(gate);
    return 0;
}

/* The whole op: every output row. */
AF2O_EXPORT int af2o_triangle(int direction, int64_t n, int64_t cz, int64_t ch, const float *z,
                              const float *mask, const float *packed, double eps, float *out,
                              int threads) {
    if (n <= 0) return 1;
    int64_t *rows = (int64_t *)malloc(sizeof(int64_t) * n);
    if (!rows) return 2;
    for (int64_t i = 0; i < n; ++i) rows[i] = i;
    int rc = af2o_triangle_rows(direction, n, cz, ch, z, mask, packed, eps, rows, n, out, threads);
    free(rows);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* Outer-product mean, restating test/outer-product-mean-reference.gpu.test.ts:22-79 */
/* (the reference's independent CPU formulation of OuterProductMeanGpu).     */
/* Packed weights in the order of src/evoformer/outer-product-mean.ts:68-72: */
/* LN scale [cm], LN offset [cm], left W [cm,c] ([in,out]), left b [c],      */
/* right W [cm,c], right b [c], output W [c*c, cz] (index (a*c+b)*cz+z),     */
/* output b [cz].                                                            */
/* ------------------------------------------------------------------------ */

AF2O_EXPORT int64_t af2o_opm_weight_count(int64_t cm, int64_t c, int64_t cz) {
    return 2 * cm + 2 * (cm * c + c) + c * c * cz + cz;
}

AF2O_EXPORT int af2o_outer_product_mean(int64_t s, int64_t n, int64_t cm, int64_t c, int64_t cz,
                                        const float *m, const float *mask, const float *packed,
                                        double ln_eps, double norm_eps, float *out, int threads) {
    if (s <= 0 || n <= 0 || cm <= 0 || c <= 0 || cz <= 0) return 1;
    set_threads(threads);
    const float *ln_w = packed, *ln_b = ln_w + cm, *lw = ln_b + cm, *lb = lw + cm * c;
    const float *rw = lb + c, *rb = rw + cm * c, *ow = rb + c, *ob = ow + c * c * cz;
    int64_t rows = s * n;
    float *normalized = (float *)malloc(sizeof(float) * rows * cm);
    float *left = (float *)malloc(sizeof(float) * rows * c);
    float *right = (float *)malloc(sizeof(float) * rows * c);
    if (!normalized || !left || !right) { free(normalized); free(left); free(right); return 2; }
    normalize_rows(m, rows, cm, ln_w, ln_b, ln_eps, normalized);
#pragma omp parallel for schedule(static)
    for (int64_t row = 0; row < rows; ++row) {
        for (int64_t o = 0; o < c; ++o) {
            double tl = lb[o], tr = rb[o];
            for (int64_t k = 0; k < cm; ++k) {
                tl += (double)normalized[row * cm + k] * (double)lw[k * c + o];
                tr += (double)normalized[row * cm + k] * (double)rw[k * c + o];
            }
            left[row * c + o] = (float)((double)mask[row] * tl);
            right[row * c + o] = (float)((double)mask[row] * tr);
        }
    }
#pragma omp parallel
    {
        float *pair = (float *)malloc(sizeof(float) * c * c);
#pragma omp for schedule(static)
        for (int64_t ij = 0; ij < n * n; ++ij) {
            int64_t i = ij / n, j = ij % n;
            memset(pair, 0, sizeof(float) * c * c);
            double count = 0;
            for (int64_t q = 0; q < s; ++q) {
                count += (double)mask[q * n + i] * (double)mask[q * n + j];
                const float *l = left + (q * n + i) * c, *r = right + (q * n + j) * c;
                for (int64_t a = 0; a < c; ++a) {
                    double lv = l[a];
                    /* pair is a Float32Array in the reference: each += rounds to f32. */
                    for (int64_t b = 0; b < c; ++b) pair[a * c + b] = (float)((double)pair[a * c + b] + lv * (double)r[b]);
                }
            }
            double scale = 1.0 / (norm_eps + count);
            for (int64_t zc = 0; zc < cz; ++zc) {
                double total = ob[zc];
                for (int64_t k = 0; k < c * c; ++k) total += (double)pair[k] * (double)ow[k * cz + zc];
                out[ij * cz + zc] = (float)(total * scale);
            }
        }
        free(pair);
    }
    free(normalized); free(left); free(right);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Transition (MSA / pair), restating src/evoformer/transition.ts:91-138 and */
/* :185-232: LN (eps), hidden = relu(x W1 + b1), out = hidden W2 + b2, with   */
/* W1 [C, H] and W2 [H, C] in [in, out] layout (transition.ts:115).          */
/* Packed order (transition.ts:140-177): LN scale [C], LN offset [C], W1,    */
/* b1 [H], W2, b2 [C].  residual != 0 adds the input (the in-model form,     */
/* block.ts:625-740).                                                        */
/* ------------------------------------------------------------------------ */

AF2O_EXPORT int64_t af2o_transition_weight_count(int64_t c, int64_t h) {
    return 2 * c + c * h + h + h * c + c;
}

AF2O_EXPORT int af2o_transition(int64_t rows, int64_t c, int64_t h, const float *x, const float *packed,
                                double eps, int residual, float *out, int threads) {
    if (rows <= 0 || c <= 0 || h <= 0) return 1;
    set_threads(threads);
    const float *ln_w = packed, *ln_b = ln_w + c, *w1 = ln_b + c, *b1 = w1 + c * h;
    const float *w2 = b1 + h, *b2 = w2 + h * c;
    float *normalized = (float *)malloc(sizeof(float) * rows * c);
    if (!normalized) return 2;
    normalize_rows(x, rows, c, ln_w, ln_b, eps, normalized);
#pragma omp parallel
    {
        float *hidden = (float *)malloc(sizeof(float) * h);
#pragma omp for schedule(static)
        for (int64_t row = 0; row < rows; ++row) {
            const float *xn = normalized + row * c;
            for (int64_t o = 0; o < h; ++o) {
                double v = b1[o];
                for (int64_t k = 0; k < c; ++k) v += (double)xn[k] * (double)w1[k * h + o];
                hidden[o] = (float)(v > 0 ? v : 0);
            }
            for (int64_t o = 0; o < c; ++o) {
                double v = b2[o];
                for (int64_t k = 0; k < h; ++k) v += (double)hidden[k] * (double)w2[k * c + o];
                out[row * c + o] = (float)(residual ? (double)x[row * c + o] + (float)v : v);
            }
        }
        free(hidden);
    }
    free(normalized);
    return 0;
}

/* errorMetrics, src/triangle/types.ts:91-110: mean / max / RMS of |a - e|. */
AF2O_EXPORT int af2o_error_metrics(const float *actual, const float *expected, int64_t n, double *metrics) {
    if (n <= 0) return 1;
    double sum = 0, sq = 0, mx = 0;
    for (int64_t i = 0; i < n; ++i) {
        double d = fabs((double)actual[i] - (double)expected[i]);
        sum += d;
        sq += d * d;
        mx = fmax(mx, d);
    }
    metrics[0] = sum / (double)n;
    metrics[1] = mx;
    metrics[2] = sqrt(sq / (double)n);
    return 0;
}

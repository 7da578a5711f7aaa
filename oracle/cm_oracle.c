/* cm_oracle.c -- CPU restatement of the four Cormorant kernels (see cm_oracle.h).
 *
 * TEST INFRASTRUCTURE ONLY.  The arithmetic restates the reference C-simulation
 * semantics of ap_fixed<16,8> data with ap_fixed<32,16> accumulators:
 *   - products are exact at 2^-16, the accumulator is int32 that wraps mod 2^32
 *     (AP_WRAP), so any summation order gives the same bits;
 *   - one saturating narrowing at the output: floor (AP_TRN) to 2^-8, clamp to
 *     int16 (AP_SAT)  -- saturate_cast, kernels/matmul/include/MatmulKernel.h:23-38;
 *   - pooling AVG / LP(p!=1) go through IEEE float32 exactly as
 *     kernels/pool/kernel/PoolingKernel.cpp:168-172 and :253-263 do.
 * Accumulation uses uint32 arithmetic, which is the same ring as the wrap.
 */
#include "cm_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* helpers                                                                   */
/* ------------------------------------------------------------------------ */

static inline int16_t sat16(int64_t v) {
    if (v > 32767) return 32767;
    if (v < -32768) return -32768;
    return (int16_t)v;
}

/* floor(v / 2^s) for signed v without relying on >> of negatives */
static inline int64_t floor_shift(int64_t v, int s) {
    const int64_t d = (int64_t)1 << s;
    int64_t q = v / d;
    if ((v % d) != 0 && v < 0) q -= 1;
    return q;
}

static inline int32_t as_i32(uint32_t u) { return (int32_t)u; }

/* saturate_cast<ap_fixed<16,8>>(ap_fixed<32,16> acc): floor by 8 bits, clamp. */
static inline int16_t narrow_acc(uint32_t acc) { return sat16(floor_shift((int64_t)as_i32(acc), 8)); }

/* AccData_t(float f): exact value floored to 2^-16, then wrapped into 32 bits.
 * NaN gives 0 (the oracle fixed-point shim's rule, oracle/ap_fixed.h). */
static inline uint32_t acc_from_float(float f) {
    if (isnan(f)) return 0u;
    const double t = floor((double)f * 65536.0); /* exact: |f| <= 2^15 here */
    const int64_t r = (int64_t)t;
    return (uint32_t)(uint64_t)r;
}

/* (float)acc for ap_fixed<32,16>: round the exact value to nearest-even. */
static inline float acc_to_float(uint32_t acc) { return (float)as_i32(acc) * 0x1p-16f; }

/* ------------------------------------------------------------------------ */
/* threads                                                                   */
/* ------------------------------------------------------------------------ */

static int g_threads = 1;
void orc_set_threads(int n) { g_threads = n < 1 ? 1 : (n > 256 ? 256 : n); }
int orc_get_threads(void) { return g_threads; }

typedef void (*range_fn)(void* ctx, uint64_t lo, uint64_t hi);
typedef struct { range_fn fn; void* ctx; uint64_t lo, hi; } job_t;

static void* job_main(void* p) {
    job_t* j = (job_t*)p;
    j->fn(j->ctx, j->lo, j->hi);
    return NULL;
}

static void par_for(uint64_t n, range_fn fn, void* ctx) {
    int t = g_threads;
    if ((uint64_t)t > n) t = (int)n;
    if (t <= 1) { if (n) fn(ctx, 0, n); return; }
    pthread_t th[256];
    job_t jobs[256];
    for (int i = 0; i < t; ++i) {
        jobs[i].fn = fn; jobs[i].ctx = ctx;
        jobs[i].lo = n * (uint64_t)i / (uint64_t)t;
        jobs[i].hi = n * (uint64_t)(i + 1) / (uint64_t)t;
        pthread_create(&th[i], NULL, job_main, &jobs[i]);
    }
    for (int i = 0; i < t; ++i) pthread_join(th[i], NULL);
}

/* ------------------------------------------------------------------------ */
/* VectorOP -- kernels/vectorop/kernel/VectorOP.cpp:8-35 (ops), :98-110 (switch) */
/* ------------------------------------------------------------------------ */

int16_t orc_vectorop_scalar(uint32_t op, int16_t a, int16_t b) {
    switch (op) {
        case 0: return sat16((int64_t)a + b);                         /* OP_ADD  :8-10  */
        case 1: return sat16((int64_t)a - b);                         /* OP_SUB  :12-14 */
        case 2: return sat16(floor_shift((int64_t)a * b, 8));         /* OP_MUL  :17-19 */
        case 3:                                                       /* OP_DIV  :22-25 */
            if (b == 0) return 0;
            return sat16(((int64_t)a * 256) / (int64_t)b);            /* C division truncates toward zero */
        case 4: return a < 0 ? 0 : a;                                 /* OP_RELU :27-29 */
        case 5: return a < 0 ? 0 : (a > 0x600 ? 0x600 : a);           /* OP_RELU6 :31-35 */
        default: return a;                                            /* default  :108 */
    }
}

/* c[o*(a_inc+b_inc)+i] = op(a[o*a_inc+i], b[o*b_inc+i]), written in (o, i)
 * order so that a later write to the same c element wins (VectorOP.cpp:140-188). */
void orc_vectorop(const int16_t* a, const int16_t* b, int16_t* c, uint32_t size, uint32_t op,
                  uint32_t outer, uint32_t a_inc, uint32_t b_inc) {
    const uint64_t c_inc = (uint64_t)a_inc + (uint64_t)b_inc;
    const int unary = op >= 4;
    for (uint64_t o = 0; o < outer; ++o) {
        const int16_t* ap = a + o * a_inc;
        const int16_t* bp = unary ? NULL : b + o * b_inc;
        int16_t* cp = c + o * c_inc;
        for (uint64_t i = 0; i < size; ++i) cp[i] = orc_vectorop_scalar(op, ap[i], unary ? 0 : bp[i]);
    }
}

typedef struct { uint32_t op; int32_t a_first; const int16_t* got; uint64_t bad; int64_t first; pthread_mutex_t mu; } chk_ctx;

static void chk_range(void* p, uint64_t lo, uint64_t hi) {
    chk_ctx* x = (chk_ctx*)p;
    uint64_t bad = 0; int64_t first = -1;
    for (uint64_t r = lo; r < hi; ++r) {
        const int16_t av = (int16_t)(x->a_first + (int32_t)r);
        const int16_t* g = x->got + r * 65536u;
        for (int32_t bi = 0; bi < 65536; ++bi) {
            const int16_t bv = (int16_t)(bi - 32768);
            if (g[bi] != orc_vectorop_scalar(x->op, av, bv)) {
                if (first < 0) first = (int64_t)(r * 65536u + (uint64_t)bi);
                ++bad;
            }
        }
    }
    pthread_mutex_lock(&x->mu);
    x->bad += bad;
    if (first >= 0 && (x->first < 0 || first < x->first)) x->first = first;
    pthread_mutex_unlock(&x->mu);
}

uint64_t orc_vectorop_check_pairs(uint32_t op, int32_t a_first, uint32_t a_count, const int16_t* got,
                                  int64_t* first_bad) {
    chk_ctx x;
    x.op = op; x.a_first = a_first; x.got = got; x.bad = 0; x.first = -1;
    pthread_mutex_init(&x.mu, NULL);
    par_for(a_count, chk_range, &x);
    pthread_mutex_destroy(&x.mu);
    if (first_bad) *first_bad = x.first;
    return x.bad;
}

/* ------------------------------------------------------------------------ */
/* MatMul -- kernels/matmul/kernel/MatmulKernel.cpp:108-219                   */
/* C[b][r][col] = sat(floor((sum_k A[b][r][k] * B[b][k][col]) mod 2^32 / 256))  */
/* ------------------------------------------------------------------------ */

static void matmul_row(const int16_t* ap, const int16_t* bp, uint32_t k, uint32_t m, int16_t* out,
                       uint32_t* acc) {
    memset(acc, 0, sizeof(uint32_t) * m);                         /* acc clear :160-167 */
    for (uint32_t kk = 0; kk < k; ++kk) {
        const int32_t av = ap[kk];
        const int16_t* brow = bp + (uint64_t)kk * m;
        for (uint32_t j = 0; j < m; ++j) acc[j] += (uint32_t)(av * (int32_t)brow[j]); /* MAC :204 */
    }
    for (uint32_t j = 0; j < m; ++j) out[j] = narrow_acc(acc[j]);  /* saturate_cast :217-218 */
}

typedef struct {
    const int16_t *a, *b; int16_t* c; uint32_t n, k, m;
    uint64_t a_bs, b_bs, c_bs; const uint32_t *bidx, *ridx; int16_t* out;
} mm_ctx;

static void mm_range(void* p, uint64_t lo, uint64_t hi) {
    mm_ctx* x = (mm_ctx*)p;
    uint32_t* acc = (uint32_t*)malloc(sizeof(uint32_t) * (x->m ? x->m : 1));
    for (uint64_t t = lo; t < hi; ++t) {
        const uint64_t bi = t / x->n, r = t % x->n;
        matmul_row(x->a + bi * x->a_bs + r * x->k, x->b + bi * x->b_bs, x->k, x->m,
                   x->c + bi * x->c_bs + r * x->m, acc);
    }
    free(acc);
}

void orc_matmul(const int16_t* a, const int16_t* b, int16_t* c, uint32_t n, uint32_t k, uint32_t m,
                uint32_t batch, uint32_t a_batch_stride, uint32_t b_batch_stride,
                uint32_t c_batch_stride) {
    if (batch > 1 && (uint64_t)c_batch_stride < (uint64_t)n * m) {
        /* output slices of different batch steps overlap: the reference's batch loop runs in
           order and later steps overwrite earlier ones (:108-112), so the steps run one after
           another here too (rows of one step never overlap) */
        for (uint32_t bi = 0; bi < batch; ++bi) {
            mm_ctx x = {a + (uint64_t)bi * a_batch_stride, b + (uint64_t)bi * b_batch_stride,
                        c + (uint64_t)bi * c_batch_stride, n, k, m, 0, 0, 0, NULL, NULL, NULL};
            par_for(n, mm_range, &x);
        }
        return;
    }
    mm_ctx x = {a, b, c, n, k, m, a_batch_stride, b_batch_stride, c_batch_stride, NULL, NULL, NULL};
    par_for((uint64_t)batch * n, mm_range, &x);
}

static void mm_rows_range(void* p, uint64_t lo, uint64_t hi) {
    mm_ctx* x = (mm_ctx*)p;
    uint32_t* acc = (uint32_t*)malloc(sizeof(uint32_t) * (x->m ? x->m : 1));
    for (uint64_t t = lo; t < hi; ++t)
        matmul_row(x->a + (uint64_t)x->bidx[t] * x->a_bs + (uint64_t)x->ridx[t] * x->k,
                   x->b + (uint64_t)x->bidx[t] * x->b_bs, x->k, x->m, x->out + t * x->m, acc);
    free(acc);
}

void orc_matmul_rows(const int16_t* a, const int16_t* b, uint32_t n, uint32_t k, uint32_t m,
                     uint32_t a_batch_stride, uint32_t b_batch_stride, const uint32_t* bidx,
                     const uint32_t* ridx, uint32_t count, int16_t* out) {
    mm_ctx x = {a, b, NULL, n, k, m, a_batch_stride, b_batch_stride, 0, bidx, ridx, out};
    par_for(count, mm_rows_range, &x);
}

/* ------------------------------------------------------------------------ */
/* Conv -- kernels/conv/kernel/ConvKernel.cpp:142-342                          */
/* standard: y[n][m][oh][ow] = sat(floor((bias[m]<<8 + sum_{c,r,s} x*w) / 256)) */
/* depthwise: input channel = output channel m, weights [M][1][kh][kw]          */
/* out-of-bounds input taps read 0 (:184-202, :262-279)                         */
/* ------------------------------------------------------------------------ */

typedef struct {
    const int16_t *x, *w, *bias; int16_t* y;
    uint32_t in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, sh, sw, dh, dw, pt, pl, has_bias, dwise;
    const uint32_t *nidx, *midx; int16_t* out;
} conv_ctx;

static void conv_plane(const conv_ctx* p, uint64_t n, uint64_t m, int16_t* dst) {
    const uint64_t plane = (uint64_t)p->in_h * p->in_w;
    for (uint32_t oh = 0; oh < p->out_h; ++oh) {
        for (uint32_t ow = 0; ow < p->out_w; ++ow) {
            uint32_t acc = p->has_bias ? (uint32_t)((int32_t)p->bias[m] * 256) : 0u; /* bias init :160-169 */
            const uint32_t c_lo = p->dwise ? (uint32_t)m : 0u;
            const uint32_t c_hi = p->dwise ? (uint32_t)m + 1u : p->in_ch;
            for (uint32_t c = c_lo; c < c_hi; ++c) {
                const int16_t* xc = p->x + (n * p->in_ch + c) * plane;
                const int16_t* wc = p->dwise ? p->w + m * (uint64_t)p->kh * p->kw
                                             : p->w + (m * p->in_ch + c) * (uint64_t)p->kh * p->kw;
                for (uint32_t r = 0; r < p->kh; ++r) {
                    const int64_t ih = (int64_t)oh * p->sh + (int64_t)r * p->dh - (int64_t)p->pt;
                    if (ih < 0 || ih >= (int64_t)p->in_h) continue;
                    for (uint32_t s = 0; s < p->kw; ++s) {
                        const int64_t iw = (int64_t)ow * p->sw + (int64_t)s * p->dw - (int64_t)p->pl;
                        if (iw < 0 || iw >= (int64_t)p->in_w) continue;
                        acc += (uint32_t)((int32_t)xc[ih * p->in_w + iw] * (int32_t)wc[r * p->kw + s]);
                    }
                }
            }
            dst[(uint64_t)oh * p->out_w + ow] = narrow_acc(acc);           /* write :329-335 */
        }
    }
}

static void conv_range(void* pp, uint64_t lo, uint64_t hi) {
    conv_ctx* p = (conv_ctx*)pp;
    const uint64_t ohw = (uint64_t)p->out_h * p->out_w;
    for (uint64_t t = lo; t < hi; ++t) {
        const uint64_t n = t / p->out_ch, m = t % p->out_ch;
        conv_plane(p, n, m, p->y + t * ohw);
    }
}

static void conv_sel_range(void* pp, uint64_t lo, uint64_t hi) {
    conv_ctx* p = (conv_ctx*)pp;
    const uint64_t ohw = (uint64_t)p->out_h * p->out_w;
    for (uint64_t t = lo; t < hi; ++t) conv_plane(p, p->nidx[t], p->midx[t], p->out + t * ohw);
}

void orc_conv(const int16_t* x, const int16_t* w, const int16_t* bias, int16_t* y, uint32_t batch,
              uint32_t in_ch, uint32_t in_h, uint32_t in_w, uint32_t out_ch, uint32_t out_h,
              uint32_t out_w, uint32_t kh, uint32_t kw, uint32_t stride_h, uint32_t stride_w,
              uint32_t dilation_h, uint32_t dilation_w, uint32_t pad_top, uint32_t pad_left,
              uint32_t has_bias, uint32_t is_depthwise) {
    conv_ctx p = {x, w, bias, y, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h, stride_w,
                  dilation_h, dilation_w, pad_top, pad_left, has_bias, is_depthwise, NULL, NULL, NULL};
    par_for((uint64_t)batch * out_ch, conv_range, &p);
}

void orc_conv_planes(const int16_t* x, const int16_t* w, const int16_t* bias, uint32_t in_ch,
                     uint32_t in_h, uint32_t in_w, uint32_t out_ch, uint32_t out_h, uint32_t out_w,
                     uint32_t kh, uint32_t kw, uint32_t stride_h, uint32_t stride_w,
                     uint32_t dilation_h, uint32_t dilation_w, uint32_t pad_top,
                     uint32_t pad_left, uint32_t has_bias, uint32_t is_depthwise,
                     const uint32_t* nidx, const uint32_t* midx, uint32_t count, int16_t* out) {
    conv_ctx p = {x, w, bias, NULL, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h, stride_w,
                  dilation_h, dilation_w, pad_top, pad_left, has_bias, is_depthwise, nidx, midx, out};
    par_for(count, conv_sel_range, &p);
}

/* ------------------------------------------------------------------------ */
/* Pooling -- kernels/pool/kernel/PoolingKernel.cpp:112-267                   */
/* ------------------------------------------------------------------------ */

typedef struct {
    const int16_t* x; int16_t* y;
    uint32_t channels, in_h, in_w, out_h, out_w, ph, pw, sh, sw, pt, pl, dh, dw, type, lp, cip;
} pool_ctx;

static void pool_range(void* pp, uint64_t lo, uint64_t hi) {
    const pool_ctx* p = (const pool_ctx*)pp;
    const uint64_t plane = (uint64_t)p->in_h * p->in_w, ohw = (uint64_t)p->out_h * p->out_w;
    for (uint64_t t = lo; t < hi; ++t) {               /* t = n * channels + c */
        const int16_t* xc = p->x + t * plane;
        int16_t* yc = p->y + t * ohw;
        for (uint32_t oh = 0; oh < p->out_h; ++oh) {
            for (uint32_t ow = 0; ow < p->out_w; ++ow) {
                /* valid_count and reciprocal, :122-137 */
                uint32_t valid = 0;
                uint32_t acc = (p->type == 0) ? 0x80000000u : 0u;   /* kAccMin = -32768.0 :193-197 */
                for (uint32_t r = 0; r < p->ph; ++r) {
                    const int64_t ih = (int64_t)oh * p->sh + (int64_t)r * p->dh - (int64_t)p->pt;
                    for (uint32_t s = 0; s < p->pw; ++s) {
                        const int64_t iw = (int64_t)ow * p->sw + (int64_t)s * p->dw - (int64_t)p->pl;
                        const int ok = ih >= 0 && ih < (int64_t)p->in_h && iw >= 0 && iw < (int64_t)p->in_w;
                        if (ok) ++valid;
                        /* window value; padded taps hold -128 for MAX, 0 otherwise (:168-172) */
                        const int32_t v = ok ? xc[ih * p->in_w + iw] : (p->type == 0 ? -32768 : 0);
                        const uint32_t val = (uint32_t)(v * 256);           /* AccData_t(x) */
                        if (p->type == 0) {                                 /* MAX :212-213 */
                            if (as_i32(val) > as_i32(acc)) acc = val;
                        } else if (p->type == 1) {                          /* AVG :214-215 */
                            acc += val;
                        } else if (p->lp == 1u) {                           /* LP1: |x|, :220-221 */
                            acc += (uint32_t)((v < 0 ? -v : v) * 256);
                        } else {                                            /* LP2: x*x, :222 */
                            acc += (uint32_t)(v * v);
                        }
                    }
                }
                const uint32_t denom = p->cip ? p->ph * p->pw : valid;
                const float inv = denom > 0u ? 1.0f / (float)denom : 0.0f;
                uint32_t res;                                                /* finalize :253-263 */
                if (p->type == 0) res = acc;
                else if (p->type == 1) res = acc_from_float(acc_to_float(acc) * inv);
                else res = (p->lp == 1u) ? acc : acc_from_float(sqrtf(acc_to_float(acc)));
                yc[(uint64_t)oh * p->out_w + ow] = narrow_acc(res);
            }
        }
    }
}

void orc_pool(const int16_t* x, int16_t* y, uint32_t batch, uint32_t channels, uint32_t in_h,
              uint32_t in_w, uint32_t out_h, uint32_t out_w, uint32_t pool_h, uint32_t pool_w,
              uint32_t stride_h, uint32_t stride_w, uint32_t pad_top, uint32_t pad_left,
              uint32_t dil_h, uint32_t dil_w, uint32_t pool_type, uint32_t lp_order,
              uint32_t count_include_pad) {
    pool_ctx p = {x, y, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h, stride_w,
                  pad_top, pad_left, dil_h, dil_w, pool_type, lp_order, count_include_pad};
    par_for((uint64_t)batch * channels, pool_range, &p);
}

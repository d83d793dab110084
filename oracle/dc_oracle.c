/*
 * dc_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of DenseCore's float32 CPU flash-attention path, used as the
 * parity checker for the CUDA kernels and as the timed CPU baseline. Nothing in the
 * product library links or calls this file; only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg load it.
 *
 * What it restates (paths are inside the DenseCore project):
 *   src/torch_attention.rs:14-40    KV_SPLIT, q_split, scale_factor
 *   src/torch_attention.rs:42-105   std_max, mul_reduce_max, exp_reduce_sum
 *   src/torch_attention.rs:107-128  par_chunks (independent (batch, head) tasks)
 *   src/torch_attention.rs:130-141  scale_add_mask
 *   src/torch_attention.rs:146-284  forward
 *   src/torch_attention.rs:291-468  backward
 *   src/torch_softmax.rs:14-54      reduce_all, add, maximum
 *   src/torch_softmax.rs:57-67,90-97 softmax_lastdim, softmax_backward_lastdim (MHA math path)
 *   src/torch_blas.rs:59-79         normalize_last_dims
 *   src/torch_blas.rs:94-133        the portable (non-macOS) column-major sgemm_
 *   src/torch_blas.rs:404-445       bmm (MHA math path)
 *   src/torch_blas.rs:584-642       gemm_raw
 *   src/sleef.rs:310-322,499-515    SLEEF xexpf (ldexp2 / pow2i helpers)
 *   src/sleef.rs:1184-1196          libm expf / logf (glibc here, as on any Linux build)
 *   src/sleef.rs:1227-1256          exp_u20 (Arm Optimized Routines vexpq_f32_u20)
 *   src/torch_random.rs:9-13,43-97  mt19937: seeding, twist, tempering, random, random64
 *   src/torch_random.rs:106-110     uniform_real_distribution<double> (53 bits)
 *   src/torch_random.rs:242-254     bernoulli with a scalar p (the dropout keep draw)
 *
 * Rounding rules that matter for parity: build with -ffp-contract=off so that no a*b+c is
 * fused behind our back; fmaf() is used exactly where the Rust code calls mul_add (or a
 * SLEEF/AOR fused helper). Sums are sequential in the reference's order.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define DCO_EXPORT __attribute__((visibility("default")))

enum { DCO_OK = 0, DCO_EVALUE = 1, DCO_ERUNTIME = 2, DCO_ENOMEM = 3 };

static const size_t KV_SPLIT = 512; /* torch_attention.rs:14 */

/* ---------------------------------------------------------------- scalar helpers -- */

static inline float f_from_bits(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static inline uint32_t f_bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

/* torch_softmax.rs:44-54 -- NEON FMAX: NaN if either is NaN; max(+0,-0) is +0. */
static inline float maximum(float a, float b) {
    if (isnan(a) || isnan(b)) return NAN;
    if (a == b) return signbit(a) ? b : a;
    return a > b ? a : b;
}
static inline float add(float a, float b) { return a + b; }

/* torch_attention.rs:42-45 -- std::max: the first unless it is less than the second. */
static inline float std_max(float a, float b) { return a < b ? b : a; }

typedef float (*dco_op)(float, float);

/* torch_softmax.rs:14-37 -- vec::reduce_all over 4 lanes, then op(op(a0,a2), op(a1,a3)). */
static float reduce_all(const float *v, size_t size, dco_op op) {
    if (size < 4) {
        float acc = v[0];
        for (size_t i = 1; i < size; i++) acc = op(acc, v[i]);
        return acc;
    }
    float acc[4] = {v[0], v[1], v[2], v[3]};
    size_t whole = size - size % 4, d = 4;
    while (d < whole) {
        for (int l = 0; l < 4; l++) acc[l] = op(acc[l], v[d + l]);
        d += 4;
    }
    for (size_t l = 0; l < size - d; l++) acc[l] = op(acc[l], v[d + l]);
    return op(op(acc[0], acc[2]), op(acc[1], acc[3]));
}

/* reduce_all over the products g[i]*y[i] (the map2_reduce_all form). */
static float reduce_all_dot(const float *g, const float *y, size_t size) {
    if (size < 4) {
        float acc = g[0] * y[0];
        for (size_t i = 1; i < size; i++) acc = acc + g[i] * y[i];
        return acc;
    }
    float acc[4];
    for (int l = 0; l < 4; l++) acc[l] = g[l] * y[l];
    size_t whole = size - size % 4, d = 4;
    while (d < whole) {
        for (int l = 0; l < 4; l++) acc[l] = acc[l] + g[d + l] * y[d + l];
        d += 4;
    }
    for (size_t l = 0; l < size - d; l++) acc[l] = acc[l] + g[d + l] * y[d + l];
    return (acc[0] + acc[2]) + (acc[1] + acc[3]);
}

/* ------------------------------------------------------------------- exp / log -- */

/* sleef.rs:313-322 -- vpow2i / vldexp2. */
static inline float pow2i(int32_t q) { return f_from_bits((uint32_t)(q + 0x7f) << 23); }
static inline float ldexp2(float d, int32_t e) {
    int32_t h = e >> 1; /* arithmetic shift, as vshrq_n_s32 */
    return d * pow2i(h) * pow2i(e - h);
}

/* SLEEF xexpf (1.0 ULP), sleef.rs:497-515. The polynomial coefficients are SLEEF's
 * published ones, written as C double literals converted to float, as SLEEF does. */
DCO_EXPORT float dco_sleef_expf(float d) {
    const float R_LN2F = 1.442695040888963407359924681001892137426645954152985934135449406931f;
    const float L2UF = 0.693145751953125f;
    const float L2LF = 1.428606765330187045e-06f;
    float t = d * R_LN2F;
    int32_t q = (int32_t)nearbyintf(t); /* round half to even */
    float qf = (float)q;
    float s = fmaf(qf, -L2UF, d);
    s = fmaf(qf, -L2LF, s);
    float u = (float)0.000198527617612853646278381;
    u = fmaf(u, s, (float)0.00139304355252534151077271);
    u = fmaf(u, s, (float)0.00833336077630519866943359);
    u = fmaf(u, s, (float)0.0416664853692054748535156);
    u = fmaf(u, s, (float)0.166666671633720397949219);
    u = fmaf(u, s, (float)0.5);
    u = 1.0f + fmaf(s * s, u, s);
    u = ldexp2(u, q);
    if (d < -104.0f) u = 0.0f;
    if (100.0f < d) u = INFINITY;
    return u;
}

/* exp_u20, sleef.rs:1227-1256 (Arm Optimized Routines vexpq_f32_u20): a 4-lane group with
 * any |x| > 0x1.5d5e2ap+6 goes to SLEEF expf as a whole. */
static void exp_u20(const float x[4], float y[4]) {
    const float BOUND = f_from_bits(0x42AEAF15u);
    int big = 0;
    for (int l = 0; l < 4; l++) big |= fabsf(x[l]) > BOUND;
    if (big) {
        for (int l = 0; l < 4; l++) y[l] = dco_sleef_expf(x[l]);
        return;
    }
    const float INV_LN2 = f_from_bits(0x3FB8AA3Bu), LN2_HI = f_from_bits(0x3F317200u),
                LN2_LO = f_from_bits(0x35BFBE8Eu), C0 = f_from_bits(0x3C072010u),
                C1 = f_from_bits(0x3D2B9F17u), C2 = f_from_bits(0x3E2AAF33u),
                C3 = f_from_bits(0x3EFFFEDBu), C4 = f_from_bits(0x3F7FFFF6u);
    for (int l = 0; l < 4; l++) {
        float n = roundf(x[l] * INV_LN2); /* vrndaq: halves away from zero */
        float r = fmaf(-n, LN2_HI, x[l]);
        r = fmaf(-n, LN2_LO, r);
        float scale = f_from_bits((uint32_t)(((int32_t)n << 23) + 0x3f800000));
        float r2 = r * r;
        float p = fmaf(r, C0, C1);
        float q = fmaf(r, C2, C3);
        q = fmaf(p, r2, q);
        p = C4 * r;
        float poly = fmaf(q, r2, p);
        y[l] = fmaf(poly, scale, scale);
    }
}

DCO_EXPORT void dco_exp_u20_groups(const float *x, float *y, int64_t n) {
    int64_t i = 0;
    for (; i + 4 <= n; i += 4) exp_u20(x + i, y + i);
    if (i < n) {
        float a[4] = {0, 0, 0, 0}, b[4];
        for (int64_t j = i; j < n; j++) a[j - i] = x[j];
        exp_u20(a, b);
        for (int64_t j = i; j < n; j++) y[j] = b[j - i];
    }
}

DCO_EXPORT void dco_sleef_expf_array(const float *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = dco_sleef_expf(x[i]);
}

/* ------------------------------------------------------------------------ GEMM -- */

/* torch_blas.rs:94-133 -- the portable column-major sgemm_: for each (j, i) a sequential
 * fp32 dot product over p, then alpha*sum (+ beta*c; with beta == 0 C is not read). */
static void sgemm_portable(int ta, int tb, size_t m, size_t n, size_t k, float alpha,
                           const float *a, size_t lda, const float *b, size_t ldb, float beta,
                           float *c, size_t ldc) {
    for (size_t j = 0; j < n; j++) {
        for (size_t i = 0; i < m; i++) {
            float sum = 0.0f;
            for (size_t p = 0; p < k; p++) {
                float av = a[ta ? p + i * lda : i + p * lda];
                float bv = b[tb ? j + p * ldb : p + j * ldb];
                sum += av * bv;
            }
            float *out = c + i + j * ldc;
            *out = beta == 0.0f ? alpha * sum : alpha * sum + beta * *out;
        }
    }
}

/* torch_blas.rs:59-79 + 584-642 -- cpublas::gemm with explicit leading dimensions. */
static int gemm_raw(int ta, int tb, size_t m, size_t n, size_t k, float alpha, const float *a,
                    size_t lda, const float *b, size_t ldb, float beta, float *c, size_t ldc) {
    if (n == 1) ldc = m;
    if (ta) {
        if (m == 1) lda = k;
    } else if (k == 1) {
        lda = m;
    }
    if (tb) {
        if (k == 1) ldb = n;
    } else if (n == 1) {
        ldb = k;
    }
    const size_t imax = 2147483647u;
    size_t need_a = ta ? k : m, need_b = tb ? n : k;
    int fits = m <= imax && n <= imax && k <= imax && lda <= imax && ldb <= imax && ldc <= imax &&
               lda >= (need_a ? need_a : 1) && ldb >= (need_b ? need_b : 1) && ldc >= (m ? m : 1);
    if (!fits) return DCO_ERUNTIME;
    if (m == 0 || n == 0) return DCO_OK;
    sgemm_portable(ta, tb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc);
    return DCO_OK;
}

/* --------------------------------------------------------------- row kernels ---- */

/* torch_attention.rs:47-87 -- row *= scale in place, returns the NaN-aware row max. */
static float mul_reduce_max(float *row, size_t size, float scale) {
    size_t end_n = size / 8 * 8, end = size / 4 * 4, i = 0;
    float acc[2][4], tail[4];
    for (int h = 0; h < 2; h++)
        for (int l = 0; l < 4; l++) acc[h][l] = -INFINITY;
    for (int l = 0; l < 4; l++) tail[l] = -INFINITY;
    while (i < end_n) {
        for (int h = 0; h < 2; h++)
            for (int l = 0; l < 4; l++) {
                float x = row[i + 4 * h + l] * scale;
                row[i + 4 * h + l] = x;
                acc[h][l] = maximum(acc[h][l], x);
            }
        i += 8;
    }
    while (i < end) {
        for (int l = 0; l < 4; l++) {
            float x = row[i + l] * scale;
            row[i + l] = x;
            tail[l] = maximum(tail[l], x);
        }
        i += 4;
    }
    for (int l = 0; l < 4; l++) acc[0][l] = maximum(acc[0][l], tail[l]);
    float tmp_max = -INFINITY;
    for (; i < size; i++) {
        row[i] *= scale;
        tmp_max = std_max(tmp_max, row[i]);
    }
    float v[4];
    for (int l = 0; l < 4; l++) v[l] = maximum(acc[0][l], acc[1][l]);
    float reduced = maximum(maximum(v[0], v[2]), maximum(v[1], v[3]));
    return isnan(reduced) ? NAN : std_max(tmp_max, reduced);
}

/* torch_attention.rs:89-105 -- row = exp(row - max) in place, returns the sum. */
static float exp_reduce_sum(float *row, size_t size, float max) {
    size_t end = size / 4 * 4;
    float acc[4] = {0, 0, 0, 0};
    for (size_t i = 0; i < end; i += 4) {
        float x[4], e[4];
        for (int l = 0; l < 4; l++) x[l] = row[i + l] - max;
        exp_u20(x, e);
        for (int l = 0; l < 4; l++) {
            acc[l] = acc[l] + e[l];
            row[i + l] = e[l];
        }
    }
    float sum = (acc[0] + acc[2]) + (acc[1] + acc[3]);
    for (size_t i = end; i < size; i++) {
        float e = expf(row[i] - max);
        sum += e;
        row[i] = e;
    }
    return sum;
}

/* torch_attention.rs:130-141 -- x*scale + m: unfused in 4-lane groups, fused in the tail. */
static void scale_add_mask(float *row, const float *mask, size_t size, float scale) {
    size_t whole = size / 4 * 4;
    for (size_t i = 0; i < size; i++)
        row[i] = i < whole ? row[i] * scale + mask[i] : fmaf(row[i], scale, mask[i]);
}

/* torch_attention.rs:26-35 */
static size_t q_split(size_t q_len) { return q_len >= 768 ? 256 : q_len >= 192 ? 64 : 32; }

/* torch_attention.rs:37-40 -- computed in double, stored as float. */
static float scale_factor(size_t head_dim, int has_scale, double scale) {
    return has_scale ? (float)scale : (float)(1.0 / sqrt((double)head_dim));
}

/* --------------------------------------------------------------- threading ----- */

typedef struct {
    size_t parts;
    int threads;
    void (*fn)(void *ctx, size_t task);
    void *ctx;
    int index;
} par_arg;

static void *par_worker(void *p) {
    par_arg *a = (par_arg *)p;
    /* torch_attention.rs:113-116: task i goes to bucket i*threads/parts. */
    for (size_t i = 0; i < a->parts; i++)
        if ((int)(i * (size_t)a->threads / a->parts) == a->index) a->fn(a->ctx, i);
    return NULL;
}

/* torch_attention.rs:107-128 -- independent (batch, head) tasks over scoped threads. */
static void par_chunks(size_t parts, int threads, void (*fn)(void *, size_t), void *ctx) {
    if (parts == 0) return;
    if (threads < 1) threads = 1;
    if ((size_t)threads > parts) threads = (int)parts;
    if (threads == 1) {
        for (size_t i = 0; i < parts; i++) fn(ctx, i);
        return;
    }
    pthread_t *tid = (pthread_t *)malloc(sizeof(pthread_t) * threads);
    par_arg *args = (par_arg *)malloc(sizeof(par_arg) * threads);
    for (int t = 0; t < threads; t++) {
        args[t] = (par_arg){parts, threads, fn, ctx, t};
        if (pthread_create(&tid[t], NULL, par_worker, &args[t]) != 0) {
            par_worker(&args[t]);
            tid[t] = 0;
        }
    }
    for (int t = 0; t < threads; t++)
        if (tid[t]) pthread_join(tid[t], NULL);
    free(tid);
    free(args);
}

/* ------------------------------------------------------------------ forward ----- */

typedef struct {
    size_t batch, heads, kv_heads, q_len, kv_len, head_dim;
} dims_t;

typedef struct {
    const float *q, *k, *v, *mask;
    dims_t d;
    int causal;
    float scale;
    float *out, *lse;
    volatile int failed;
} fwd_ctx;

static void fwd_task(void *p, size_t t) {
    fwd_ctx *c = (fwd_ctx *)p;
    dims_t d = c->d;
    size_t e = d.head_dim;
    size_t qs = q_split(d.q_len);
    if (qs > d.q_len) qs = d.q_len;
    size_t kvs = KV_SPLIT < d.kv_len ? KV_SPLIT : d.kv_len;
    size_t repeat = d.heads / d.kv_heads;
    size_t b = t / d.heads, h = t % d.heads;
    size_t qb_base = t * d.q_len * e;
    size_t kv_base = (b * d.kv_heads + h / repeat) * d.kv_len * e;
    float *out = c->out + t * d.q_len * e, *lse = c->lse + t * d.q_len;
    float *qk = (float *)calloc(qs * kvs + 1, sizeof(float));
    float *dst = (float *)calloc(qs * e + 1, sizeof(float));
    float *qk_max = (float *)calloc(qs + 1, sizeof(float));
    float *qk_sum = (float *)calloc(qs + 1, sizeof(float));
    if (!qk || !dst || !qk_max || !qk_sum) {
        c->failed = DCO_ENOMEM;
        goto done;
    }
    size_t step_q = qs ? qs : 1, step_kv = kvs ? kvs : 1;
    for (size_t m = 0; m < d.q_len; m += step_q) {
        size_t qb = qs < d.q_len - m ? qs : d.q_len - m;
        for (size_t r = 0; r < qb; r++) {
            qk_max[r] = -INFINITY;
            qk_sum[r] = 0.0f;
        }
        size_t num_keys = c->causal ? (m + qb < d.kv_len ? m + qb : d.kv_len) : d.kv_len;
        for (size_t n = 0; n < num_keys; n += step_kv) {
            size_t kvb = kvs < d.kv_len - n ? kvs : d.kv_len - n;
            if (gemm_raw(1, 0, kvb, qb, e, 1.0f, c->k + kv_base + n * e, e, c->q + qb_base + m * e,
                         e, 0.0f, qk, kvb)) {
                c->failed = DCO_ERUNTIME;
                goto done;
            }
            if (c->causal && num_keys - n <= kvs) {
                for (size_t row = 0; row < qb; row++) {
                    size_t from = m + row + 1 > n ? m + row + 1 - n : 0;
                    if (from > kvb) from = kvb;
                    for (size_t i = row * kvb + from; i < (row + 1) * kvb; i++) qk[i] = -INFINITY;
                }
            }
            for (size_t row = 0; row < qb; row++) {
                float *r = qk + row * kvb;
                float tmp_max;
                if (c->mask) {
                    size_t at = (t * d.q_len + m + row) * d.kv_len + n;
                    scale_add_mask(r, c->mask + at, kvb, c->scale);
                    tmp_max = reduce_all(r, kvb, maximum);
                } else {
                    tmp_max = mul_reduce_max(r, kvb, c->scale);
                }
                tmp_max = qk_max[row] > tmp_max ? qk_max[row] : tmp_max;
                if (tmp_max == -INFINITY) {
                    for (size_t i = 0; i < kvb; i++) r[i] = 0.0f;
                    continue;
                }
                float tmp_sum = exp_reduce_sum(r, kvb, tmp_max);
                float exp_tmp = expf(qk_max[row] - tmp_max);
                qk_sum[row] = fmaf(exp_tmp, qk_sum[row], tmp_sum);
                qk_max[row] = tmp_max;
                if (n > 0)
                    for (size_t x = 0; x < e; x++) dst[row * e + x] *= exp_tmp;
            }
            if (gemm_raw(0, 0, e, qb, kvb, 1.0f, c->v + kv_base + n * e, e, qk, kvb,
                         n == 0 ? 0.0f : 1.0f, dst, e)) {
                c->failed = DCO_ERUNTIME;
                goto done;
            }
        }
        for (size_t row = 0; row < qb; row++) {
            if (qk_max[row] == -INFINITY) qk_max[row] = 0.0f;
            if (qk_sum[row] == 0.0f) qk_sum[row] = 1.0f;
            float recip = 1.0f / qk_sum[row];
            float *o = out + (m + row) * e;
            for (size_t x = 0; x < e; x++) o[x] = dst[row * e + x] * recip;
            lse[m + row] = qk_max[row] + logf(qk_sum[row]);
        }
    }
done:
    free(qk);
    free(dst);
    free(qk_max);
    free(qk_sum);
}

static int check_dims(dims_t d) {
    if (d.kv_heads == 0 || d.heads % d.kv_heads != 0) return DCO_EVALUE;
    return DCO_OK;
}

/* Forward: out (B,H,L,E) and lse (B,H,L). mask, when given, is the additive float mask
 * already broadcast to a contiguous (B,H,L,S). torch_attention.rs:146-284. */
DCO_EXPORT int dco_flash_forward(const float *q, const float *k, const float *v, const float *mask,
                                 int64_t batch, int64_t heads, int64_t kv_heads, int64_t q_len,
                                 int64_t kv_len, int64_t head_dim, int causal, int has_scale,
                                 double scale, int threads, float *out, float *lse) {
    dims_t d = {(size_t)batch, (size_t)heads, (size_t)kv_heads,
                (size_t)q_len, (size_t)kv_len, (size_t)head_dim};
    if (check_dims(d)) return DCO_EVALUE;
    fwd_ctx c = {q, k, v, mask, d, causal, scale_factor(d.head_dim, has_scale, scale), out, lse, 0};
    memset(out, 0, sizeof(float) * d.batch * d.heads * d.q_len * d.head_dim);
    memset(lse, 0, sizeof(float) * d.batch * d.heads * d.q_len);
    par_chunks(d.batch * d.heads, threads, fwd_task, &c);
    return c.failed;
}

/* Forward restricted to a subset of (batch, head) tasks: task ids in `tasks`. Used for the
 * bounded CPU-baseline sample of long sequences; tasks are independent
 * (torch_attention.rs:8), so a subset's bits equal the full run's bits for those tasks. */
typedef struct {
    fwd_ctx *c;
    const int64_t *tasks;
} sub_ctx;
static void fwd_sub_task(void *p, size_t i) {
    sub_ctx *s = (sub_ctx *)p;
    fwd_task(s->c, (size_t)s->tasks[i]);
}
DCO_EXPORT int dco_flash_forward_tasks(const float *q, const float *k, const float *v,
                                       const float *mask, int64_t batch, int64_t heads,
                                       int64_t kv_heads, int64_t q_len, int64_t kv_len,
                                       int64_t head_dim, int causal, int has_scale, double scale,
                                       int threads, const int64_t *tasks, int64_t ntasks,
                                       float *out, float *lse) {
    dims_t d = {(size_t)batch, (size_t)heads, (size_t)kv_heads,
                (size_t)q_len, (size_t)kv_len, (size_t)head_dim};
    if (check_dims(d)) return DCO_EVALUE;
    fwd_ctx c = {q, k, v, mask, d, causal, scale_factor(d.head_dim, has_scale, scale), out, lse, 0};
    sub_ctx s = {&c, tasks};
    par_chunks((size_t)ntasks, threads, fwd_sub_task, &s);
    return c.failed;
}

/* ----------------------------------------------------------------- backward ----- */

typedef struct {
    const float *g, *q, *k, *v, *o, *lse, *mask;
    dims_t d;
    int causal;
    float scale;
    float *gq, *gk, *gv;
    volatile int failed;
} bwd_ctx;

static void bwd_task(void *p, size_t t) {
    bwd_ctx *c = (bwd_ctx *)p;
    dims_t d = c->d;
    size_t e = d.head_dim;
    size_t qs = q_split(d.q_len);
    if (qs > d.q_len) qs = d.q_len;
    size_t kvs = KV_SPLIT < d.kv_len ? KV_SPLIT : d.kv_len;
    size_t repeat = d.heads / d.kv_heads;
    size_t kv_base = t * d.kv_len * e;
    float *gk = c->gk + t * d.kv_len * e, *gv = c->gv + t * d.kv_len * e;
    float *attn = (float *)calloc(qs * kvs + 1, sizeof(float));
    float *grad_attn = (float *)calloc(qs * kvs + 1, sizeof(float));
    float *dsum = (float *)calloc(qs + 1, sizeof(float));
    size_t step_q = qs ? qs : 1, step_kv = kvs ? kvs : 1;
    if (!attn || !grad_attn || !dsum) {
        c->failed = DCO_ENOMEM;
        goto done;
    }
    for (size_t r = 0; r < repeat; r++) {
        size_t j = t * repeat + r; /* (batch, head) index of this query head */
        size_t q_base = j * d.q_len * e;
        float *gq = c->gq + j * d.q_len * e;
        for (size_t m = 0; m < d.q_len; m += step_q) {
            size_t qb = qs < d.q_len - m ? qs : d.q_len - m;
            for (size_t row = 0; row < qb; row++) {
                size_t at = q_base + (m + row) * e;
                dsum[row] = reduce_all_dot(c->g + at, c->o + at, e);
            }
            size_t num_keys = c->causal ? (m + qb < d.kv_len ? m + qb : d.kv_len) : d.kv_len;
            for (size_t n = 0; n < num_keys; n += step_kv) {
                size_t kvb = kvs < d.kv_len - n ? kvs : d.kv_len - n;
                int err = gemm_raw(1, 0, kvb, qb, e, c->scale, c->k + kv_base + n * e, e,
                                   c->q + q_base + m * e, e, 0.0f, attn, kvb);
                if (err) goto fail;
                if (c->mask) {
                    for (size_t row = 0; row < qb; row++) {
                        size_t at = (j * d.q_len + m + row) * d.kv_len + n;
                        float *rr = attn + row * kvb;
                        for (size_t i = 0; i < kvb; i++) rr[i] += c->mask[at + i];
                    }
                }
                for (size_t row = 0; row < qb; row++) {
                    float norm = c->lse[j * d.q_len + m + row];
                    float *rr = attn + row * kvb;
                    for (size_t i = 0; i < kvb; i++) rr[i] = dco_sleef_expf(rr[i] - norm);
                }
                if (c->causal && num_keys - n <= kvs) {
                    for (size_t row = 0; row < qb; row++) {
                        size_t from = m + row + 1 > n ? m + row + 1 - n : 0;
                        if (from > kvb) from = kvb;
                        for (size_t i = row * kvb + from; i < (row + 1) * kvb; i++) attn[i] = 0.0f;
                    }
                }
                err = gemm_raw(0, 1, e, kvb, qb, 1.0f, c->g + q_base + m * e, e, attn, kvb, 1.0f,
                               gv + n * e, e);
                if (err) goto fail;
                err = gemm_raw(1, 0, kvb, qb, e, 1.0f, c->v + kv_base + n * e, e,
                               c->g + q_base + m * e, e, 0.0f, grad_attn, kvb);
                if (err) goto fail;
                for (size_t row = 0; row < qb; row++) {
                    float dr = dsum[row];
                    for (size_t i = row * kvb; i < (row + 1) * kvb; i++)
                        grad_attn[i] = attn[i] * (grad_attn[i] - dr);
                }
                err = gemm_raw(0, 0, e, qb, kvb, c->scale, c->k + kv_base + n * e, e, grad_attn,
                               kvb, 1.0f, gq + m * e, e);
                if (err) goto fail;
                err = gemm_raw(0, 1, e, kvb, qb, c->scale, c->q + q_base + m * e, e, grad_attn,
                               kvb, 1.0f, gk + n * e, e);
                if (err) goto fail;
            }
        }
    }
    goto done;
fail:
    c->failed = DCO_ERUNTIME;
done:
    free(attn);
    free(grad_attn);
    free(dsum);
}

/* Backward: grad_q (B,H,L,E), grad_k and grad_v (B,Hkv,S,E). torch_attention.rs:291-468. */
DCO_EXPORT int dco_flash_backward(const float *grad_out, const float *q, const float *k,
                                  const float *v, const float *out, const float *lse,
                                  const float *mask, int64_t batch, int64_t heads,
                                  int64_t kv_heads, int64_t q_len, int64_t kv_len,
                                  int64_t head_dim, int causal, int has_scale, double scale,
                                  int threads, float *gq, float *gk, float *gv) {
    dims_t d = {(size_t)batch, (size_t)heads, (size_t)kv_heads,
                (size_t)q_len, (size_t)kv_len, (size_t)head_dim};
    if (check_dims(d)) return DCO_EVALUE;
    memset(gq, 0, sizeof(float) * d.batch * d.heads * d.q_len * d.head_dim);
    memset(gk, 0, sizeof(float) * d.batch * d.kv_heads * d.kv_len * d.head_dim);
    memset(gv, 0, sizeof(float) * d.batch * d.kv_heads * d.kv_len * d.head_dim);
    bwd_ctx c = {grad_out, q, k, v, out, lse, mask, d, causal,
                 scale_factor(d.head_dim, has_scale, scale), gq, gk, gv, 0};
    par_chunks(d.batch * d.kv_heads, threads, bwd_task, &c);
    return c.failed;
}

/* Backward restricted to a subset of (batch, kv head) tasks (torch_attention.rs:313: the
 * backward's tasks are (batch, kv head) pairs); other tasks' gradients stay zero. */
typedef struct {
    bwd_ctx *c;
    const int64_t *tasks;
} bsub_ctx;
static void bwd_sub_task(void *p, size_t i) {
    bsub_ctx *s = (bsub_ctx *)p;
    bwd_task(s->c, (size_t)s->tasks[i]);
}
DCO_EXPORT int dco_flash_backward_tasks(const float *grad_out, const float *q, const float *k,
                                        const float *v, const float *out, const float *lse,
                                        const float *mask, int64_t batch, int64_t heads,
                                        int64_t kv_heads, int64_t q_len, int64_t kv_len,
                                        int64_t head_dim, int causal, int has_scale, double scale,
                                        int threads, const int64_t *tasks, int64_t ntasks,
                                        float *gq, float *gk, float *gv) {
    dims_t d = {(size_t)batch, (size_t)heads, (size_t)kv_heads,
                (size_t)q_len, (size_t)kv_len, (size_t)head_dim};
    if (check_dims(d)) return DCO_EVALUE;
    bwd_ctx c = {grad_out, q, k, v, out, lse, mask, d, causal,
                 scale_factor(d.head_dim, has_scale, scale), gq, gk, gv, 0};
    bsub_ctx s = {&c, tasks};
    par_chunks((size_t)ntasks, threads, bwd_sub_task, &s);
    return c.failed;
}

/* ----------------------------------------------------- MHA math path pieces ----- */

/* torch_softmax.rs:56-67 -- max, SLEEF exp of (x - max), times 1/sum. */
DCO_EXPORT void dco_softmax_lastdim(const float *x, int64_t rows, int64_t width, float *out) {
    for (int64_t r = 0; r < rows; r++) {
        const float *row = x + r * width;
        float *o = out + r * width;
        float max = reduce_all(row, (size_t)width, maximum);
        for (int64_t i = 0; i < width; i++) o[i] = dco_sleef_expf(row[i] - max);
        float inv = 1.0f / reduce_all(o, (size_t)width, add);
        for (int64_t i = 0; i < width; i++) o[i] = o[i] * inv;
    }
}

/* torch_softmax.rs:89-97 -- (g - sum(g*y)) * y per row. */
DCO_EXPORT void dco_softmax_backward_lastdim(const float *g, const float *y, int64_t rows,
                                             int64_t width, float *out) {
    for (int64_t r = 0; r < rows; r++) {
        const float *gr = g + r * width, *yr = y + r * width;
        float sum = reduce_all_dot(gr, yr, (size_t)width);
        for (int64_t i = 0; i < width; i++) out[r * width + i] = (gr[i] - sum) * yr[i];
    }
}

/* torch_blas.rs:404-445 -- bmm of row-major contiguous (bs,rows,k) x (bs,k,cols). For
 * k*rows*cols >= 400 each batch item is one mm, which PyTorch's CPU BLAS computes as the
 * column-major product C^T = B^T A^T with the sequential-sum portable sgemm. */
DCO_EXPORT void dco_bmm(const float *a, const float *b, int64_t bs, int64_t rows, int64_t k,
                        int64_t cols, float *out) {
    for (int64_t t = 0; t < bs; t++) {
        const float *s = a + t * rows * k, *m = b + t * k * cols;
        float *o = out + t * rows * cols;
        if (k * rows * cols < 400) {
            int64_t unfused = k > 3 ? k - k % 4 : 0;
            for (int64_t i = 0; i < rows; i++)
                for (int64_t j = 0; j < cols; j++) {
                    float acc = 0.0f;
                    for (int64_t p = 0; p < k; p++) {
                        float x = s[i * k + p], y = m[p * cols + j];
                        acc = p < unfused ? acc + x * y : fmaf(x, y, acc);
                    }
                    o[i * cols + j] = acc;
                }
        } else {
            sgemm_portable(0, 0, (size_t)cols, (size_t)rows, (size_t)k, 1.0f, m, (size_t)cols, s,
                           (size_t)k, 0.0f, o, (size_t)cols);
        }
    }
}

/* ------------------------------------------------ PyTorch's CPU generator (mt19937) -- */
/* Engine state as DenseCore keeps it (src/torch_random.rs:19-26): 624 state words, then
 * `left` and `next`. The seed and the cached normal samples are not needed by dropout. */
enum { MT_N = 624, MT_M = 397 };
#define MT_MATRIX_A 0x9908b0dfu
#define MT_UMASK 0x80000000u
#define MT_LMASK 0x7fffffffu

/* manual_seed (torch_random.rs:43-56): Knuth's multiplier 1812433253, left = 1, next = 0. */
DCO_EXPORT void dco_mt_seed(uint64_t seed, uint32_t st[MT_N + 2]) {
    st[0] = (uint32_t)seed;
    for (uint32_t j = 1; j < MT_N; j++) st[j] = 1812433253u * (st[j - 1] ^ (st[j - 1] >> 30)) + j;
    st[MT_N] = 1;     /* left */
    st[MT_N + 1] = 0; /* next */
}

static inline uint32_t mt_twist(uint32_t u, uint32_t v) {
    return (((u & MT_UMASK) | (v & MT_LMASK)) >> 1) ^ ((v & 1u) ? MT_MATRIX_A : 0u);
}

/* next_state (torch_random.rs:66-77), in place. */
static void mt_next_state(uint32_t *s) {
    int j;
    for (j = 0; j < MT_N - MT_M; j++) s[j] = s[j + MT_M] ^ mt_twist(s[j], s[j + 1]);
    for (; j < MT_N - 1; j++) s[j] = s[j + MT_M - MT_N] ^ mt_twist(s[j], s[j + 1]);
    s[MT_N - 1] = s[MT_M - 1] ^ mt_twist(s[MT_N - 1], s[0]);
}

/* random (torch_random.rs:79-91): decrement left, twist when it reaches 0, temper. */
static uint32_t mt_random(uint32_t *st) {
    if (--st[MT_N] == 0) {
        mt_next_state(st);
        st[MT_N] = MT_N;
        st[MT_N + 1] = 0;
    }
    uint32_t y = st[st[MT_N + 1]++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

DCO_EXPORT void dco_mt_random(uint32_t *st, int64_t n, uint32_t *out) {
    for (int64_t i = 0; i < n; i++) out[i] = mt_random(st);
}

/* n outputs drawn and discarded (advances the engine exactly as n random() calls). */
DCO_EXPORT void dco_mt_discard(uint32_t *st, int64_t n) {
    for (int64_t i = 0; i < n; i++) (void)mt_random(st);
}

/* bernoulli(n, p) (torch_random.rs:242-254): each draw is uniform_real_distribution<double>
 * (:106-110): random64 = (first random << 32) | second, its low 53 bits times 2^-53, then
 * fma(x, 1 - 0, 0) = x; the element is 1 when that is below p. Written as packed bits:
 * element e is bit e % 32 of word e / 32 (the caller zeroes the words). */
DCO_EXPORT void dco_mt_bernoulli_bits(uint32_t *st, int64_t n, double p, uint32_t *bits) {
    for (int64_t e = 0; e < n; e++) {
        uint64_t hi = mt_random(st), lo = mt_random(st);
        double x = (double)(((hi << 32) | lo) & ((1ull << 53) - 1)) * (1.0 / (double)(1ull << 53));
        if (fma(x, 1.0 - 0.0, 0.0) < p) bits[e >> 5] |= 1u << (e & 31);
    }
}

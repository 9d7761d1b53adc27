/* CPU restatement of the Redshift hot path in float64, in plain C.
 *
 * TEST INFRASTRUCTURE ONLY: the product library never links or calls it.
 * tests/ pin it to the numpy oracle (oracle/hotpath.py) and to the golden
 * vectors produced by the reference's own tests/cpu_reference.py, and
 * bench.py times it on the host cores as the CPU baseline of the path.
 *
 * Both functions follow the reference's scalar oracle
 * (cristianku/redshift tests/cpu_reference.py) step by step:
 *   qvo_attention  restates cpu_reference.py:55-89 (RMSNorm with weight, the
 *                  partial rotary embedding at position+t with angle
 *                  pos * 1e7^(-i/32), fp16 rounding of the appended keys and
 *                  values, scores q.k/16 over keys [0, position+t], softmax,
 *                  P.V, times sigmoid(gate));
 *   qvo_delta      restates cpu_reference.py:18-52 (causal depthwise conv over
 *                  three history rows plus the new row, SiLU, q/k L2 norms with
 *                  +1e-6 and q times 1/sqrt(dim), per value head h with key
 *                  head h % key_heads: a = exp(decay*log1p(exp(alpha+bias))),
 *                  b = sigmoid(beta), row update S = a S; S += b (v - S.k) k,
 *                  readout S.q, gated RMSNorm with silu(gate)).
 * Only the evaluation order of sums differs: the attention softmax runs over
 * blocks of keys whose (max, sum, P.V) are merged with exp(m_b - M), the
 * usual split-softmax identity; everything is float64 as in the reference.
 * Work is spread over `threads` POSIX threads (no OpenMP runtime).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define HEADS 24
#define KV_HEADS 4
#define HEAD_DIM 256
#define GROUP (HEADS / KV_HEADS)
#define KEY_BLOCK 2048

/* ------------------------------------------------------------ binary16 */
static double half_to_double(uint16_t h) {
    const int sign = h >> 15, exp = (h >> 10) & 31, man = h & 1023;
    double v;
    if (exp == 0) v = ldexp((double)man, -24);                 /* subnormal or zero */
    else if (exp == 31) v = man ? NAN : INFINITY;
    else v = ldexp((double)(man | 1024), exp - 25);
    return sign ? -v : v;
}

/* Round a double to the nearest binary16, ties to even (what Python's
 * struct.pack('<e', x) and numpy's float16 cast do). */
static uint16_t double_to_half(double x) {
    uint16_t sign = signbit(x) ? 0x8000 : 0;
    double a = fabs(x);
    if (isnan(x)) return 0x7e00;
    if (a >= 65520.0) return sign | 0x7c00;                   /* rounds to infinity */
    int e;
    frexp(a, &e);                                              /* a = f * 2^e, f in [0.5, 1) */
    int exp = e - 1;                                           /* a in [2^exp, 2^(exp+1)) */
    if (a == 0.0) return sign;
    double q;                                                  /* value in units of the last place */
    if (exp < -14) {                                           /* subnormal range: ulp 2^-24 */
        q = ldexp(a, 24);
    } else {
        q = ldexp(a, 10 - exp);                                /* in [1024, 2048) */
    }
    double r = nearbyint(q);                                   /* default rounding: ties to even */
    if (exp < -14) {
        const uint32_t m = (uint32_t)r;                        /* may round up into the normal range */
        return sign | (uint16_t)m;                             /* 1024 encodes the smallest normal */
    }
    uint32_t m = (uint32_t)r;
    int be = exp + 15;
    if (m == 2048) { m = 1024; be += 1; }
    if (be >= 31) return sign | 0x7c00;
    return sign | (uint16_t)((be << 10) | (m - 1024));
}

static double sigmoid(double x) { return 1.0 / (1.0 + exp(-x)); }
static double silu(double x) { return x * sigmoid(x); }

/* ------------------------------------------------------------ threads */
typedef void (*task_fn)(void *ctx, int index);
struct pool_arg { task_fn fn; void *ctx; int begin, end, stride; };

static void *pool_worker(void *p) {
    struct pool_arg *a = (struct pool_arg *)p;
    for (int i = a->begin; i < a->end; i += a->stride) a->fn(a->ctx, i);
    return NULL;
}

/* Run fn(ctx, i) for i in [0, n) on up to `threads` threads (round robin). */
static void parallel_for(int n, int threads, task_fn fn, void *ctx) {
    if (threads < 1) threads = 1;
    if (threads > n) threads = n;
    if (threads <= 1) {
        for (int i = 0; i < n; ++i) fn(ctx, i);
        return;
    }
    pthread_t *tid = (pthread_t *)malloc(sizeof(pthread_t) * threads);
    struct pool_arg *args = (struct pool_arg *)malloc(sizeof(struct pool_arg) * threads);
    for (int t = 0; t < threads; ++t) {
        args[t] = (struct pool_arg){fn, ctx, t, n, threads};
        if (t > 0) pthread_create(&tid[t], NULL, pool_worker, &args[t]);
    }
    pool_worker(&args[0]);
    for (int t = 1; t < threads; ++t) pthread_join(tid[t], NULL);
    free(args);
    free(tid);
}

/* ------------------------------------------------------------ attention */
/* q.k over 256 dimensions as eight interleaved partial sums (vectorisable;
 * float64 either way, so the reordering moves results by ~1e-16 relative). */
static inline double dot256(const double *a, const double *b) {
    double s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int i = 0; i < HEAD_DIM; i += 8)
        for (int u = 0; u < 8; ++u) s[u] += a[i + u] * b[i + u];
    return ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
}

/* RMSNorm with weight, then the partial rotary embedding (cpu_reference.py:62-70). */
static void prepare_row(double *out, const float *row, const float *weight, int pos, double eps) {
    double ss = 0.0;
    for (int i = 0; i < HEAD_DIM; ++i) ss += (double)row[i] * (double)row[i];
    const double inv = 1.0 / sqrt(ss / HEAD_DIM + eps);
    for (int i = 0; i < HEAD_DIM; ++i) out[i] = (double)row[i] * inv * (double)weight[i];
    for (int i = 0; i < 32; ++i) {
        const double angle = pos * pow(10000000.0, -i / 32.0);
        const double c = cos(angle), s = sin(angle);
        const double x = out[i], y = out[i + 32];
        out[i] = x * c - y * s;
        out[i + 32] = x * s + y * c;
    }
}

struct attn_ctx {
    const uint16_t *kc, *vc;
    const double *query;       /* [batch][24][256] */
    int batch, position, nblocks;
    double *part_m, *part_l, *part_o;   /* per (kv head, block): [rows], [rows], [rows][256] */
    const double *h2d;         /* binary16 -> double table */
};

static void attn_block(void *p, int task) {
    struct attn_ctx *c = (struct attn_ctx *)p;
    const int g = task / c->nblocks, blk = task % c->nblocks;
    const int rows = c->batch * GROUP, n = c->position + c->batch;
    const int k0 = blk * KEY_BLOCK, k1 = k0 + KEY_BLOCK < n ? k0 + KEY_BLOCK : n;
    double *m = c->part_m + (size_t)task * rows, *l = c->part_l + (size_t)task * rows;
    double *o = c->part_o + (size_t)task * rows * HEAD_DIM;
    double *s = (double *)malloc(sizeof(double) * rows * KEY_BLOCK);
    double kv[HEAD_DIM];
    for (int r = 0; r < rows; ++r) { m[r] = -INFINITY; l[r] = 0.0; }
    memset(o, 0, sizeof(double) * rows * HEAD_DIM);
    for (int p = k0; p < k1; ++p) {
        const uint16_t *kr = c->kc + ((size_t)p * KV_HEADS + g) * HEAD_DIM;
        for (int i = 0; i < HEAD_DIM; ++i) kv[i] = c->h2d[kr[i]];
        for (int r = 0; r < rows; ++r) {
            const int t = r / GROUP, h = g * GROUP + r % GROUP;
            double acc = -INFINITY;
            if (p <= c->position + t) {                        /* causal: keys [0, position+t] */
                const double *q = c->query + ((size_t)t * HEADS + h) * HEAD_DIM;
                acc = dot256(q, kv) / 16.0;
            }
            s[(size_t)r * KEY_BLOCK + (p - k0)] = acc;
            if (acc > m[r]) m[r] = acc;
        }
    }
    for (int r = 0; r < rows; ++r)
        for (int p = k0; p < k1; ++p) {
            double *x = &s[(size_t)r * KEY_BLOCK + (p - k0)];
            *x = m[r] == -INFINITY ? 0.0 : exp(*x - m[r]);
            l[r] += *x;
        }
    for (int p = k0; p < k1; ++p) {
        const uint16_t *vr = c->vc + ((size_t)p * KV_HEADS + g) * HEAD_DIM;
        for (int i = 0; i < HEAD_DIM; ++i) kv[i] = c->h2d[vr[i]];
        for (int r = 0; r < rows; ++r) {
            const double w = s[(size_t)r * KEY_BLOCK + (p - k0)];
            if (w == 0.0) continue;
            double *orow = o + (size_t)r * HEAD_DIM;
            for (int i = 0; i < HEAD_DIM; ++i) orow[i] += w * kv[i];
        }
    }
    free(s);
}

static double *g_h2d = NULL;
static pthread_once_t g_h2d_once = PTHREAD_ONCE_INIT;
static void build_h2d(void) {
    g_h2d = (double *)malloc(sizeof(double) * 65536);
    for (int i = 0; i < 65536; ++i) g_h2d[i] = half_to_double((uint16_t)i);
}

/* One attention layer: out [batch][24][256] (float64), key_cache / value_cache
 * binary16 bits [position+batch][4][256] (rows [0, position) read, the batch's
 * rows written).  Returns 0, or -1 on invalid arguments / allocation failure. */
int qvo_attention(double *out, uint16_t *key_cache, uint16_t *value_cache, const float *q_gate, const float *key,
                  const float *value, const float *q_norm, const float *k_norm, int batch, int position,
                  double epsilon, int threads) {
    if (batch < 1 || position < 0 || !out || !key_cache || !value_cache || !q_gate || !key || !value || !q_norm ||
        !k_norm)
        return -1;
    pthread_once(&g_h2d_once, build_h2d);
    double row[HEAD_DIM];
    for (int t = 0; t < batch; ++t)                            /* cpu_reference.py:73-76 */
        for (int h = 0; h < KV_HEADS; ++h) {
            const size_t off = ((size_t)t * KV_HEADS + h) * HEAD_DIM;
            const size_t dst = ((size_t)(position + t) * KV_HEADS + h) * HEAD_DIM;
            prepare_row(row, key + off, k_norm, position + t, epsilon);
            for (int i = 0; i < HEAD_DIM; ++i) {
                key_cache[dst + i] = double_to_half(row[i]);
                value_cache[dst + i] = double_to_half((double)value[off + i]);
            }
        }
    double *query = (double *)malloc(sizeof(double) * batch * HEADS * HEAD_DIM);
    if (!query) return -1;
    for (int t = 0; t < batch; ++t)                            /* cpu_reference.py:78-79 */
        for (int h = 0; h < HEADS; ++h)
            prepare_row(query + ((size_t)t * HEADS + h) * HEAD_DIM, q_gate + ((size_t)t * HEADS + h) * 2 * HEAD_DIM,
                        q_norm, position + t, epsilon);
    const int n = position + batch, rows = batch * GROUP;
    const int nblocks = (n + KEY_BLOCK - 1) / KEY_BLOCK, tasks = KV_HEADS * nblocks;
    struct attn_ctx c = {key_cache, value_cache, query, batch, position, nblocks, NULL, NULL, NULL, g_h2d};
    c.part_m = (double *)malloc(sizeof(double) * tasks * rows);
    c.part_l = (double *)malloc(sizeof(double) * tasks * rows);
    c.part_o = (double *)malloc(sizeof(double) * (size_t)tasks * rows * HEAD_DIM);
    if (!c.part_m || !c.part_l || !c.part_o) {
        free(c.part_m); free(c.part_l); free(c.part_o); free(query);
        return -1;
    }
    parallel_for(tasks, threads, attn_block, &c);
    for (int g = 0; g < KV_HEADS; ++g)                        /* merge the blocks: cpu_reference.py:83-88 */
        for (int r = 0; r < rows; ++r) {
            const int t = r / GROUP, h = g * GROUP + r % GROUP;
            double M = -INFINITY;
            for (int b = 0; b < nblocks; ++b) {
                const double mb = c.part_m[((size_t)g * nblocks + b) * rows + r];
                if (mb > M) M = mb;
            }
            double total = 0.0, acc[HEAD_DIM];
            memset(acc, 0, sizeof(acc));
            for (int b = 0; b < nblocks; ++b) {
                const size_t task = (size_t)g * nblocks + b;
                const double mb = c.part_m[task * rows + r];
                if (mb == -INFINITY) continue;
                const double w = exp(mb - M);
                total += w * c.part_l[task * rows + r];
                const double *ob = c.part_o + (task * rows + r) * HEAD_DIM;
                for (int i = 0; i < HEAD_DIM; ++i) acc[i] += w * ob[i];
            }
            const float *gate = q_gate + ((size_t)t * HEADS + h) * 2 * HEAD_DIM + HEAD_DIM;
            double *o = out + ((size_t)t * HEADS + h) * HEAD_DIM;
            for (int i = 0; i < HEAD_DIM; ++i) o[i] = acc[i] / total * sigmoid((double)gate[i]);
        }
    free(c.part_m); free(c.part_l); free(c.part_o); free(query);
    return 0;
}

/* ------------------------------------------------------------ gated DeltaNet */
struct delta_ctx {
    double *state;              /* [Hv][dim][dim] */
    const double *filtered;     /* [batch][C]: conv + SiLU outputs */
    const double *qn, *kn;      /* [batch][Hk][dim] normalised q (times 1/sqrt(dim)) and k */
    const float *gate, *alpha, *beta, *decay, *bias, *norm;
    double *out;                /* [batch][Hv][dim] */
    int batch, key_heads, value_heads, dim;
    double eps;
};

static void delta_head(void *p, int h) {
    struct delta_ctx *c = (struct delta_ctx *)p;
    const int dim = c->dim, Hk = c->key_heads, Hv = c->value_heads;
    const int C = (2 * Hk + Hv) * dim;
    double *result = (double *)malloc(sizeof(double) * dim);
    double *S = c->state + (size_t)h * dim * dim;
    for (int t = 0; t < c->batch; ++t) {                       /* cpu_reference.py:35-51 */
        const double *q = c->qn + ((size_t)t * Hk + h % Hk) * dim, *k = c->kn + ((size_t)t * Hk + h % Hk) * dim;
        const int index = t * Hv + h;
        const double a = exp((double)c->decay[h] * log1p(exp((double)c->alpha[index] + (double)c->bias[h])));
        const double b = sigmoid((double)c->beta[index]);
        for (int v = 0; v < dim; ++v) {
            double *row = S + (size_t)v * dim;
            for (int i = 0; i < dim; ++i) row[i] *= a;
            const double target = c->filtered[(size_t)t * C + 2 * Hk * dim + h * dim + v];
            double dot = 0.0;
            for (int i = 0; i < dim; ++i) dot += row[i] * k[i];
            const double residual = b * (target - dot);
            double r = 0.0;
            for (int i = 0; i < dim; ++i) {
                row[i] += residual * k[i];
                r += row[i] * q[i];
            }
            result[v] = r;
        }
        double ss = 0.0;
        for (int v = 0; v < dim; ++v) ss += result[v] * result[v];
        const double scale = 1.0 / sqrt(ss / dim + c->eps);
        const size_t offset = ((size_t)t * Hv + h) * dim;
        for (int i = 0; i < dim; ++i)
            c->out[offset + i] = result[i] * scale * (double)c->norm[i] * silu((double)c->gate[offset + i]);
    }
    free(result);
}

/* One gated-DeltaNet layer over `batch` tokens: out [batch][Hv][dim], state
 * [Hv][dim][dim] and history [3][C] (in/out) in float64; inputs as the
 * reference ABI passes them (float32).  With `round_filtered` the conv + SiLU
 * outputs are rounded to binary16 before anything else uses them (a model of
 * a kernel that takes them as fp16 operands; the reference does not round).
 * Returns 0, or -1 on invalid arguments. */
int qvo_delta(double *out, double *state, double *history, const float *qkv, const float *gate, const float *alpha,
              const float *beta, const float *conv, const float *decay, const float *bias, const float *norm,
              int batch, int key_heads, int value_heads, int dim, double epsilon, int threads, int round_filtered) {
    if (batch < 1 || key_heads < 1 || value_heads < key_heads || value_heads % key_heads || dim < 1 || !out || !state ||
        !history || !qkv || !gate || !alpha || !beta || !conv || !decay || !bias || !norm)
        return -1;
    const int C = (2 * key_heads + value_heads) * dim;
    double *filtered = (double *)malloc(sizeof(double) * batch * C);
    double *qn = (double *)malloc(sizeof(double) * batch * key_heads * dim);
    double *kn = (double *)malloc(sizeof(double) * batch * key_heads * dim);
    if (!filtered || !qn || !kn) { free(filtered); free(qn); free(kn); return -1; }
    for (int t = 0; t < batch; ++t) {                          /* cpu_reference.py:24-34 */
        const float *raw = qkv + (size_t)t * C;
        double *f = filtered + (size_t)t * C;
        for (int ch = 0; ch < C; ++ch) {
            double acc = 0.0;
            for (int j = 0; j < 3; ++j) acc += (double)conv[4 * ch + j] * history[(size_t)j * C + ch];
            f[ch] = silu(acc + (double)conv[4 * ch + 3] * (double)raw[ch]);
            if (round_filtered) f[ch] = half_to_double(double_to_half((double)(float)f[ch]));
        }
        memmove(history, history + C, sizeof(double) * 2 * C);   /* history = history[C:] + raw */
        for (int ch = 0; ch < C; ++ch) history[2 * (size_t)C + ch] = (double)raw[ch];
        for (int h = 0; h < key_heads; ++h) {
            const double *q = f + (size_t)h * dim, *k = f + (size_t)(key_heads + h) * dim;
            double sq = 0.0, sk = 0.0;
            for (int i = 0; i < dim; ++i) { sq += q[i] * q[i]; sk += k[i] * k[i]; }
            const double iq = sqrt(sq + 1e-6), ik = sqrt(sk + 1e-6), rd = sqrt((double)dim);
            for (int i = 0; i < dim; ++i) {
                qn[((size_t)t * key_heads + h) * dim + i] = q[i] / iq / rd;
                kn[((size_t)t * key_heads + h) * dim + i] = k[i] / ik;
            }
        }
    }
    struct delta_ctx c = {state, filtered, qn, kn, gate, alpha, beta, decay, bias, norm, out,
                          batch, key_heads, value_heads, dim, epsilon};
    parallel_for(value_heads, threads, delta_head, &c);
    free(filtered); free(qn); free(kn);
    return 0;
}

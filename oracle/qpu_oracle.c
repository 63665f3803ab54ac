/*
 * qpu_oracle.c - CPU restatement of the PIton reference's arithmetic for the
 * B200 hot path.  TEST INFRASTRUCTURE ONLY: the parity tests, smoke() and the
 * CPU-baseline leg of bench.py call it as the checker; the B200 product path
 * never links or calls it.
 *
 * What it restates (file:line of the reference, foxboxxx/PIton):
 *   - the VideoCore IV float ALU model of the strict emulator,
 *     piton/qpu/emulator.py:137-212 (round-toward-zero, denormals as +0,
 *     NaN read as inf, 0*inf = +0, inf + -inf = second operand, fmax/fmin on
 *     sign-magnitude keys, ftoi truncation);
 *   - the compiler's ALU-only math, piton/backend/lower.py:633-667 (Newton
 *     reciprocal from seed 0x7EF311C3), :669-694 (fdiv), :2716-2797 (exp/exp2:
 *     clamp, n*ln2 reduction, degree-6 polynomial, exponent construction);
 *   - tl.dot as a sequential-k round-toward-zero multiply then add,
 *     lower.py:3761-3878;
 *   - 16-lane butterfly reductions, lower.py:4043-4064 (rotation = np.roll,
 *     emulator.py:965-967);
 *   - the operator programs: add_kernel examples/kernels.py:6-15, matmul_kernel
 *     :18-57, softmax_kernel :60-76, dense_layer_kernel examples/nn_kernels.py:23-74,
 *     attn_fwd_kernel / _attn_fwd_inner examples/attention.py:33-113.
 *
 * Pinned against golden outputs of the reference emulator run in a container
 * holding the reference (tests/golden/make_golden.py): add, matmul and dense
 * match bit for bit; softmax and attention within stated tolerances where
 * the emulator's reduction order is a compiler decision.
 */
#define _GNU_SOURCE
#include <fenv.h>
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#pragma STDC FENV_ACCESS ON

typedef union {
    float f;
    uint32_t u;
} fu;

static inline uint32_t bits(float x) { fu v; v.f = x; return v.u; }
static inline float fbits(uint32_t u) { fu v; v.u = u; return v.f; }

#define INF_BITS 0x7F800000u

/* operand as the float ALUs read it (emulator.py:170-175) */
static inline float qin(float x) {
    uint32_t u = bits(x), e = (u >> 23) & 0xFF;
    if (e == 0) return 0.0f;
    if (e == 255) return fbits((u & 0x80000000u) | INF_BITS);
    return x;
}

/* result rules (emulator.py:153-167): truncation is done by the FPU in
   round-toward-zero mode; |r| < 2^-126 -> +0; exact >= 2^128 -> inf */
static inline float qout(float r, double exact) {
    if (fabsf(r) < 1.17549435e-38f) return 0.0f;
    if (fabs(exact) >= 3.4028236692093846e38) return copysignf(INFINITY, (float)exact);
    return r;
}

float oracle_qpu_fadd(float a, float b) {
    float fa = qin(a), fb = qin(b);
    if (isinf(fb)) return fb;
    if (isinf(fa)) return fa;
    volatile float r = fa + fb; /* FE_TOWARDZERO is set by every entry point */
    /* the double sum is exact whenever it can reach 2^128 (exponents within 29) */
    return qout(r, (double)fa + (double)fb);
}

float oracle_qpu_fsub(float a, float b) { return oracle_qpu_fadd(a, fbits(bits(b) ^ 0x80000000u)); }

float oracle_qpu_fmul(float a, float b) {
    float fa = qin(a), fb = qin(b);
    if ((fa == 0.0f && isinf(fb)) || (isinf(fa) && fb == 0.0f)) return 0.0f;
    volatile float r = fa * fb;
    return qout(r, (double)fa * (double)fb); /* the double product of two floats is exact */
}

/* fmin/fmax ordering key (emulator.py:201-206) */
static inline int64_t fkey(float x) {
    uint32_t u = bits(x);
    int64_t m = u & 0x7FFFFFFF;
    return ((u >> 31) && ((u >> 23) & 0xFF)) ? -m : m;
}
float oracle_qpu_fmax(float a, float b) { return fkey(a) > fkey(b) ? a : b; }
float oracle_qpu_fmin(float a, float b) { return fkey(a) <= fkey(b) ? a : b; }

/* ftoi: truncate, low 32 bits; zero/denormal exponent and |x| >= 2^55 give 0 (emulator.py:208-212) */
static inline int32_t qftoi(float a) {
    uint32_t e = (bits(a) >> 23) & 0xFF;
    if (e == 0 || e >= 127 + 55) return 0;
    return (int32_t)(uint32_t)(uint64_t)(int64_t)truncf(a);
}
/* itof: int32 -> float, rounded toward zero (FE_TOWARDZERO is active) */
static inline float qitof(int32_t n) { volatile float f = (float)n; return qout(f, (double)n); }

static inline int is_nan_bits(float x) { return (bits(x) & 0x7FFFFFFFu) > INF_BITS; }

/* exp / exp2, lower.py:2716-2797 */
float oracle_qpu_exp(float x, int base2) {
    float xc = oracle_qpu_fmin(x, base2 ? 128.0f : 89.0f);
    xc = oracle_qpu_fmax(xc, base2 ? -150.0f : -104.0f);
    /* float32 constants (round-to-nearest from the decimal literals of lower.py),
       given as bits so that no conversion runs under the round-toward-zero mode */
    const float LOG2E = fbits(0x3fb8aa3bu), LN2 = fbits(0x3f317218u), LN2_HI = fbits(0x3f317200u),
                LN2_LO = fbits(0x35bfbe8eu);
    static const uint32_t cs[5] = {0x3c088889u, 0x3d2aaaabu, 0x3e2aaaabu, 0x3f000000u, 0x3f800000u};
    float y = base2 ? xc : oracle_qpu_fmul(xc, LOG2E);
    float half = fbits((bits(y) & 0x80000000u) | 0x3F000000u);
    float t = oracle_qpu_fadd(y, half);
    int32_t n = qftoi(t);
    float nf = qitof(n);
    float r;
    if (base2) {
        r = oracle_qpu_fsub(xc, nf);
        r = oracle_qpu_fmul(r, LN2);
    } else {
        float t1 = oracle_qpu_fmul(nf, LN2_HI);
        float t2 = oracle_qpu_fsub(xc, t1);
        t1 = oracle_qpu_fmul(nf, LN2_LO);
        r = oracle_qpu_fsub(t2, t1);
    }
    float p = oracle_qpu_fmul(r, fbits(0x3ab60b61u));
    for (int i = 0; i < 5; ++i) {
        float q = oracle_qpu_fadd(p, fbits(cs[i]));
        p = oracle_qpu_fmul(q, r);
    }
    float q = oracle_qpu_fadd(p, 1.0f);
    int32_t nc = n < -127 ? -127 : (n > 127 ? 127 : n);
    uint32_t c = (uint32_t)(n - nc) << 23;
    float q2 = fbits(bits(q) + c);
    float scale = fbits((uint32_t)(nc + 127) << 23);
    float d = oracle_qpu_fmul(q2, scale);
    if (base2) {
        if (!(bits(oracle_qpu_fsub(x, 128.0f)) >> 31)) d = fbits(INF_BITS);
    } else {
        if (bits(oracle_qpu_fsub(fbits(0x42B17217u), x)) >> 31) d = fbits(INF_BITS);
    }
    if (is_nan_bits(x)) d = x;
    return d;
}

/* Newton reciprocal, lower.py:633-667 */
float oracle_qpu_recip(float b) {
    float r = fbits(0x7EF311C3u - bits(b));
    for (int k = 0; k < 3; ++k) {
        float t = oracle_qpu_fmul(b, r);
        float e = oracle_qpu_fsub(2.0f, t);
        r = oracle_qpu_fmul(r, e);
    }
    uint32_t eb = bits(b) & 0x7F800000u, sg = bits(b) & 0x80000000u;
    if ((int32_t)(eb - 0x7E800000u) >= 0) r = fbits(sg);
    if (eb == 0) r = fbits(sg | INF_BITS);
    if (is_nan_bits(b)) r = b;
    return r;
}

/* a / b, lower.py:669-694 */
float oracle_qpu_fdiv(float a, float b) {
    float d = oracle_qpu_fmul(a, oracle_qpu_recip(b));
    uint32_t ma = bits(a) & 0x7FFFFFFFu, mb = bits(b) & 0x7FFFFFFFu;
    uint32_t mx = ma > mb ? ma : mb;
    if ((int32_t)(mx - 0x7F800001u) >= 0) d = fbits(0x7FC00000u);
    if ((int32_t)((ma | mb) - 0x00800000u) < 0) d = fbits(0x7FC00000u);
    if ((int32_t)((ma & mb) - 0x7F800000u) >= 0) d = fbits(0x7FC00000u);
    return d;
}

/* tl.sum over one row of `n` values laid out 16 to a vector register:
   lanes accumulate the registers in order, then the butterfly of
   lower.py:4043-4064 (n[i] = src[i] + src[i - s] for s = 8, 4, 2, 1), lane 0 */
static float lane_sum(const float *v, int n) {
    float lane[16];
    for (int l = 0; l < 16; ++l) lane[l] = l < n ? v[l] : 0.0f;
    for (int r = 16; r < n; r += 16)
        for (int l = 0; l < 16 && r + l < n; ++l) lane[l] = oracle_qpu_fadd(lane[l], v[r + l]);
    for (int s = 8; s >= 1; s >>= 1) {
        float nx[16];
        for (int i = 0; i < 16; ++i) nx[i] = oracle_qpu_fadd(lane[i], lane[(i - s + 16) % 16]);
        memcpy(lane, nx, sizeof lane);
    }
    return lane[0];
}

/* ------------------------------------------------------------------ operators */

void oracle_add(const float *x, const float *y, float *out, int64_t n) {
    int old = fegetround();
    fesetround(FE_TOWARDZERO);
    for (int64_t i = 0; i < n; ++i) out[i] = oracle_qpu_fadd(x[i], y[i]);
    fesetround(old);
}

typedef struct {
    const float *a, *b;
    float *c;
    int64_t M, N, K, sam, sak, sbk, sbn, scm, scn, m0, m1;
    const float *bias;
    int relu;
} mm_job;

/* C[m, n] = sum over k in order of RTZ(a*b) with RTZ adds, from +0 (lower.py:3761-3878) */
static void *mm_worker(void *p) {
    mm_job *j = (mm_job *)p;
    fesetround(FE_TOWARDZERO);
    float *acc = (float *)malloc(sizeof(float) * (size_t)(j->N > 0 ? j->N : 1));
    for (int64_t m = j->m0; m < j->m1; ++m) {
        for (int64_t n = 0; n < j->N; ++n) acc[n] = 0.0f;
        for (int64_t k = 0; k < j->K; ++k) {
            float av = j->a[m * j->sam + k * j->sak];
            const float *brow = j->b + k * j->sbk;
            for (int64_t n = 0; n < j->N; ++n) acc[n] = oracle_qpu_fadd(acc[n], oracle_qpu_fmul(av, brow[n * j->sbn]));
        }
        for (int64_t n = 0; n < j->N; ++n) {
            float v = acc[n];
            if (j->bias) v = oracle_qpu_fadd(v, j->bias[n]);
            if (j->relu) v = oracle_qpu_fmax(v, 0.0f);
            j->c[m * j->scm + n * j->scn] = v;
        }
    }
    free(acc);
    return NULL;
}

static void run_mm(mm_job base, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if (nthreads > base.M) nthreads = base.M > 0 ? (int)base.M : 1;
    pthread_t th[256];
    mm_job jobs[256];
    int64_t per = (base.M + nthreads - 1) / nthreads;
    for (int t = 0; t < nthreads; ++t) {
        jobs[t] = base;
        jobs[t].m0 = t * per < base.M ? t * per : base.M;
        jobs[t].m1 = (t + 1) * per < base.M ? (t + 1) * per : base.M;
        if (nthreads > 1) pthread_create(&th[t], NULL, mm_worker, &jobs[t]);
    }
    if (nthreads == 1) mm_worker(&jobs[0]);
    else
        for (int t = 0; t < nthreads; ++t) pthread_join(th[t], NULL);
}

/* matmul_kernel with a covering grid (every C element written); rows m0..m1
   only when m1 > 0 (bounded samples for timing) */
void oracle_matmul(const float *a, const float *b, float *c, int64_t M, int64_t N, int64_t K, int64_t sam,
                   int64_t sak, int64_t sbk, int64_t sbn, int64_t scm, int64_t scn, int nthreads) {
    int old = fegetround();
    mm_job j = {a, b, c, M, N, K, sam, sak, sbk, sbn, scm, scn, 0, M, NULL, 0};
    run_mm(j, nthreads);
    fesetround(old);
}

/* dense_layer_kernel: X[M,K] W[K,N] contiguous, then + bias (RTZ) and ReLU (fmax) */
void oracle_dense(const float *x, const float *w, const float *bias, float *y, int64_t M, int64_t N, int64_t K,
                  int add_bias, int relu, int nthreads) {
    int old = fegetround();
    mm_job j = {x, w, y, M, N, K, K, 1, N, 1, N, 1, 0, M, add_bias ? bias : NULL, relu};
    run_mm(j, nthreads);
    fesetround(old);
}

/* softmax_kernel row: masked columns read -inf (kernels.py:60-76); BLOCK
   columns laid out 16 per register; max by fmax, exp, sum, division */
void oracle_softmax(const float *in, float *out, int64_t rows, int64_t n_cols, int64_t block, int64_t sin,
                    int64_t sout) {
    int old = fegetround();
    fesetround(FE_TOWARDZERO);
    int64_t n = n_cols < block ? n_cols : block;
    float *e = (float *)malloc(sizeof(float) * (size_t)(block > 0 ? block : 1));
    for (int64_t r = 0; r < rows; ++r) {
        const float *x = in + r * sin;
        float m = -INFINITY;
        for (int64_t j = 0; j < block; ++j) m = oracle_qpu_fmax(m, j < n ? x[j] : -INFINITY);
        for (int64_t j = 0; j < block; ++j) e[j] = oracle_qpu_exp(oracle_qpu_fsub(j < n ? x[j] : -INFINITY, m), 0);
        float s = lane_sum(e, (int)block);
        for (int64_t j = 0; j < n; ++j) out[r * sout + j] = oracle_qpu_fdiv(e[j], s);
    }
    free(e);
    fesetround(old);
}

typedef struct {
    const float *q, *k, *v;
    int64_t skn, skk, svn, n_ctx, d, bm, bn;
    float qk_scale;
    float *qrow;   /* [bm][d] */
    float *acc;    /* [bm][d] */
    float *m_i, *l_i;
    float *qk;     /* [bm][bn] */
    int64_t start_m;
} attn_state;

/* _attn_fwd_inner (attention.py:37-63) over key blocks [lo, hi) */
static void attn_inner(attn_state *s, int64_t lo, int64_t hi, int mask_keys, int causal_mask) {
    int64_t bm = s->bm, bn = s->bn, d = s->d;
    for (int64_t start_n = lo; start_n < hi; start_n += bn) {
        for (int64_t i = 0; i < bm; ++i) {
            int64_t row = s->start_m * bm + i;
            float mx = -INFINITY;
            for (int64_t j = 0; j < bn; ++j) {
                int64_t col = start_n + j;
                float acc = 0.0f;
                int valid = !mask_keys || col < s->n_ctx;
                for (int64_t t = 0; t < d; ++t) {
                    float kv = valid ? s->k[col * s->skn + t * s->skk] : 0.0f;
                    acc = oracle_qpu_fadd(acc, oracle_qpu_fmul(s->qrow[i * d + t], kv));
                }
                float v = oracle_qpu_fmul(acc, s->qk_scale);
                if (mask_keys && !(col < s->n_ctx)) v = -INFINITY;
                if (causal_mask && !(row >= col)) v = -INFINITY;
                s->qk[i * bn + j] = v;
                mx = j == 0 ? v : oracle_qpu_fmax(mx, v);
            }
            float m_ij = oracle_qpu_fmax(s->m_i[i], mx);
            for (int64_t j = 0; j < bn; ++j) s->qk[i * bn + j] = oracle_qpu_exp(oracle_qpu_fsub(s->qk[i * bn + j], m_ij), 1);
            float alpha = oracle_qpu_exp(oracle_qpu_fsub(s->m_i[i], m_ij), 1);
            s->l_i[i] = oracle_qpu_fadd(oracle_qpu_fmul(s->l_i[i], alpha), lane_sum(s->qk + i * bn, (int)bn));
            for (int64_t t = 0; t < d; ++t) {
                float a = oracle_qpu_fmul(s->acc[i * d + t], alpha);
                for (int64_t j = 0; j < bn; ++j) {
                    int64_t col = start_n + j;
                    float vv = (!mask_keys || col < s->n_ctx) ? s->v[col * s->svn + t] : 0.0f;
                    a = oracle_qpu_fadd(a, oracle_qpu_fmul(s->qk[i * bn + j], vv));
                }
                s->acc[i * d + t] = a;
            }
            s->m_i[i] = m_ij;
        }
    }
}

/* attn_fwd_kernel (attention.py:75-113) for heads [0, heads) and query blocks
   [0, cdiv(n_ctx, bm)); rows >= n_ctx are not written */
void oracle_attention(const float *q, const float *k, const float *v, float *o, int64_t heads, int64_t n_ctx,
                      int64_t d, int64_t sqh, int64_t sqm, int64_t skh, int64_t skn, int64_t skk, int64_t svh,
                      int64_t svn, int64_t soh, int64_t som, float sm_scale, int causal, int even_n, int64_t bm,
                      int64_t bn) {
    int old = fegetround();
    fesetround(FE_TOWARDZERO);
    attn_state s;
    s.skn = skn; s.skk = skk; s.svn = svn; s.n_ctx = n_ctx; s.d = d; s.bm = bm; s.bn = bn;
    s.qk_scale = oracle_qpu_fmul(sm_scale, fbits(0x3fb8aa3bu)); /* sm_scale * 1.44269504 */
    s.qrow = (float *)malloc(sizeof(float) * bm * d);
    s.acc = (float *)malloc(sizeof(float) * bm * d);
    s.m_i = (float *)malloc(sizeof(float) * bm);
    s.l_i = (float *)malloc(sizeof(float) * bm);
    s.qk = (float *)malloc(sizeof(float) * bm * bn);
    for (int64_t h = 0; h < heads; ++h) {
        s.q = q + h * sqh;
        s.k = k + h * skh;
        s.v = v + h * svh;
        for (int64_t sm = 0; sm * bm < n_ctx; ++sm) {
            s.start_m = sm;
            for (int64_t i = 0; i < bm; ++i) {
                int64_t row = sm * bm + i;
                for (int64_t t = 0; t < d; ++t) {
                    s.qrow[i * d + t] = row < n_ctx ? s.q[row * sqm + t] : 0.0f;
                    s.acc[i * d + t] = 0.0f;
                }
                s.m_i[i] = -INFINITY;
                s.l_i[i] = 0.0f;
            }
            if (causal) {
                int64_t lo = (sm * bm) / bn * bn;
                attn_inner(&s, 0, lo, 0, 0);
                int64_t hi = (sm + 1) * bm < n_ctx ? (sm + 1) * bm : n_ctx;
                attn_inner(&s, lo, hi, !even_n, 1);
            } else {
                int64_t n_full = n_ctx / bn * bn;
                attn_inner(&s, 0, n_full, 0, 0);
                if (!even_n) attn_inner(&s, n_full, n_ctx, 1, 0);
            }
            for (int64_t i = 0; i < bm; ++i) {
                int64_t row = sm * bm + i;
                if (row >= n_ctx) continue;
                for (int64_t t = 0; t < d; ++t) o[h * soh + row * som + t] = oracle_qpu_fdiv(s.acc[i * d + t], s.l_i[i]);
            }
        }
    }
    free(s.qrow); free(s.acc); free(s.m_i); free(s.l_i); free(s.qk);
    fesetround(old);
}

/* element-wise helpers exported for unit tests (rounding mode set around them) */
void oracle_map_fadd(const float *a, const float *b, float *out, int64_t n) { oracle_add(a, b, out, n); }
void oracle_map_fmul(const float *a, const float *b, float *out, int64_t n) {
    int old = fegetround();
    fesetround(FE_TOWARDZERO);
    for (int64_t i = 0; i < n; ++i) out[i] = oracle_qpu_fmul(a[i], b[i]);
    fesetround(old);
}
void oracle_map_exp(const float *x, float *out, int64_t n, int base2) {
    int old = fegetround();
    fesetround(FE_TOWARDZERO);
    for (int64_t i = 0; i < n; ++i) out[i] = oracle_qpu_exp(x[i], base2);
    fesetround(old);
}
void oracle_map_fdiv(const float *a, const float *b, float *out, int64_t n) {
    int old = fegetround();
    fesetround(FE_TOWARDZERO);
    for (int64_t i = 0; i < n; ++i) out[i] = oracle_qpu_fdiv(a[i], b[i]);
    fesetround(old);
}

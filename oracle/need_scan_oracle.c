/*
 * need_scan_oracle.c -- CPU restatement of NEED's recurrent-scan path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA kernels in
 * need_b200/csrc: only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg load it.  The product path never links or calls it.
 *
 * Parity is pinned: tests/test_oracle_golden.py checks every function here
 * against fixtures that tests/golden/make_golden.py produced by running the
 * reference's own Python functions (need_kernels.py, need_core.py).
 *
 * What is restated (reference file:line):
 *   ora_affine_scan      need_kernels.py:177-226  _chunked_affine_recurrence_scan
 *                        (== need_core.py:1419-1461 affine_recurrence_scan_torch):
 *                        per 64-token chunk, a Hillis-Steele prefix composition of
 *                        the affine maps (a, b): s -> a*s + b, combined as
 *                        (a_cur*a_prev, b_cur + a_cur*b_prev), then the chunk's
 *                        outputs b_pref + a_pref*state and state := last output.
 *                        Every fp32 product and sum is rounded separately, in the
 *                        same order as the torch ops (no fused multiply-add).
 *   ora_gated_prep       the gate arithmetic that feeds the scan in
 *                        need_kernels.py:330-336 / need_core.py:1630-1636, in the
 *                        sigmoid-decay form: decay = sigmoid(z), update =
 *                        (1 - decay) * (sigmoid(g) * x), each op rounded to the
 *                        storage dtype when that dtype is bf16 (torch computes a
 *                        bf16 op in fp32 and rounds the result).
 *   ora_ssd_prep /       need_kernels.py:330-339 (ssd_scan, torch path).
 *   ora_ssd_epilogue
 *   ora_assoc_memory     need_core.py:1960-2001 (HierarchicalMemory's linear
 *                        associative memory, the matrix-state recurrence).
 *   ora_assoc_step       need_core.py:2067-2080 (its one-token streaming step).
 *   ora_rms_norm         need_kernels.py:99-107 (rms_norm's GPU kernel), the SSD
 *                        block's out_norm after ssd_scan (need_core.py:1643).
 *   ora_stream_step      need_core.py:6420-6428 (_stream_retention_step) and
 *                        :1674-1685 (StructuredDualRetention.stream_step): one
 *                        token, state kept in the model dtype.
 *   ora_conv_step        need_core.py:6395-6409 (_stream_depthwise_conv1d_step)
 *                        and the SiLU of :6414: the SSD block's causal depthwise
 *                        conv for one token from its history, in the model dtype.
 *
 * Extensions with no reference counterpart, defined by reduction to the above:
 *   resets   : decay[t] := 0 at a segment start (the update is unchanged);
 *   h0       : the chunk carry `state` starts at h0 instead of zeros;
 *   h_final  : the fp32 `state` after the last chunk.
 *
 * Arrays are fp32, row-major [N, T, C] (channel fastest).  bf16 values are
 * carried as fp32 numbers that are exactly representable in bf16.
 * Build: see oracle/Makefile (gcc -O2 -ffp-contract=off, pthreads).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORA_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------ */
/* rounding helpers                                                    */
/* ------------------------------------------------------------------ */

/* Round-to-nearest-even fp32 -> bf16 -> fp32 (c10::BFloat16 conversion). */
static inline float rbf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) { /* NaN: keep quiet NaN */
        u = 0x7fc00000u;
    } else {
        u += 0x7fffu + ((u >> 16) & 1u);
        u &= 0xffff0000u;
    }
    float r;
    memcpy(&r, &u, 4);
    return r;
}

/* fp32 -> fp16 -> fp32 with round-to-nearest-even (via the compiler's
 * _Float16 conversion, which is IEEE RNE on x86-64 with gcc >= 12). */
static inline float rf16(float f) { return (float)(_Float16)f; }

/* mode: 0 = fp32 (no rounding), 1 = bf16, 2 = fp16 */
static inline float rnd(float f, int mode) {
    return mode == 1 ? rbf16(f) : (mode == 2 ? rf16(f) : f);
}

/* torch CPU sigmoid: 1 / (1 + exp(-x)) computed in fp32. */
static inline float sigm(float x) {
    const float e = expf(-x);
    const float d = 1.0f + e;
    return 1.0f / d;
}

ORA_API void ora_round(float* x, int64_t n, int mode) {
    for (int64_t i = 0; i < n; ++i) x[i] = rnd(x[i], mode);
}

/* ------------------------------------------------------------------ */
/* thread pool over independent rows                                   */
/* ------------------------------------------------------------------ */

typedef void (*row_fn)(void* ctx, int64_t row);
typedef struct {
    row_fn fn;
    void* ctx;
    int64_t nrows;
    int64_t next;
    pthread_mutex_t mu;
} pool_t;

static void* pool_worker(void* p_) {
    pool_t* p = (pool_t*)p_;
    for (;;) {
        pthread_mutex_lock(&p->mu);
        int64_t r = p->next++;
        pthread_mutex_unlock(&p->mu);
        if (r >= p->nrows) break;
        p->fn(p->ctx, r);
    }
    return NULL;
}

static void run_rows(row_fn fn, void* ctx, int64_t nrows, int nthreads) {
    if (nthreads <= 1 || nrows <= 1) {
        for (int64_t r = 0; r < nrows; ++r) fn(ctx, r);
        return;
    }
    if (nthreads > 256) nthreads = 256;
    pool_t p;
    p.fn = fn;
    p.ctx = ctx;
    p.nrows = nrows;
    p.next = 0;
    pthread_mutex_init(&p.mu, NULL);
    pthread_t th[256];
    int started = 0;
    for (int i = 0; i < nthreads; ++i)
        if (pthread_create(&th[i], NULL, pool_worker, &p) == 0) ++started;
    if (started == 0) pool_worker(&p);
    for (int i = 0; i < started; ++i) pthread_join(th[i], NULL);
    pthread_mutex_destroy(&p.mu);
}

/* ------------------------------------------------------------------ */
/* chunked affine scan (need_kernels.py:177-226)                       */
/* ------------------------------------------------------------------ */

typedef struct {
    const float* a;
    const float* b;
    const float* h0;
    float* h;
    float* h_final;
    int64_t T, C, chunk, cblk;
} scan_ctx;

/* One work row = (n, channel block of cblk channels).  The chunk carry and the
 * doubling are independent per channel, so splitting channels changes no
 * result; it only spreads the work over threads. */
static void scan_row(void* ctx_, int64_t row) {
    scan_ctx* s = (scan_ctx*)ctx_;
    const int64_t T = s->T, C = s->C;
    const int64_t nblk = (C + s->cblk - 1) / s->cblk;
    const int64_t n = row / nblk;
    const int64_t c0 = (row % nblk) * s->cblk;
    const int64_t cw = (C - c0) < s->cblk ? (C - c0) : s->cblk;
    const int64_t chunk = s->chunk < 1 ? 1 : (s->chunk > T ? T : s->chunk);
    float* ap = (float*)malloc(sizeof(float) * chunk * cw);
    float* bp = (float*)malloc(sizeof(float) * chunk * cw);
    float* state = (float*)malloc(sizeof(float) * cw);
    for (int64_t c = 0; c < cw; ++c)
        state[c] = s->h0 ? s->h0[n * C + c0 + c] : 0.0f;
    const float* A = s->a + n * T * C;
    const float* B = s->b + n * T * C;
    float* H = s->h + n * T * C;
    for (int64_t start = 0; start < T; start += chunk) {
        const int64_t end = (start + chunk) < T ? (start + chunk) : T;
        const int64_t width = end - start;
        for (int64_t j = 0; j < width; ++j)
            for (int64_t c = 0; c < cw; ++c) {
                ap[j * cw + c] = A[(start + j) * C + c0 + c];
                bp[j * cw + c] = B[(start + j) * C + c0 + c];
            }
        for (int64_t shift = 1; shift < width; shift *= 2) {
            /* descending j keeps [j - shift] at its value from before this pass */
            for (int64_t j = width - 1; j >= shift; --j)
                for (int64_t c = 0; c < cw; ++c) {
                    const float a_cur = ap[j * cw + c];
                    const float a_prev = ap[(j - shift) * cw + c];
                    const float b_prev = bp[(j - shift) * cw + c];
                    const float prod = a_cur * b_prev;
                    bp[j * cw + c] = bp[j * cw + c] + prod;
                    ap[j * cw + c] = a_cur * a_prev;
                }
        }
        for (int64_t j = 0; j < width; ++j)
            for (int64_t c = 0; c < cw; ++c) {
                const float prod = ap[j * cw + c] * state[c];
                H[(start + j) * C + c0 + c] = bp[j * cw + c] + prod;
            }
        for (int64_t c = 0; c < cw; ++c) state[c] = H[(end - 1) * C + c0 + c];
    }
    if (s->h_final)
        for (int64_t c = 0; c < cw; ++c) s->h_final[n * C + c0 + c] = state[c];
    free(ap);
    free(bp);
    free(state);
}

/* h[n,t,c] = a[n,t,c] * h[n,t-1,c] + b[n,t,c], h[n,-1,c] = h0 (or 0).
 * Output is fp32 (round it with ora_round to the update dtype afterwards, as
 * the reference's final `.to(dtype=update.dtype)` does). */
ORA_API void ora_affine_scan(const float* a, const float* b, const float* h0, float* h,
                             float* h_final, int64_t N, int64_t T, int64_t C,
                             int64_t chunk, int nthreads) {
    if (N <= 0 || T <= 0 || C <= 0) return;
    scan_ctx s = {a, b, h0, h, h_final, T, C, chunk, 64};
    const int64_t nblk = (C + s.cblk - 1) / s.cblk;
    run_rows(scan_row, &s, N * nblk, nthreads);
}

/* Plain sequential recurrence in fp32 (h = a*h + b, separately rounded), the
 * definition the chunked form computes; used to cross-check the chunked form. */
ORA_API void ora_affine_scan_seq(const float* a, const float* b, const float* h0, float* h,
                                 float* h_final, int64_t N, int64_t T, int64_t C) {
    for (int64_t n = 0; n < N; ++n)
        for (int64_t c = 0; c < C; ++c) {
            float st = h0 ? h0[n * C + c] : 0.0f;
            for (int64_t t = 0; t < T; ++t) {
                const int64_t i = (n * T + t) * C + c;
                const float prod = a[i] * st;
                st = prod + b[i];
                h[i] = st;
            }
            if (h_final) h_final[n * C + c] = st;
        }
}

/* ------------------------------------------------------------------ */
/* gate arithmetic                                                     */
/* ------------------------------------------------------------------ */

/* The gate and epilogue passes are elementwise: a work row is (sequence n,
 * block of ORA_TBLK tokens), so one long sequence still spreads over every
 * thread.  Splitting changes no result. */
#define ORA_TBLK 64
static inline int64_t tblocks(int64_t T) { return (T + ORA_TBLK - 1) / ORA_TBLK; }

typedef struct {
    const float *x, *z, *g;
    const uint8_t* seg;
    float *a, *b;
    int64_t T, C;
    int mode;
} gated_ctx;

static void gated_row(void* ctx_, int64_t row) {
    gated_ctx* s = (gated_ctx*)ctx_;
    const int m = s->mode;
    const int64_t n = row / tblocks(s->T), t0 = (row % tblocks(s->T)) * ORA_TBLK;
    const int64_t t1 = t0 + ORA_TBLK < s->T ? t0 + ORA_TBLK : s->T;
    for (int64_t t = t0; t < t1; ++t) {
        const int reset = s->seg ? (s->seg[n * s->T + t] != 0) : 0;
        for (int64_t c = 0; c < s->C; ++c) {
            const int64_t i = (n * s->T + t) * s->C + c;
            const float dec = rnd(sigm(s->z[i]), m);
            const float gate = rnd(sigm(s->g[i]), m);
            const float gx = rnd(gate * s->x[i], m);
            const float om = rnd(1.0f - dec, m);
            s->b[i] = rnd(om * gx, m);
            s->a[i] = reset ? 0.0f : dec;
        }
    }
}

/* decay = sigmoid(z); update = (1 - decay) * (sigmoid(g) * x); decay := 0 where
 * seg[n,t] != 0.  mode: 0 fp32, 1 bf16, 2 fp16 (rounding after every op). */
ORA_API void ora_gated_prep(const float* x, const float* z, const float* g, const uint8_t* seg,
                            float* a, float* b, int64_t N, int64_t T, int64_t C, int mode,
                            int nthreads) {
    gated_ctx s = {x, z, g, seg, a, b, T, C, mode};
    run_rows(gated_row, &s, N * tblocks(T), nthreads);
}

typedef struct {
    const float *u, *bg, *dt;
    const uint8_t* seg;
    float *a, *b;
    int64_t T, C;
    float scale, off;
    int mode;
} ssdp_ctx;

static void ssd_prep_row(void* ctx_, int64_t row) {
    ssdp_ctx* s = (ssdp_ctx*)ctx_;
    const int m = s->mode;
    const int64_t n = row / tblocks(s->T), t0 = (row % tblocks(s->T)) * ORA_TBLK;
    const int64_t t1 = t0 + ORA_TBLK < s->T ? t0 + ORA_TBLK : s->T;
    for (int64_t t = t0; t < t1; ++t) {
        const int reset = s->seg ? (s->seg[n * s->T + t] != 0) : 0;
        for (int64_t c = 0; c < s->C; ++c) {
            const int64_t i = (n * s->T + t) * s->C + c;
            /* need_kernels.py:330-332: dt is fp32 whatever the input dtype */
            const float sd = sigm(s->dt[i]);
            const float scaled = sd * s->scale;
            const float dtv = scaled + s->off;
            const float dec = rnd(expf(-dtv), m);
            const float bgs = rnd(sigm(s->bg[i]), m);
            const float bu = rnd(bgs * s->u[i], m);
            const float om = rnd(1.0f - dec, m);
            s->b[i] = rnd(om * bu, m);
            s->a[i] = reset ? 0.0f : dec;
        }
    }
}

/* ssd_scan's decay/update (need_kernels.py:330-336).  dt_min/dt_max are the
 * Python floats; their difference is taken in double and cast to fp32 exactly
 * as torch casts a Python scalar operand to the tensor's compute type. */
ORA_API void ora_ssd_prep(const float* u, const float* bg, const float* dt, const uint8_t* seg,
                          float* a, float* b, int64_t N, int64_t T, int64_t C, double dt_min,
                          double dt_max, int mode, int nthreads) {
    ssdp_ctx s = {u, bg, dt, seg, a, b, T, C, (float)(dt_max - dt_min), (float)dt_min, mode};
    run_rows(ssd_prep_row, &s, N * tblocks(T), nthreads);
}

typedef struct {
    const float *h, *u, *cg, *og, *dskip;
    float* y;
    int64_t T, C;
    int mode;
} ssde_ctx;

static void ssd_epi_row(void* ctx_, int64_t row) {
    ssde_ctx* s = (ssde_ctx*)ctx_;
    const int m = s->mode;
    const int64_t n = row / tblocks(s->T), t0 = (row % tblocks(s->T)) * ORA_TBLK;
    const int64_t t1 = t0 + ORA_TBLK < s->T ? t0 + ORA_TBLK : s->T;
    for (int64_t t = t0; t < t1; ++t)
        for (int64_t c = 0; c < s->C; ++c) {
            const int64_t i = (n * s->T + t) * s->C + c;
            const float cgs = rnd(sigm(s->cg[i]), m);
            const float ogs = rnd(sigm(s->og[i]), m);
            const float d = rnd(s->dskip[c], m);
            const float hs = rnd(s->h[i], m); /* state_seq in u.dtype */
            const float p1 = rnd(cgs * hs, m);
            const float p2 = rnd(d * s->u[i], m);
            const float sum = rnd(p1 + p2, m);
            s->y[i] = rnd(sum * ogs, m);
        }
}

/* y = (sigmoid(cg) * state_seq + D * u) * sigmoid(og)  (need_kernels.py:333-339) */
ORA_API void ora_ssd_epilogue(const float* h, const float* u, const float* cg, const float* og,
                              const float* dskip, float* y, int64_t N, int64_t T, int64_t C,
                              int mode, int nthreads) {
    ssde_ctx s = {h, u, cg, og, dskip, y, T, C, mode};
    run_rows(ssd_epi_row, &s, N * tblocks(T), nthreads);
}

/* ------------------------------------------------------------------ */
/* RMSNorm after the scan (the SSD block's out_norm)                   */
/* ------------------------------------------------------------------ */

/* out[r, :] = x[r, :] * rsqrt(sum_c(x[r, c]^2) / n + eps) * w, the reference's
 * GPU rms_norm (need_kernels.py:99-107, the kernel need_core.py:1396 reaches on
 * CUDA): x widened to fp32, the sum of squares and the scale in fp32, the two
 * products separately rounded fp32 ops, the result rounded once to `mode` (the
 * store into a tensor of x's dtype).  The sum is accumulated in double and
 * rounded to fp32, so the checker is independent of the kernel's order of
 * summation; rsqrt is 1/sqrt in double, rounded to fp32. */
ORA_API void ora_rms_norm(const float* x, const float* w, float* out, int64_t rows, int64_t n, double eps,
                          int mode) {
    for (int64_t r = 0; r < rows; ++r) {
        const float* xr = x + r * n;
        double acc = 0.0;
        for (int64_t c = 0; c < n; ++c) acc += (double)xr[c] * (double)xr[c];
        const float ss = (float)acc / (float)n;
        const float inv = (float)(1.0 / sqrt((double)(ss + (float)eps)));
        for (int64_t c = 0; c < n; ++c) {
            const float p = xr[c] * inv;
            out[r * n + c] = rnd(p * w[c], mode);
        }
    }
}

/* ------------------------------------------------------------------ */
/* matrix-state associative memory                                     */
/* ------------------------------------------------------------------ */

/* HierarchicalMemory._linear_associative_memory (need_core.py:1960-2001):
 *   qf = rnd(elu(q_raw) + 1), kf = rnd(elu(k_raw) + 1)   (fp32 in, model dtype out;
 *        torch's CPU elu is expm1 below 0)
 *   with a write mask: kf = rnd(kf * wm), v = rnd(v * wm)
 *   per chunk of `chunk` tokens, with state [r, d] and denom_state [r] in the model dtype:
 *     kv[s]      = rnd(kf[s] (x) v[s])                     (outer product)
 *     state_c[s] = rnd(state + rnd(cumsum_s kv))            (fp32 running sum, rounded per s)
 *     denom_c[s] = rnd(denom_state + rnd(cumsum_s kf))
 *     numer[s]   = rnd(sum_i qf[s,i] * state_c[s,i,:])     (fp32 accumulation)
 *     den[s]     = max(rnd(sum_i rnd(qf[s,i] * denom_c[s,i])), rnd(1e-6))
 *     out[s]     = rnd(numer[s] / den[s])
 *   and state, denom_state := state_c, denom_c of the chunk's last token.
 * q_raw, k_raw [B, T, r] fp32; v [B, T, d] (values in the model dtype); wm [B, T]
 * or NULL; out [B, T, d]. */
typedef struct {
    const float *q, *k, *v, *wm;
    float* out;
    int64_t T, r, d, chunk;
    int mode;
} assoc_ctx;

static void assoc_row(void* ctx_, int64_t b) {
    const assoc_ctx* s = (const assoc_ctx*)ctx_;
    const int m = s->mode;
    const int64_t T = s->T, r = s->r, d = s->d;
    float* state = calloc((size_t)(r * d), sizeof(float));
    float* denom_state = calloc((size_t)r, sizeof(float));
    float* acc = malloc(sizeof(float) * (size_t)(r * d));    /* fp32 cumsum of kv */
    float* acck = malloc(sizeof(float) * (size_t)r);         /* fp32 cumsum of kf */
    float* sc = malloc(sizeof(float) * (size_t)(r * d));     /* state_c[s] */
    float* dc = malloc(sizeof(float) * (size_t)r);           /* denom_c[s] */
    float* qf = malloc(sizeof(float) * (size_t)r);
    float* kf = malloc(sizeof(float) * (size_t)r);
    float* vv = malloc(sizeof(float) * (size_t)d);
    const float eps = rnd(1e-6f, m);
    for (int64_t t0 = 0; t0 < T; t0 += s->chunk) {
        const int64_t t1 = t0 + s->chunk < T ? t0 + s->chunk : T;
        memset(acc, 0, sizeof(float) * (size_t)(r * d));
        memset(acck, 0, sizeof(float) * (size_t)r);
        for (int64_t t = t0; t < t1; ++t) {
            const int64_t row = b * T + t;
            const float w = s->wm ? rnd(fminf(fmaxf(s->wm[row], 0.0f), 1.0f), m) : 1.0f;
            for (int64_t i = 0; i < r; ++i) {
                const float qv = s->q[row * r + i], kv = s->k[row * r + i];
                qf[i] = rnd((qv > 0.0f ? qv : expm1f(qv)) + 1.0f, m);
                kf[i] = rnd((kv > 0.0f ? kv : expm1f(kv)) + 1.0f, m);
                if (s->wm) kf[i] = rnd(kf[i] * w, m);
            }
            for (int64_t j = 0; j < d; ++j) vv[j] = s->wm ? rnd(s->v[row * d + j] * w, m) : s->v[row * d + j];
            for (int64_t i = 0; i < r; ++i) {
                acck[i] += kf[i];
                dc[i] = rnd(denom_state[i] + rnd(acck[i], m), m);
                for (int64_t j = 0; j < d; ++j) {
                    acc[i * d + j] += rnd(kf[i] * vv[j], m);
                    sc[i * d + j] = rnd(state[i * d + j] + rnd(acc[i * d + j], m), m);
                }
            }
            float den = 0.0f;
            for (int64_t i = 0; i < r; ++i) den += rnd(qf[i] * dc[i], m);
            den = rnd(den, m);
            if (den < eps) den = eps;
            for (int64_t j = 0; j < d; ++j) {
                float num = 0.0f;
                for (int64_t i = 0; i < r; ++i) num += qf[i] * sc[i * d + j];
                s->out[row * d + j] = rnd(rnd(num, m) / den, m);
            }
        }
        memcpy(state, sc, sizeof(float) * (size_t)(r * d));
        memcpy(denom_state, dc, sizeof(float) * (size_t)r);
    }
    free(state); free(denom_state); free(acc); free(acck); free(sc); free(dc); free(qf); free(kf); free(vv);
}

/* One token of HierarchicalMemory.stream_step's associative memory
 * (need_core.py:2067-2080), in place on the model-dtype state [N, r, d] and
 * denom [N, r]:
 *   state = rnd(state + rnd(kf (x) v)), denom = rnd(denom + kf),
 *   out = rnd(rnd(sum_i qf_i state_i) / max(rnd(sum_i rnd(qf_i denom_i)), rnd(1e-6)))
 * with qf, kf and the write mask as in ora_assoc_memory.  q_raw, k_raw [N, r]
 * fp32; v [N, d]; wm [N] or NULL; out [N, d]. */
ORA_API void ora_assoc_step(const float* q_raw, const float* k_raw, const float* v, const float* wm, float* state,
                            float* denom, float* out, int64_t N, int64_t r, int64_t d, int mode) {
    const float eps = rnd(1e-6f, mode);
    float* qf = malloc(sizeof(float) * (size_t)r);
    float* kf = malloc(sizeof(float) * (size_t)r);
    float* vv = malloc(sizeof(float) * (size_t)d);
    for (int64_t n = 0; n < N; ++n) {
        const float w = wm ? rnd(fminf(fmaxf(wm[n], 0.0f), 1.0f), mode) : 1.0f;
        for (int64_t i = 0; i < r; ++i) {
            const float qv = q_raw[n * r + i], kv = k_raw[n * r + i];
            qf[i] = rnd((qv > 0.0f ? qv : expm1f(qv)) + 1.0f, mode);
            kf[i] = rnd((kv > 0.0f ? kv : expm1f(kv)) + 1.0f, mode);
            if (wm) kf[i] = rnd(kf[i] * w, mode);
        }
        for (int64_t j = 0; j < d; ++j) vv[j] = wm ? rnd(v[n * d + j] * w, mode) : v[n * d + j];
        float* st = state + n * r * d;
        float* dn = denom + n * r;
        float den = 0.0f;
        for (int64_t i = 0; i < r; ++i) {
            dn[i] = rnd(dn[i] + kf[i], mode);
            den += rnd(qf[i] * dn[i], mode);
            for (int64_t j = 0; j < d; ++j) st[i * d + j] = rnd(st[i * d + j] + rnd(kf[i] * vv[j], mode), mode);
        }
        den = rnd(den, mode);
        if (den < eps) den = eps;
        for (int64_t j = 0; j < d; ++j) {
            float num = 0.0f;
            for (int64_t i = 0; i < r; ++i) num += qf[i] * st[i * d + j];
            out[n * d + j] = rnd(rnd(num, mode) / den, mode);
        }
    }
    free(qf); free(kf); free(vv);
}

ORA_API void ora_assoc_memory(const float* q_raw, const float* k_raw, const float* v, const float* wm, float* out,
                              int64_t B, int64_t T, int64_t r, int64_t d, int64_t chunk, int mode, int nthreads) {
    assoc_ctx s = {q_raw, k_raw, v, wm, out, T, r, d, chunk, mode};
    run_rows(assoc_row, &s, B, nthreads);
}

/* ------------------------------------------------------------------ */
/* one-token recurrent step (streaming decode)                         */
/* ------------------------------------------------------------------ */

/* form 2 (selective retention, need_core.py:1590-1592 and :6440-6444):
 *                  state = decay*state + k*v; y = q*state, with p0 = decay (the
 *                  per-head value repeated over its channels), p1 = k, p2 = v, p3 = q
 * form 0 (gated):  dec = sigmoid(p0); upd = (1-dec)*(sigmoid(p1)*p2)
 *                  state = dec*state + upd; y = state
 * form 1 (ssd):    p0=dt_raw, p1=b_gate, p2=u_act, p3=c_gate, p4=out_gate
 *                  dec = exp(-(dt_min + (dt_max-dt_min)*sigmoid(p0)))
 *                  state = dec*state + (1-dec)*(sigmoid(p1)*p2)
 *                  y = (sigmoid(p3)*state + D*p2) * sigmoid(p4)
 * (need_core.py:6420-6428 and :1674-1685).  Every op rounds to `mode`;
 * state is [N, C] in the model dtype; p* are [N, C]. */
/* One token of the SSD block's causal depthwise conv from its history, then
 * SiLU, in the model dtype (need_core.py:6395-6409 and :6413-6414):
 *   full = [hist_0 .. hist_{K-2}, u]          (oldest first)
 *   u_conv = rnd(rnd(sum_j rnd(full_j * rnd(w[c, j]))) + rnd(b[c]))
 *   hist := full[1:], u_act = rnd(u_conv / (1 + exp(-u_conv)))
 * The tap products are separately rounded (a bf16 elementwise product), their
 * sum is accumulated in fp32 in tap order and rounded once (torch's bf16
 * sum), and SiLU is computed in fp32 (torch's CPU silu for 16-bit inputs).
 * hist: [N, C, K-1] in/out; u, u_act: [N, C]; w: [C, K] fp32; bias: [C] or
 * NULL. */
ORA_API void ora_conv_step(float* hist, const float* u, const float* w, const float* bias, float* u_act,
                           int64_t N, int64_t C, int64_t K, int mode) {
    for (int64_t n = 0; n < N; ++n)
        for (int64_t c = 0; c < C; ++c) {
            float* h = hist + (n * C + c) * (K - 1);
            const float un = u[n * C + c];
            float acc = 0.0f;
            for (int64_t j = 0; j < K; ++j) {
                const float fj = j < K - 1 ? h[j] : un;
                acc = acc + rnd(fj * rnd(w[c * K + j], mode), mode);
            }
            float uc = rnd(acc, mode);
            if (bias) uc = rnd(uc + rnd(bias[c], mode), mode);
            for (int64_t j = 0; j + 1 < K - 1; ++j) h[j] = h[j + 1];
            if (K > 1) h[K - 2] = un;
            const float e = expf(-uc);
            u_act[n * C + c] = rnd(uc / (1.0f + e), mode);
        }
}

/* The SSD block's input prologue over a whole sequence (need_core.py:1620-1623):
 *   u_conv = dwconv(u)[..., :T]   (nn.Conv1d(C, C, K, padding=K-1, groups=C))
 *   u_act  = F.silu(u_conv)
 * in the model dtype as the reference computes it on CPU: per (t, c) the
 * bias plus the K taps w[c, j] * u[t-K+1+j, c] (oldest first) summed in fp32
 * and rounded once, then SiLU in fp32 (x / (1 + exp(-x))) rounded once; rows
 * before t = 0 are zero.  With seg (optional [N, T]) rows before the segment
 * start of t are zero too (a reset the reference's module has no input for).
 * u, out [N, T, C]; w [C, K]; bias [C] or NULL. */
ORA_API void ora_conv_silu(const float* u, const float* w, const float* bias, const uint8_t* seg, float* out,
                           int64_t N, int64_t T, int64_t C, int64_t K, int mode) {
    for (int64_t n = 0; n < N; ++n) {
        int64_t start = 0; /* first row of the current segment */
        for (int64_t t = 0; t < T; ++t) {
            if (seg && seg[n * T + t]) start = t;
            for (int64_t c = 0; c < C; ++c) {
                float acc = bias ? bias[c] : 0.0f;
                for (int64_t j = 0; j < K; ++j) {
                    const int64_t tt = t - (K - 1) + j;
                    const float x = (tt >= 0 && tt >= start) ? u[(n * T + tt) * C + c] : 0.0f;
                    acc = fmaf(w[c * K + j], x, acc);
                }
                const float uc = rnd(acc, mode);
                out[(n * T + t) * C + c] = rnd(uc / (1.0f + expf(-uc)), mode);
            }
        }
    }
}

ORA_API void ora_stream_step(int form, float* state, const float* p0, const float* p1,
                             const float* p2, const float* p3, const float* p4,
                             const float* dskip, float* y, int64_t N, int64_t C,
                             double dt_min, double dt_max, int mode) {
    const float scale = (float)(dt_max - dt_min), off = (float)dt_min;
    if (form == 2) { /* selective retention: p0 = decay (per channel), p1 = k, p2 = v, p3 = q */
        for (int64_t i = 0; i < N * C; ++i) {
            const float st = rnd(rnd(p0[i] * state[i], mode) + rnd(p1[i] * p2[i], mode), mode);
            state[i] = st;
            y[i] = rnd(p3[i] * st, mode);
        }
        return;
    }
    for (int64_t n = 0; n < N; ++n)
        for (int64_t c = 0; c < C; ++c) {
            const int64_t i = n * C + c;
            float dec;
            if (form == 0) {
                dec = rnd(sigm(p0[i]), mode);
            } else {
                const float sd = sigm(p0[i]);
                const float scaled = sd * scale;
                const float dtv = scaled + off;
                dec = rnd(expf(-dtv), mode);
            }
            const float gs = rnd(sigm(p1[i]), mode);
            const float prev = state[i];
            const float t1 = rnd(dec * prev, mode);
            const float om = rnd(1.0f - dec, mode);
            const float gu = rnd(gs * p2[i], mode);
            const float upd = rnd(om * gu, mode);
            const float st = rnd(t1 + upd, mode);
            state[i] = st;
            if (form == 0) {
                y[i] = st;
            } else {
                const float cgs = rnd(sigm(p3[i]), mode);
                const float ogs = rnd(sigm(p4[i]), mode);
                const float d = rnd(dskip[c], mode);
                const float q1 = rnd(cgs * st, mode);
                const float q2 = rnd(d * p2[i], mode);
                const float sum = rnd(q1 + q2, mode);
                y[i] = rnd(sum * ogs, mode);
            }
        }
}

/*
 * moe_oracle.c — CPU restatement of the mlx-rs MoE (SwitchGLU) block.
 *
 * TEST INFRASTRUCTURE ONLY (the checker for the CUDA path; see moe_oracle.h for the
 * parity status: unpinned, MLX absent). Built with -ffp-contract=off so that every
 * fused multiply-add is an explicit fmaf() and nothing else is contracted.
 *
 * Reference op sequence restated here (paths relative to the reference project):
 *   SparseMoeBlock::forward        crates/mlx-models/src/qwen3_moe_python_port.rs:420-488
 *   SwitchGlu::forward             crates/mlx-models/src/qwen3_moe_python_port.rs:352-359
 *   SwitchLinear::forward          crates/mlx-models/src/qwen3_moe_python_port.rs:311-334
 *   SharedExpert::forward          crates/mlx-models/src/qwen3_moe_python_port.rs:385-390
 *   MoeFeedForward::forward        crates/mlx-models/src/lfm2_moe_python_port.rs:541-740
 *   Linear::forward (quantized)    crates/mlx-nn/src/linear.rs:117-139
 *   Array::gather_qmm              crates/mlx-core/src/ops.rs:830-891
 *   Array::quantized_matmul        crates/mlx-core/src/ops.rs:592-637
 *   RmsNorm::forward               crates/mlx-nn/src/rms_norm.rs:30-34
 */
#include "moe_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------------------- */
/* parallel_for: n work items over nthreads pthreads, dynamic chunks of `chunk`.
 * Every output element is written by exactly one item, so results do not depend
 * on the thread count or the schedule. */
/* ------------------------------------------------------------------------- */

typedef void (*pf_fn)(int64_t begin, int64_t end, void* ctx, void* scratch);

typedef struct {
    pf_fn fn;
    void* ctx;
    int64_t n, chunk;
    size_t scratch_bytes;
    int64_t next; /* guarded by mu */
    pthread_mutex_t mu;
} pf_state;

static void* pf_worker(void* arg) {
    pf_state* st = (pf_state*)arg;
    void* scratch = st->scratch_bytes ? malloc(st->scratch_bytes) : NULL;
    for (;;) {
        pthread_mutex_lock(&st->mu);
        int64_t b = st->next;
        st->next += st->chunk;
        pthread_mutex_unlock(&st->mu);
        if (b >= st->n) break;
        int64_t e = b + st->chunk < st->n ? b + st->chunk : st->n;
        st->fn(b, e, st->ctx, scratch);
    }
    free(scratch);
    return NULL;
}

static int default_threads(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

static void parallel_for(int64_t n, int64_t chunk, int nthreads, size_t scratch_bytes, pf_fn fn,
                         void* ctx) {
    if (n <= 0) return;
    if (nthreads <= 0) nthreads = default_threads();
    if (chunk <= 0) chunk = 1;
    pf_state st;
    st.fn = fn;
    st.ctx = ctx;
    st.n = n;
    st.chunk = chunk;
    st.scratch_bytes = scratch_bytes;
    st.next = 0;
    pthread_mutex_init(&st.mu, NULL);
    if (nthreads == 1 || n <= chunk) {
        pf_worker(&st);
        pthread_mutex_destroy(&st.mu);
        return;
    }
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nthreads);
    int started = 0;
    for (int i = 0; i < nthreads; ++i) {
        if (pthread_create(&th[i], NULL, pf_worker, &st) != 0) break;
        started++;
    }
    if (started == 0) pf_worker(&st);
    for (int i = 0; i < started; ++i) pthread_join(th[i], NULL);
    free(th);
    pthread_mutex_destroy(&st.mu);
}

/* ------------------------------------------------------------------------- */
/* bf16 helpers                                                               */
/* ------------------------------------------------------------------------- */

static inline float bf2f(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Round-to-nearest-even fp32 -> bf16 (NaN kept quiet). */
static inline uint16_t f2bf(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float rbf(float f) { return bf2f(f2bf(f)); }

uint16_t oracle_f32_to_bf16(float x) { return f2bf(x); }

/* ------------------------------------------------------------------------- */
/* exp / sigmoid                                                              */
/* ------------------------------------------------------------------------- */

/*
 * exp(x) by Cody-Waite range reduction (W. J. Cody, W. Waite, "Software Manual for
 * the Elementary Functions", 1980): n = rint(x*log2(e)), r = x - n*ln2 with ln2
 * split into a 12-bit-short high part (n*LN2_HI is exact) and a low part, then
 * exp(r) by the degree-7 Taylor polynomial sum r^i/i! (|r| <= 0.347, truncation
 * error < 1e-8 relative) in Horner form with fmaf, scaled by 2^n. Inputs above 88
 * give +inf and below -87 give 0 by definition. The CUDA kernels evaluate the same
 * sequence of IEEE operations, so both produce identical bits.
 */
#define OR_LOG2E 0x1.715476p+0f
#define OR_LN2_HI 0x1.62ep-1f /* 0.693115234375 */
#define OR_LN2_LO 0x1.0bfbe8p-15f
#define OR_C2 0x1.0p-1f
#define OR_C3 0x1.555556p-3f
#define OR_C4 0x1.555556p-5f
#define OR_C5 0x1.111112p-7f
#define OR_C6 0x1.6c16c2p-10f
#define OR_C7 0x1.a01a02p-13f

float oracle_exp(float x) {
    if (x != x) return x;
    if (x > 88.0f) return INFINITY;
    if (x < -87.0f) return 0.0f;
    float t = x * OR_LOG2E;
    float n = rintf(t);
    float r = fmaf(-n, OR_LN2_HI, x);
    r = fmaf(-n, OR_LN2_LO, r);
    float p = OR_C7;
    p = fmaf(p, r, OR_C6);
    p = fmaf(p, r, OR_C5);
    p = fmaf(p, r, OR_C4);
    p = fmaf(p, r, OR_C3);
    p = fmaf(p, r, OR_C2);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int32_t ni = (int32_t)n;
    uint32_t sb = (uint32_t)(ni + 127) << 23;
    float scale;
    memcpy(&scale, &sb, 4);
    return p * scale;
}

/* sigmoid(x) = 1 / (1 + exp(-x)), IEEE add and divide. */
float oracle_sigmoid(float x) { return 1.0f / (1.0f + oracle_exp(-x)); }

/* ------------------------------------------------------------------------- */
/* Canonical dot product                                                      */
/* ------------------------------------------------------------------------- */

/*
 * The canonical fp32 accumulation order of every quantized matmul in this oracle
 * (and, bit for bit, of the CUDA router kernel):
 *   K is cut into chunks of 32 consecutive elements. 32 "lanes" l = 0..31 each own
 *   the chunks c = l, l+32, l+64, ... and accumulate, starting from +0.0f,
 *       acc_l = fmaf(x[e], w[e], acc_l)   for e = 32c .. 32c+31 in order,
 *   where w[e] = fmaf(scale[g], (float)q[e], bias[g]), g = e / group_size, is the
 *   affine dequantisation of the packed field q[e] (lowest bits first in each
 *   uint32, the MLX packing). The 32 partial sums are then combined by the xor
 *   butterfly acc_l <- acc_l + acc_(l^o) for o = 16, 8, 4, 2, 1, and the result is
 *   acc_0.
 */
static float butterfly32(float* a) {
    float t[32];
    for (int off = 16; off >= 1; off >>= 1) {
        for (int l = 0; l < 32; ++l) t[l] = a[l] + a[l ^ off];
        memcpy(a, t, sizeof(t));
    }
    return a[0];
}

static inline uint32_t qfield(const uint32_t* wrow, int64_t e, int bits) {
    const int epw = 32 / bits;
    const uint32_t mask = (1u << bits) - 1u;
    return (wrow[e / epw] >> ((e % epw) * bits)) & mask;
}

float oracle_dot_canonical(const uint16_t* x, const uint32_t* wrow, const uint16_t* srow,
                           const uint16_t* brow, int64_t K, int gs, int bits) {
    float acc[32];
    const int64_t nchunks = K / 32;
    for (int l = 0; l < 32; ++l) {
        float a = 0.0f;
        for (int64_t c = l; c < nchunks; c += 32) {
            for (int j = 0; j < 32; ++j) {
                const int64_t e = 32 * c + j;
                const int64_t g = e / gs;
                const float q = (float)qfield(wrow, e, bits);
                const float wv = fmaf(bf2f(srow[g]), q, brow ? bf2f(brow[g]) : 0.0f);
                a = fmaf(bf2f(x[e]), wv, a);
            }
        }
        acc[l] = a;
    }
    return butterfly32(acc);
}

/*
 * Fast evaluation of the same order: x and the dequantised row are first laid out
 * "lane-major" (element 32*(l+32r)+j stored at [(r*32 + j)*32 + l], zero padded),
 * so the 32 lane accumulators update as one vector per (r, j). Each lane still sees
 * its elements in the canonical sequence and padding adds fmaf(0,0,acc) == acc
 * (acc is never -0: it starts at +0 and a round-to-nearest sum is -0 only when
 * both addends are).
 */
static int64_t lane_rounds(int64_t K) { return (K / 32 + 31) / 32; }

static void x_to_lane_major(const uint16_t* x, int64_t K, float* xt) {
    const int64_t nr = lane_rounds(K), nchunks = K / 32;
    for (int64_t r = 0; r < nr; ++r)
        for (int j = 0; j < 32; ++j)
            for (int l = 0; l < 32; ++l) {
                const int64_t c = l + 32 * r;
                xt[(r * 32 + j) * 32 + l] = (c < nchunks) ? bf2f(x[32 * c + j]) : 0.0f;
            }
}

static void w_to_lane_major(const uint32_t* wrow, const uint16_t* srow, const uint16_t* brow,
                            int64_t K, int gs, int bits, float* wt) {
    const int64_t nr = lane_rounds(K), nchunks = K / 32;
    for (int64_t r = 0; r < nr; ++r)
        for (int j = 0; j < 32; ++j)
            for (int l = 0; l < 32; ++l) {
                const int64_t c = l + 32 * r;
                float v = 0.0f;
                if (c < nchunks) {
                    const int64_t e = 32 * c + j, g = e / gs;
                    v = fmaf(bf2f(srow[g]), (float)qfield(wrow, e, bits),
                             brow ? bf2f(brow[g]) : 0.0f);
                }
                wt[(r * 32 + j) * 32 + l] = v;
            }
}

static float dot_lane_major(const float* xt, const float* wt, int64_t nr) {
    float acc[32];
    for (int l = 0; l < 32; ++l) acc[l] = 0.0f;
    for (int64_t r = 0; r < nr; ++r)
        for (int j = 0; j < 32; ++j) {
            const float* xp = xt + (r * 32 + j) * 32;
            const float* wp = wt + (r * 32 + j) * 32;
            for (int l = 0; l < 32; ++l) acc[l] = fmaf(xp[l], wp[l], acc[l]);
        }
    return butterfly32(acc);
}

static int check_q(int64_t K, int gs, int bits) {
    if (!(bits == 2 || bits == 4 || bits == 8)) return -1;
    if (!(gs == 32 || gs == 64 || gs == 128)) return -2;
    if (K <= 0 || K % gs != 0) return -3;
    return 0;
}

/* ------------------------------------------------------------------------- */
/* quantized_matmul / gather_qmm (transpose = true)                          */
/* ------------------------------------------------------------------------- */

typedef struct {
    const float* xt;
    const uint32_t* w;
    const uint16_t *s, *b;
    uint16_t* out;
    int64_t M, K, N;
    int gs, bits;
    int64_t nr, L, wpr, gpr;
} qmm_ctx;

static void qmm_rows(int64_t n0, int64_t n1, void* vctx, void* scratch) {
    const qmm_ctx* c = (const qmm_ctx*)vctx;
    float* wt = (float*)scratch;
    for (int64_t n = n0; n < n1; ++n) {
        w_to_lane_major(c->w + n * c->wpr, c->s + n * c->gpr, c->b ? c->b + n * c->gpr : NULL, c->K,
                        c->gs, c->bits, wt);
        for (int64_t m = 0; m < c->M; ++m)
            c->out[m * c->N + n] = f2bf(dot_lane_major(c->xt + m * c->L, wt, c->nr));
    }
}

/* out[m, n] = bf16(dot(x[m], W[n])) — mlx_quantized_matmul, transpose=true, affine
 * (crates/mlx-core/src/ops.rs:592-637 via crates/mlx-nn/src/linear.rs:117-128). */
int oracle_qmm(const uint16_t* x, int64_t M, int64_t K, const uint32_t* w, const uint16_t* s,
               const uint16_t* b, int64_t N, int gs, int bits, uint16_t* out, int nthreads) {
    int rc = check_q(K, gs, bits);
    if (rc) return rc;
    if (M == 0 || N == 0) return 0;
    const int64_t nr = lane_rounds(K), L = nr * 32 * 32;
    const int64_t wpr = K * bits / 32, gpr = K / gs;
    float* xt = (float*)malloc(sizeof(float) * L * M);
    if (!xt) return -10;
    for (int64_t m = 0; m < M; ++m) x_to_lane_major(x + m * K, K, xt + m * L);
    qmm_ctx c = {xt, w, s, b, out, M, K, N, gs, bits, nr, L, wpr, gpr};
    parallel_for(N, 4, nthreads, sizeof(float) * L, qmm_rows, &c);
    free(xt);
    return 0;
}

typedef struct {
    const float* xt;
    const uint32_t* w;
    const uint16_t *s, *b;
    uint16_t* out;
    const uint32_t* lhs;
    const int64_t *cnt, *order;
    int64_t x_repeat, K, N;
    int gs, bits;
    int64_t nr, L, wpr, gpr;
} gqmm_ctx;

static void gqmm_rows(int64_t r0, int64_t r1, void* vctx, void* scratch) {
    const gqmm_ctx* c = (const gqmm_ctx*)vctx;
    float* wt = (float*)scratch;
    for (int64_t row = r0; row < r1; ++row) {
        const int64_t e = row / c->N, n = row % c->N;
        if (c->cnt[e + 1] == c->cnt[e]) continue;
        w_to_lane_major(c->w + row * c->wpr, c->s + row * c->gpr, c->b ? c->b + row * c->gpr : NULL,
                        c->K, c->gs, c->bits, wt);
        for (int64_t p = c->cnt[e]; p < c->cnt[e + 1]; ++p) {
            const int64_t i = c->order[p];
            const int64_t r = c->lhs ? (int64_t)c->lhs[i] : i / c->x_repeat;
            c->out[i * c->N + n] = f2bf(dot_lane_major(c->xt + r * c->L, wt, c->nr));
        }
    }
}

/*
 * out[i, n] = bf16(dot(x[row(i)], W[rhs[i], n])) for i < batch, with
 * row(i) = lhs ? lhs[i] : i / x_repeat — mlx_gather_qmm with transpose=true and
 * one row per batch element, the form SwitchLinear::forward uses
 * (qwen3_moe_python_port.rs:311-324: x [T,1,1,K] broadcast against rhs [T,k] gives
 * x_repeat = k; the down projection passes x [T,k,1,I], x_repeat = 1).
 */
int oracle_gather_qmm(const uint16_t* x, int64_t K, int64_t x_repeat, const uint32_t* lhs,
                      const uint32_t* w, const uint16_t* s, const uint16_t* b, int64_t E,
                      int64_t N, const uint32_t* rhs, int64_t batch, int gs, int bits,
                      uint16_t* out, int nthreads) {
    int rc = check_q(K, gs, bits);
    if (rc) return rc;
    if (batch == 0 || N == 0) return 0;
    if (x_repeat <= 0) return -4;
    for (int64_t i = 0; i < batch; ++i)
        if (rhs[i] >= (uint32_t)E) return -5;
    int64_t xrows = 0;
    for (int64_t i = 0; i < batch; ++i) {
        int64_t r = lhs ? (int64_t)lhs[i] : i / x_repeat;
        if (r + 1 > xrows) xrows = r + 1;
    }
    const int64_t nr = lane_rounds(K), L = nr * 32 * 32;
    const int64_t wpr = K * bits / 32, gpr = K / gs;
    float* xt = (float*)malloc(sizeof(float) * L * xrows);
    int64_t* cnt = (int64_t*)calloc((size_t)E + 1, sizeof(int64_t));
    int64_t* order = (int64_t*)malloc(sizeof(int64_t) * batch);
    int64_t* cur = (int64_t*)malloc(sizeof(int64_t) * (E + 1));
    if (!xt || !cnt || !order || !cur) {
        free(xt);
        free(cnt);
        free(order);
        free(cur);
        return -10;
    }
    for (int64_t r = 0; r < xrows; ++r) x_to_lane_major(x + r * K, K, xt + r * L);
    for (int64_t i = 0; i < batch; ++i) cnt[rhs[i] + 1]++;
    for (int64_t e = 0; e < E; ++e) cnt[e + 1] += cnt[e];
    memcpy(cur, cnt, sizeof(int64_t) * (E + 1));
    for (int64_t i = 0; i < batch; ++i) order[cur[rhs[i]]++] = i;
    gqmm_ctx c = {xt, w, s, b, out, lhs, cnt, order, x_repeat, K, N, gs, bits, nr, L, wpr, gpr};
    parallel_for(E * N, 4, nthreads, sizeof(float) * L, gqmm_rows, &c);
    free(xt);
    free(cnt);
    free(order);
    free(cur);
    return 0;
}

/* ------------------------------------------------------------------------- */
/* Routing                                                                    */
/* ------------------------------------------------------------------------- */

/* Canonical sum of n fp32 values: lane l adds elements l, l+32, ... in order
 * starting from +0.0f, then the xor butterfly. */
static float sum_canonical(const float* v, int64_t n) {
    float acc[32];
    for (int l = 0; l < 32; ++l) {
        float a = 0.0f;
        for (int64_t e = l; e < n; e += 32) a = a + v[e];
        acc[l] = a;
    }
    return butterfly32(acc);
}

/* Internal precision of the routing softmax. The reference calls mlx_softmax_axis with
 * precise=false (crates/mlx-core/src/ops.rs:226-233) on bf16 logits; whether MLX then
 * computes in fp32 or in the input type depends on its backend and version, neither of
 * which is visible here, so the oracle offers both:
 *   ORACLE_SOFTMAX_F32 (default, and what the CUDA path computes): m = max,
 *     e_i = exp(l_i - m) in fp32, p_i = bf16(e_i / canonical_sum(e));
 *   ORACLE_SOFTMAX_BF16: every intermediate in bf16, the accumulation type being the
 *     input type: d_i = bf16(l_i - m), e_i = bf16(exp(d_i)), s = bf16(s + e_i) in element
 *     order, r = bf16(1 / s), p_i = bf16(e_i * r). */
static int g_softmax_mode = ORACLE_SOFTMAX_F32;

int oracle_set_softmax_precision(int mode) {
    if (mode != ORACLE_SOFTMAX_F32 && mode != ORACLE_SOFTMAX_BF16) return -1;
    const int prev = g_softmax_mode;
    g_softmax_mode = mode;
    return prev;
}

static void softmax_row_f(const float* l, int64_t n, float* ex, uint16_t* p) {
    float m = -INFINITY;
    for (int64_t i = 0; i < n; ++i) m = l[i] > m ? l[i] : m;
    if (g_softmax_mode == ORACLE_SOFTMAX_BF16) {
        float s = 0.0f;
        for (int64_t i = 0; i < n; ++i) {
            ex[i] = rbf(oracle_exp(rbf(l[i] - m)));
            s = rbf(s + ex[i]);
        }
        const float r = rbf(1.0f / s);
        for (int64_t i = 0; i < n; ++i) p[i] = f2bf(ex[i] * r);
        return;
    }
    for (int64_t i = 0; i < n; ++i) ex[i] = oracle_exp(l[i] - m);
    const float s = sum_canonical(ex, n);
    for (int64_t i = 0; i < n; ++i) p[i] = f2bf(ex[i] / s);
}

int oracle_softmax_rows(const uint16_t* logits, int64_t rows, int64_t n, uint16_t* probs) {
    float* l = (float*)malloc(sizeof(float) * n);
    float* ex = (float*)malloc(sizeof(float) * n);
    if (!l || !ex) {
        free(l);
        free(ex);
        return -10;
    }
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t i = 0; i < n; ++i) l[i] = bf2f(logits[r * n + i]);
        softmax_row_f(l, n, ex, probs + r * n);
    }
    free(l);
    free(ex);
    return 0;
}

/*
 * Top-k of one row of bf16 keys by (key desc, index asc) — the order the reference's
 * host validator uses (sort_top_pairs / select_top_k, qwen3_moe_python_port.rs:89-93,
 * 491-510; lfm2_moe_python_port.rs:595). The returned set is what
 * argpartition(-p, k-1)[:, :k] (Qwen, :438-440) or argpartition(p, E-k)[:, E-k:]
 * (LFM2, :579-583) selects; indices are listed in that same order. NaN keys (a
 * token with a non-finite activation) rank after every other key, by index among
 * themselves.
 */
static void topk_row(const uint16_t* key, int64_t E, int k, uint32_t* sel) {
    for (int j = 0; j < k; ++j) {
        int64_t best = -1;
        float bv = 0.0f;
        for (int64_t e = 0; e < E; ++e) {
            int taken = 0;
            for (int jj = 0; jj < j; ++jj)
                if (sel[jj] == (uint32_t)e) taken = 1;
            if (taken) continue;
            const float v = bf2f(key[e]);
            /* NaN keys rank after every other key, NaN among NaN by index (e ascends,
             * so an earlier NaN is kept): a total order, k distinct valid indices */
            const int better = best < 0 || (isnan(bv) && !isnan(v)) || (!isnan(v) && v > bv);
            if (better) {
                best = e;
                bv = v;
            }
        }
        sel[j] = (uint32_t)best;
    }
}

int oracle_topk_rows(const uint16_t* keys, int64_t rows, int64_t E, int k, uint32_t* idx) {
    if (k <= 0 || k > E) return -6;
    for (int64_t r = 0; r < rows; ++r) topk_row(keys + r * E, E, k, idx + r * k);
    return 0;
}

/*
 * Router (R1-R4): logits = quantized_matmul(x, Wr) (linear.rs:117-128) then
 *   SOFTMAX:             p = softmax(logits)                (qwen3_moe_python_port.rs:437)
 *   SOFTMAX_BIAS:        p = softmax(bf16(logits + bias))   (lfm2_moe_python_port.rs:559-574)
 *   SIGMOID_BIAS_SELECT: s = bf16(sigmoid(logits)); selection key bf16(s + bias),
 *                        weights taken from s (LFM2-style sigmoid routing)
 * top-k as topk_row, weights = take_along_axis(p, idx) (:441), and when
 * norm_topk_prob: w = bf16(w / bf16(sum_j w_j)) with the sum in fp32 over j in order
 * (:442-445; lfm2_moe_python_port.rs:682-686).
 */
int oracle_route(const oracle_block_config* cfg, const oracle_block_weights* wt,
                 const uint16_t* x, int64_t T, uint32_t* idx, uint16_t* weights,
                 uint16_t* logits_out, uint16_t* scores_out, int nthreads) {
    const int64_t E = cfg->num_experts, H = cfg->hidden;
    const int k = cfg->top_k;
    if (k <= 0 || k > E || k > 64) return -6;
    if (cfg->scoring != ORACLE_SCORING_SOFTMAX && !wt->expert_bias) return -7;
    if (T == 0) return 0;
    uint16_t* logits = (uint16_t*)malloc(sizeof(uint16_t) * T * E + 2);
    if (!logits) return -10;
    int rc = oracle_qmm(x, T, H, wt->router.w, wt->router.s, wt->router.b, E, cfg->group_size,
                        cfg->bits, logits, nthreads);
    if (rc) {
        free(logits);
        return rc;
    }
    if (logits_out) memcpy(logits_out, logits, sizeof(uint16_t) * T * E);
    float* l = (float*)malloc(sizeof(float) * E);
    float* ex = (float*)malloc(sizeof(float) * E);
    uint16_t* val = (uint16_t*)malloc(sizeof(uint16_t) * E);
    uint16_t* key = (uint16_t*)malloc(sizeof(uint16_t) * E);
    for (int64_t t = 0; t < T; ++t) {
        const uint16_t* lr = logits + t * E;
        if (cfg->scoring == ORACLE_SCORING_SOFTMAX) {
            for (int64_t e = 0; e < E; ++e) l[e] = bf2f(lr[e]);
            softmax_row_f(l, E, ex, val);
            memcpy(key, val, sizeof(uint16_t) * E);
        } else if (cfg->scoring == ORACLE_SCORING_SOFTMAX_BIAS) {
            for (int64_t e = 0; e < E; ++e) l[e] = rbf(bf2f(lr[e]) + bf2f(wt->expert_bias[e]));
            softmax_row_f(l, E, ex, val);
            memcpy(key, val, sizeof(uint16_t) * E);
        } else {
            for (int64_t e = 0; e < E; ++e) {
                val[e] = f2bf(oracle_sigmoid(bf2f(lr[e])));
                key[e] = f2bf(bf2f(val[e]) + bf2f(wt->expert_bias[e]));
            }
        }
        if (scores_out) memcpy(scores_out + t * E, val, sizeof(uint16_t) * E);
        uint32_t* sel = idx + t * k;
        topk_row(key, E, k, sel);
        float wsel[64];
        for (int j = 0; j < k; ++j) wsel[j] = bf2f(val[sel[j]]);
        if (cfg->norm_topk_prob) {
            float d = 0.0f;
            for (int j = 0; j < k; ++j) d = d + wsel[j];
            d = rbf(d);
            for (int j = 0; j < k; ++j) wsel[j] = rbf(wsel[j] / d);
        }
        for (int j = 0; j < k; ++j) weights[t * k + j] = f2bf(wsel[j]);
    }
    free(l);
    free(ex);
    free(val);
    free(key);
    free(logits);
    return 0;
}

/*
 * Per-expert grouping of the T*k (token, slot) pairs p = t*k + j: offsets[e] is the
 * exclusive prefix sum of the counts and perm lists, expert by expert, the pairs in
 * ascending p. This is the grouping MLX's gather_qmm forms internally when
 * sorted_indices=false (qwen3_moe_python_port.rs:312); the CUDA path must
 * reproduce it bit for bit.
 */
int oracle_group_by_expert(int64_t T, int k, int E, const uint32_t* idx, int32_t* offsets,
                           uint32_t* perm) {
    const int64_t P = T * k;
    for (int e = 0; e <= E; ++e) offsets[e] = 0;
    for (int64_t p = 0; p < P; ++p) {
        if (idx[p] >= (uint32_t)E) return -5;
        offsets[idx[p] + 1]++;
    }
    for (int e = 0; e < E; ++e) offsets[e + 1] += offsets[e];
    int32_t* cur = (int32_t*)malloc(sizeof(int32_t) * (E + 1));
    if (!cur) return -10;
    memcpy(cur, offsets, sizeof(int32_t) * (E + 1));
    for (int64_t p = 0; p < P; ++p) perm[cur[idx[p]]++] = (uint32_t)p;
    free(cur);
    return 0;
}

/* ------------------------------------------------------------------------- */
/* RMSNorm                                                                    */
/* ------------------------------------------------------------------------- */

typedef struct {
    const uint16_t *x, *w;
    float eps;
    int64_t dim;
    uint16_t* out;
} rms_ctx;

static void rms_rows(int64_t r0, int64_t r1, void* vctx, void* scratch) {
    const rms_ctx* c = (const rms_ctx*)vctx;
    const int64_t dim = c->dim;
    for (int64_t r = r0; r < r1; ++r) {
        const uint16_t* xr = c->x + r * dim;
        float acc[32];
        for (int l = 0; l < 32; ++l) {
            float a = 0.0f;
            for (int64_t ch = l; ch < dim / 8; ch += 32)
                for (int j = 0; j < 8; ++j) {
                    const float v = bf2f(xr[8 * ch + j]);
                    a = fmaf(v, v, a);
                }
            acc[l] = a;
        }
        const float ss = butterfly32(acc);
        const float rr = 1.0f / sqrtf(ss / (float)dim + c->eps);
        for (int64_t i = 0; i < dim; ++i)
            c->out[r * dim + i] = f2bf(rbf(bf2f(xr[i]) * rr) * bf2f(c->w[i]));
    }
}

/*
 * y = bf16(bf16(x * r) * w), r = 1 / sqrt(ss / dim + eps) (IEEE sqrt and divide),
 * ss = sum x^2 in the canonical order over chunks of 8: lane l owns chunks
 * l, l+32, ... and accumulates acc = fmaf(x, x, acc) element by element, then the
 * xor butterfly. mlx_fast_rms_norm via RmsNorm::forward (crates/mlx-nn/src/rms_norm.rs:30-34).
 */
int oracle_rms_norm(const uint16_t* x, const uint16_t* w, float eps, int64_t rows, int64_t dim,
                    uint16_t* out, int nthreads) {
    if (dim <= 0 || dim % 8 != 0) return -3;
    rms_ctx c = {x, w, eps, dim, out};
    parallel_for(rows, 16, nthreads, 0, rms_rows, &c);
    return 0;
}

/* ------------------------------------------------------------------------- */
/* Block                                                                      */
/* ------------------------------------------------------------------------- */

/* h = bf16(bf16(g * bf16(sigmoid(g))) * u) — SwitchGlu::forward (:355) and
 * SharedExpert::forward (:385-390). */
static void swiglu_bf16(const uint16_t* g, const uint16_t* u, int64_t n, uint16_t* h) {
    for (int64_t i = 0; i < n; ++i) {
        const float gv = bf2f(g[i]);
        const float sg = rbf(oracle_sigmoid(gv));
        const float a = rbf(gv * sg);
        h[i] = f2bf(a * bf2f(u[i]));
    }
}

int oracle_swiglu(const uint16_t* g, const uint16_t* u, int64_t n, uint16_t* h) {
    if (n < 0) return -1;
    swiglu_bf16(g, u, n, h);
    return 0;
}

typedef struct {
    const uint16_t *y, *wsel, *ys, *gl;
    int k, has_shared, has_gate;
    int64_t H;
    uint16_t* out;
} comb_ctx;

/* out[t] = bf16(sum_j bf16(y[t,j] * w[t,j])) with the fp32 sum over j in order
 * (expert_out.multiply(score).sum_axis(1), qwen3_moe_python_port.rs:471-472), then
 * out = bf16(out + bf16(shared * bf16(sigmoid(gate)))) (:477-484). */
static void comb_rows(int64_t t0, int64_t t1, void* vctx, void* scratch) {
    const comb_ctx* c = (const comb_ctx*)vctx;
    const int64_t H = c->H;
    const int k = c->k;
    for (int64_t t = t0; t < t1; ++t) {
        const float gate = (c->has_shared && c->has_gate) ? rbf(oracle_sigmoid(bf2f(c->gl[t]))) : 1.0f;
        for (int64_t h = 0; h < H; ++h) {
            float a = 0.0f;
            for (int j = 0; j < k; ++j)
                a = a + rbf(bf2f(c->y[(t * k + j) * H + h]) * bf2f(c->wsel[t * k + j]));
            uint16_t o = f2bf(a);
            if (c->has_shared) {
                float v = bf2f(c->ys[t * H + h]);
                if (c->has_gate) v = rbf(v * gate);
                o = f2bf(bf2f(o) + v);
            }
            c->out[t * H + h] = o;
        }
    }
}

int oracle_block_forward(const oracle_block_config* cfg, const oracle_block_weights* wt,
                         const uint16_t* x, int64_t T, uint16_t* out, uint32_t* idx_out,
                         uint16_t* weights_out, int nthreads) {
    const int64_t H = cfg->hidden, E = cfg->num_experts, I = cfg->moe_inter, Is = cfg->shared_inter;
    const int k = cfg->top_k, gs = cfg->group_size, bits = cfg->bits;
    if (T == 0) return 0;
    const int64_t P = T * k;
    int rc = 0;
    uint32_t* idx = (uint32_t*)malloc(sizeof(uint32_t) * P);
    uint16_t* wsel = (uint16_t*)malloc(sizeof(uint16_t) * P);
    uint16_t* g = (uint16_t*)malloc(sizeof(uint16_t) * P * I);
    uint16_t* u = (uint16_t*)malloc(sizeof(uint16_t) * P * I);
    uint16_t* y = (uint16_t*)malloc(sizeof(uint16_t) * P * H);
    uint16_t* ys = NULL;
    uint16_t* gl = NULL;
    if (!idx || !wsel || !g || !u || !y) {
        rc = -10;
        goto done;
    }
    rc = oracle_route(cfg, wt, x, T, idx, wsel, NULL, NULL, nthreads);
    if (rc) goto done;
    /* SwitchGlu: up, gate, then down over the hidden (SwitchGlu::forward :352-359). */
    rc = oracle_gather_qmm(x, H, k, NULL, wt->up.w, wt->up.s, wt->up.b, E, I, idx, P, gs, bits, u,
                           nthreads);
    if (rc) goto done;
    rc = oracle_gather_qmm(x, H, k, NULL, wt->gate.w, wt->gate.s, wt->gate.b, E, I, idx, P, gs,
                           bits, g, nthreads);
    if (rc) goto done;
    swiglu_bf16(g, u, P * I, g);
    rc = oracle_gather_qmm(g, I, 1, NULL, wt->down.w, wt->down.s, wt->down.b, E, H, idx, P, gs,
                           bits, y, nthreads);
    if (rc) goto done;
    if (Is > 0) {
        /* SharedExpert::forward (:385-390) and shared_expert_gate (:477-479). */
        uint16_t* sg = (uint16_t*)malloc(sizeof(uint16_t) * T * Is);
        uint16_t* su = (uint16_t*)malloc(sizeof(uint16_t) * T * Is);
        ys = (uint16_t*)malloc(sizeof(uint16_t) * T * H);
        gl = (uint16_t*)malloc(sizeof(uint16_t) * T);
        if (!sg || !su || !ys || !gl) rc = -10;
        if (!rc)
            rc = oracle_qmm(x, T, H, wt->shared_gate.w, wt->shared_gate.s, wt->shared_gate.b, Is,
                            gs, bits, sg, nthreads);
        if (!rc)
            rc = oracle_qmm(x, T, H, wt->shared_up.w, wt->shared_up.s, wt->shared_up.b, Is, gs,
                            bits, su, nthreads);
        if (!rc) {
            swiglu_bf16(sg, su, T * Is, sg);
            rc = oracle_qmm(sg, T, Is, wt->shared_down.w, wt->shared_down.s, wt->shared_down.b, H,
                            gs, bits, ys, nthreads);
        }
        if (!rc && cfg->has_shared_gate)
            rc = oracle_qmm(x, T, H, wt->shared_expert_gate.w, wt->shared_expert_gate.s,
                            wt->shared_expert_gate.b, 1, gs, bits, gl, nthreads);
        free(sg);
        free(su);
        if (rc) goto done;
    }
    {
        comb_ctx c = {y, wsel, ys, gl, k, Is > 0, cfg->has_shared_gate, H, out};
        parallel_for(T, 8, nthreads, 0, comb_rows, &c);
    }
    if (idx_out) memcpy(idx_out, idx, sizeof(uint32_t) * P);
    if (weights_out) memcpy(weights_out, wsel, sizeof(uint16_t) * P);
done:
    free(idx);
    free(wsel);
    free(g);
    free(u);
    free(y);
    free(ys);
    free(gl);
    return rc;
}

/* ------------------------------------------------------------------------- */
/* Gemma4 MoE block (crates/mlx-models/src/gemma4.rs)                        */
/* ------------------------------------------------------------------------- */

/* f32 rows in lane-major order (x_to_lane_major for f32 input). */
static void xf_to_lane_major(const float* x, int64_t K, float* xt) {
    const int64_t nr = lane_rounds(K), nchunks = K / 32;
    for (int64_t r = 0; r < nr; ++r)
        for (int j = 0; j < 32; ++j)
            for (int l = 0; l < 32; ++l) {
                const int64_t c = l + 32 * r;
                xt[(r * 32 + j) * 32 + l] = (c < nchunks) ? x[32 * c + j] : 0.0f;
            }
}

typedef struct {
    const float* xt;
    const uint32_t* w;
    const uint16_t *s, *b;
    float* out;
    const int64_t *cnt, *order;
    int64_t x_repeat, K, N;
    int gs, bits;
    int64_t nr, L, wpr, gpr;
} gqmmf_ctx;

static void gqmmf_rows(int64_t r0, int64_t r1, void* vctx, void* scratch) {
    const gqmmf_ctx* c = (const gqmmf_ctx*)vctx;
    float* wt = (float*)scratch;
    for (int64_t row = r0; row < r1; ++row) {
        const int64_t e = row / c->N, n = row % c->N;
        if (c->cnt[e + 1] == c->cnt[e]) continue;
        w_to_lane_major(c->w + row * c->wpr, c->s + row * c->gpr, c->b ? c->b + row * c->gpr : NULL,
                        c->K, c->gs, c->bits, wt);
        for (int64_t p = c->cnt[e]; p < c->cnt[e + 1]; ++p) {
            const int64_t i = c->order[p];
            c->out[i * c->N + n] = dot_lane_major(c->xt + (i / c->x_repeat) * c->L, wt, c->nr);
        }
    }
}

/* out[i, n] (f32, not rounded) = dot(x[i / x_repeat] (f32), W[rhs[i], n]): gather_qmm with
 * an f32 x, whose output MLX keeps in f32 (the Gemma4 down projection, gemma4.rs:1050). */
static int gather_qmm_f32(const float* x, int64_t K, int64_t x_repeat, const uint32_t* w, const uint16_t* s,
                          const uint16_t* b, int64_t E, int64_t N, const uint32_t* rhs, int64_t batch, int gs,
                          int bits, float* out, int nthreads) {
    int rc = check_q(K, gs, bits);
    if (rc) return rc;
    const int64_t xrows = (batch + x_repeat - 1) / x_repeat;
    const int64_t nr = lane_rounds(K), L = nr * 32 * 32;
    float* xt = (float*)malloc(sizeof(float) * L * xrows);
    int64_t* cnt = (int64_t*)calloc((size_t)E + 1, sizeof(int64_t));
    int64_t* order = (int64_t*)malloc(sizeof(int64_t) * batch);
    int64_t* cur = (int64_t*)malloc(sizeof(int64_t) * (E + 1));
    if (!xt || !cnt || !order || !cur) {
        free(xt);
        free(cnt);
        free(order);
        free(cur);
        return -10;
    }
    for (int64_t r = 0; r < xrows; ++r) xf_to_lane_major(x + r * K, K, xt + r * L);
    for (int64_t i = 0; i < batch; ++i) cnt[rhs[i] + 1]++;
    for (int64_t e = 0; e < E; ++e) cnt[e + 1] += cnt[e];
    memcpy(cur, cnt, sizeof(int64_t) * (E + 1));
    for (int64_t i = 0; i < batch; ++i) order[cur[rhs[i]]++] = i;
    gqmmf_ctx c = {xt, w, s, b, out, cnt, order, x_repeat, K, N, gs, bits, nr, L, K * bits / 32, K / gs};
    parallel_for(E * N, 4, nthreads, sizeof(float) * L, gqmmf_rows, &c);
    free(xt);
    free(cnt);
    free(order);
    free(cur);
    return 0;
}

/* Top-k of f32 keys in the order of topk_row (key desc, index asc, NaN last). */
static void topk_row_f32(const float* key, int64_t E, int k, uint32_t* sel) {
    for (int j = 0; j < k; ++j) {
        int64_t best = -1;
        float bv = 0.0f;
        for (int64_t e = 0; e < E; ++e) {
            int taken = 0;
            for (int jj = 0; jj < j; ++jj)
                if (sel[jj] == (uint32_t)e) taken = 1;
            if (taken) continue;
            const float v = key[e];
            const int better = best < 0 || (isnan(bv) && !isnan(v)) || (!isnan(v) && v > bv);
            if (better) {
                best = e;
                bv = v;
            }
        }
        sel[j] = (uint32_t)best;
    }
}

/*
 * The Gemma4 SparseMoeBlock::forward (gemma4.rs:1063-1085) op by op:
 *   Router::forward (:906-936): h = fast_rms_norm(x, ones, 1e-6) (bf16), then
 *     h * from_float(hidden^-0.5) * scale — from_float is a 0-d f32 array, so h becomes
 *     f32 (the 0-d array is f32: crates/mlx-core/src/array.rs:82-87) and the router
 *     continues in f32: logits = quantized_matmul(h) (f32), probs = softmax(logits) (f32),
 *     top-k indices of -logits (argpartition), w = probs[idx] / sum_j probs[idx_j],
 *     w *= per_expert_scale[idx];
 *   SwitchGlu::forward (:1045-1052): up = gather_qmm(x) and gate = gather_qmm(x) (bf16),
 *     hidden = gelu_approx(gate) * up in f32 (gelu_approx :308-322 multiplies by 0-d f32
 *     arrays: 0.5 * (g * (1 + tanh(sqrt(2/pi) * (g + 0.044715 * g^3)))), power as powf),
 *     y = gather_qmm(hidden) in f32;
 *   the block: out = sum_j y_j * w_j (f32 products, sum in j order).
 * out [T, H] f32; idx_out [T, k] and weights_out [T, k] (f32) optional.
 */
int oracle_gemma4_block_forward(const oracle_block_config* cfg, const oracle_block_weights* wt,
                                const uint16_t* router_scale, const uint16_t* per_expert_scale,
                                const uint16_t* x, int64_t T, float* out, uint32_t* idx_out,
                                float* weights_out, int nthreads) {
    const int64_t H = cfg->hidden, E = cfg->num_experts, I = cfg->moe_inter;
    const int k = cfg->top_k, gs = cfg->group_size, bits = cfg->bits;
    if (T == 0) return 0;
    if (k <= 0 || k > E) return -6;
    const int64_t P = T * k;
    int rc = 0;
    uint16_t* ones = (uint16_t*)malloc(sizeof(uint16_t) * H);
    uint16_t* hn = (uint16_t*)malloc(sizeof(uint16_t) * T * H);
    float* hf = (float*)malloc(sizeof(float) * T * H);
    float* logits = (float*)malloc(sizeof(float) * T * E);
    float* ex = (float*)malloc(sizeof(float) * E);
    uint32_t* idx = (uint32_t*)malloc(sizeof(uint32_t) * P);
    float* w = (float*)malloc(sizeof(float) * P);
    uint16_t* g = (uint16_t*)malloc(sizeof(uint16_t) * P * I);
    uint16_t* u = (uint16_t*)malloc(sizeof(uint16_t) * P * I);
    float* hid = (float*)malloc(sizeof(float) * P * I);
    float* y = (float*)malloc(sizeof(float) * P * H);
    if (!ones || !hn || !hf || !logits || !ex || !idx || !w || !g || !u || !hid || !y) {
        rc = -10;
        goto gdone;
    }
    for (int64_t i = 0; i < H; ++i) ones[i] = 0x3f80; /* bf16 1.0 */
    rc = oracle_rms_norm(x, ones, 1e-6f, T, H, hn, nthreads);
    if (rc) goto gdone;
    {
        const float root = (float)(1.0 / sqrt((double)H)); /* (hidden_size as f32).powf(-0.5) */
        for (int64_t i = 0; i < T * H; ++i) hf[i] = (bf2f(hn[i]) * root) * bf2f(router_scale[i % H]);
    }
    {
        /* logits[t, e] = canonical dot of the f32 row with router row e */
        /* as a gather_qmm of the T*E pairs (t, e) over "experts" of one row each: pair
         * i = t*E + e reads f32 row t (x_repeat = E) against router row e */
        uint32_t* rr = (uint32_t*)malloc(sizeof(uint32_t) * T * E);
        if (!rr) {
            rc = -10;
            goto gdone;
        }
        for (int64_t i = 0; i < T * E; ++i) rr[i] = (uint32_t)(i % E);
        rc = gather_qmm_f32(hf, H, E, wt->router.w, wt->router.s, wt->router.b, E, 1, rr, T * E, gs, bits,
                            logits, nthreads);
        free(rr);
        if (rc) goto gdone;
    }
    for (int64_t t = 0; t < T; ++t) {
        const float* l = logits + t * E;
        float m = -INFINITY;
        for (int64_t e = 0; e < E; ++e) m = l[e] > m ? l[e] : m;
        for (int64_t e = 0; e < E; ++e) ex[e] = oracle_exp(l[e] - m);
        const float s = sum_canonical(ex, E);
        topk_row_f32(l, E, k, idx + t * k);
        float d = 0.0f;
        for (int j = 0; j < k; ++j) d = d + ex[idx[t * k + j]] / s;
        for (int j = 0; j < k; ++j) {
            const uint32_t e = idx[t * k + j];
            w[t * k + j] = ((ex[e] / s) / d) * bf2f(per_expert_scale[e]);
        }
    }
    rc = oracle_gather_qmm(x, H, k, NULL, wt->up.w, wt->up.s, wt->up.b, E, I, idx, P, gs, bits, u, nthreads);
    if (rc) goto gdone;
    rc = oracle_gather_qmm(x, H, k, NULL, wt->gate.w, wt->gate.s, wt->gate.b, E, I, idx, P, gs, bits, g,
                           nthreads);
    if (rc) goto gdone;
    {
        const float kS2P = sqrtf(2.0f / 3.14159265358979323846f); /* (2.0f32 / PI).sqrt() */
        const float kC = 0.044715f;
        for (int64_t i = 0; i < P * I; ++i) {
            const float gv = bf2f(g[i]);
            const float x3 = powf(gv, 3.0f);
            const float inner = (gv + x3 * kC) * kS2P;
            const float gate = 1.0f + tanhf(inner);
            hid[i] = (0.5f * (gv * gate)) * bf2f(u[i]);
        }
    }
    rc = gather_qmm_f32(hid, I, 1, wt->down.w, wt->down.s, wt->down.b, E, H, idx, P, gs, bits, y, nthreads);
    if (rc) goto gdone;
    for (int64_t t = 0; t < T; ++t)
        for (int64_t h = 0; h < H; ++h) {
            float acc = 0.0f;
            for (int j = 0; j < k; ++j) acc = acc + y[(t * k + j) * H + h] * w[t * k + j];
            out[t * H + h] = acc;
        }
    if (idx_out) memcpy(idx_out, idx, sizeof(uint32_t) * P);
    if (weights_out) memcpy(weights_out, w, sizeof(float) * P);
gdone:
    free(ones);
    free(hn);
    free(hf);
    free(logits);
    free(ex);
    free(idx);
    free(w);
    free(g);
    free(u);
    free(hid);
    free(y);
    return rc;
}

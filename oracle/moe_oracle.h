/*
 * moe_oracle.h — CPU oracle for the mlx-rs device-side MoE (SwitchGLU) block.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA path: only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm may
 * load it. The product library never links or calls it.
 *
 * PARITY UNPINNED. The reference (paulm17/mlx-rs) delegates every operation on this
 * path to the external MLX C++ library through mlx-c (crates/mlx-sys/build.rs:6-13);
 * MLX is not vendored, its version is not pinned (no Cargo.lock entry, /mlx is
 * git-ignored), and neither MLX nor a Rust toolchain is available here, so the
 * reference cannot be run. The reference's tests hold no golden vectors for
 * gather_qmm / quantized_matmul / the MoE block. This oracle therefore restates
 * the reference block op by op (file:line cited per function) with the rounding
 * points of an MLX bf16 graph (every op rounds its result to bf16) and fixes the
 * choices MLX leaves implementation-defined:
 *   - matmul accumulation: fp32, in the canonical "32-lane" order documented at
 *     oracle_dot_canonical();
 *   - affine dequantisation: w = fmaf(scale, q, bias) in fp32;
 *   - softmax: fp32 internally (max, exp, canonical sum, divide), bf16 result;
 *     oracle_set_softmax_precision(ORACLE_SOFTMAX_BF16) switches the routing softmax
 *     to bf16 intermediates (MLX's precise=false may compute in the input type);
 *   - exp: oracle_exp(), Cody-Waite range reduction + degree-7 Taylor polynomial;
 *   - argpartition ties: (value desc, index asc), the rule the reference's own
 *     host validator uses (qwen3_moe_python_port.rs:89-93, 491-510);
 *   - reductions over k (renorm denominator, weighted sum): fp32, in index order.
 * The top-k selector is cross-checked against a restatement of the reference's
 * host selector select_top_k (qwen3_moe_python_port.rs:491-510) in tests/.
 *
 * bf16 values are passed as uint16_t bit patterns.
 */
#ifndef MOE_ORACLE_H
#define MOE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Scoring modes (R2 of the block). */
enum {
    ORACLE_SCORING_SOFTMAX = 0,             /* qwen3_moe_python_port.rs:437 */
    ORACLE_SCORING_SOFTMAX_BIAS = 1,        /* lfm2_moe_python_port.rs:559-574 */
    ORACLE_SCORING_SIGMOID_BIAS_SELECT = 2  /* LFM2 sigmoid scores, bias for selection only */
};

typedef struct {
    int32_t hidden;          /* H */
    int32_t num_experts;     /* E */
    int32_t top_k;           /* k */
    int32_t moe_inter;       /* I */
    int32_t shared_inter;    /* Is, 0 = no shared expert */
    int32_t scoring;         /* ORACLE_SCORING_* */
    int32_t norm_topk_prob;  /* renormalise the selected weights */
    int32_t has_shared_gate; /* sigmoid shared_expert_gate present */
    int32_t group_size;
    int32_t bits;
} oracle_block_config;

typedef struct {
    const uint32_t* w;  /* [rows, K*bits/32] packed */
    const uint16_t* s;  /* [rows, K/gs] bf16 */
    const uint16_t* b;  /* [rows, K/gs] bf16, may be NULL */
} oracle_qweight;

typedef struct {
    oracle_qweight router;       /* [E, H] */
    const uint16_t* expert_bias; /* [E] bf16, may be NULL */
    oracle_qweight gate;         /* [E, I, H] */
    oracle_qweight up;           /* [E, I, H] */
    oracle_qweight down;         /* [E, H, I] */
    oracle_qweight shared_gate;  /* [Is, H] */
    oracle_qweight shared_up;    /* [Is, H] */
    oracle_qweight shared_down;  /* [H, Is] */
    oracle_qweight shared_expert_gate; /* [1, H] */
} oracle_block_weights;

float oracle_exp(float x);

/* Internal precision of the routing softmax (process-wide; returns the previous mode, or
 * -1 for an unknown mode). ORACLE_SOFTMAX_F32 is the default. */
#define ORACLE_SOFTMAX_F32 0
#define ORACLE_SOFTMAX_BF16 1
int oracle_set_softmax_precision(int mode);
float oracle_sigmoid(float x);
uint16_t oracle_f32_to_bf16(float x);

/* Canonical fp32 dot product of x (bf16) with one quantized row; returns fp32. */
float oracle_dot_canonical(const uint16_t* x, const uint32_t* wrow, const uint16_t* srow,
                           const uint16_t* brow, int64_t K, int gs, int bits);

int oracle_qmm(const uint16_t* x, int64_t M, int64_t K, const uint32_t* w, const uint16_t* s,
               const uint16_t* b, int64_t N, int gs, int bits, uint16_t* out, int nthreads);

int oracle_gather_qmm(const uint16_t* x, int64_t K, int64_t x_repeat, const uint32_t* lhs,
                      const uint32_t* w, const uint16_t* s, const uint16_t* b, int64_t E,
                      int64_t N, const uint32_t* rhs, int64_t batch, int gs, int bits,
                      uint16_t* out, int nthreads);

int oracle_softmax_rows(const uint16_t* logits, int64_t rows, int64_t n, uint16_t* probs);

/* Top-k of each row of bf16 keys by (key desc, index asc). */
int oracle_topk_rows(const uint16_t* keys, int64_t rows, int64_t E, int k, uint32_t* idx);

int oracle_route(const oracle_block_config* cfg, const oracle_block_weights* wt,
                 const uint16_t* x, int64_t T, uint32_t* idx, uint16_t* weights,
                 uint16_t* logits_out, uint16_t* scores_out, int nthreads);

int oracle_group_by_expert(int64_t T, int k, int E, const uint32_t* idx, int32_t* offsets,
                           uint32_t* perm);

int oracle_rms_norm(const uint16_t* x, const uint16_t* w, float eps, int64_t rows, int64_t dim,
                    uint16_t* out, int nthreads);

/* h = bf16(bf16(g * bf16(sigmoid(g))) * u) elementwise (the SwitchGLU activation). */
int oracle_swiglu(const uint16_t* g, const uint16_t* u, int64_t n, uint16_t* h);

int oracle_block_forward(const oracle_block_config* cfg, const oracle_block_weights* wt,
                         const uint16_t* x, int64_t T, uint16_t* out, uint32_t* idx_out,
                         uint16_t* weights_out, int nthreads);

/* The Gemma4 MoE block (gemma4.rs:1063-1085): f32 router input, f32 logits, top-k by
 * logit, f32 weights softmax[idx] / sum * per_expert_scale[idx], GELU-tanh SwitchGLU with
 * an f32 hidden and f32 down outputs; out [T, H] f32. shared_inter is ignored (none). */
int oracle_gemma4_block_forward(const oracle_block_config* cfg, const oracle_block_weights* wt,
                                const uint16_t* router_scale, const uint16_t* per_expert_scale,
                                const uint16_t* x, int64_t T, float* out, uint32_t* idx_out,
                                float* weights_out, int nthreads);

#ifdef __cplusplus
}
#endif
#endif

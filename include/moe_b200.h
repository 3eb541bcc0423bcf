/*
 * moe_b200.h — C ABI of the B200 (sm_100a) MoE / SwitchGLU block.
 *
 * This library stands in for mlx-sys (crates/mlx-sys, bindgen over mlx-c) on the
 * device-side MoE path of paulm17/mlx-rs. Each entry point names the reference
 * interface it replaces (paths relative to the reference project).
 *
 * Conventions (mirroring crates/mlx-core/src/array.rs:43-49, where every mlx-c call
 * returns an int and rc != 0 becomes Error::Mlx("<fn> failed (rc=N)")):
 *   - every function returns MOE_OK (0) or a positive MOE_ERR_* code and never
 *     aborts; moe_last_error() gives a one-line message for the last failure on
 *     that context;
 *   - all tensor arguments are DEVICE pointers owned by the caller, row-major and
 *     contiguous; bf16 tensors are passed as void* (2-byte elements);
 *   - optional arrays are NULL (as mlx-c's null ctx, crates/mlx-core/src/ops.rs:852-869);
 *   - calls are asynchronous and ordered on the context's stream (MLX's lazy graph
 *     + default stream, array.rs:28-40); the caller synchronises;
 *   - scratch memory is owned by the context and grows on demand (moe_ctx_reserve
 *     sizes it up front); a context must not be used by two threads at once.
 *
 * Quantized weights use the MLX affine layout (mlx_quantize, mode "affine"):
 *   w      [rows, K * bits / 32] uint32, element e of a row is bits (e % (32/bits))*bits
 *          of word e / (32/bits), lowest bits first;
 *   scales [rows, K / group_size] bf16;  biases [rows, K / group_size] bf16 or NULL;
 *   dequantised value = scale * q + bias.
 * The CUDA kernels implement bits = 4 with group_size = 64 (the configuration of
 * every model on this path); other valid MLX values return MOE_ERR_UNSUPPORTED.
 */
#ifndef MOE_B200_H
#define MOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MOE_B200_ABI_VERSION 1

enum moe_status {
    MOE_OK = 0,
    MOE_ERR_INVALID = 1,     /* bad argument or shape */
    MOE_ERR_UNSUPPORTED = 2, /* valid for MLX, not implemented by these kernels */
    MOE_ERR_CUDA = 3,        /* a CUDA runtime call or kernel launch failed */
    MOE_ERR_NO_MEMORY = 4,   /* scratch allocation failed */
    MOE_ERR_TIMEOUT = 5      /* a bounded device-side wait gave up */
};

/* Router scoring (R2). */
enum moe_scoring {
    /* probs = softmax(logits): SparseMoeBlock::forward, qwen3_moe_python_port.rs:437 */
    MOE_SCORING_SOFTMAX = 0,
    /* probs = softmax(logits + expert_bias): MoeFeedForward::forward,
     * lfm2_moe_python_port.rs:559-574 */
    MOE_SCORING_SOFTMAX_BIAS = 1,
    /* s = sigmoid(logits), select on s + expert_bias, weights from s (LFM2 sigmoid routing) */
    MOE_SCORING_SIGMOID_BIAS_SELECT = 2
};

/* Block shape and options; the fields of Qwen3MoePythonPortConfig
 * (qwen3_moe_python_port.rs:12-41) and Lfm2MoeConfig that the block reads. */
typedef struct moe_block_config {
    int32_t hidden;          /* H (hidden_size) */
    int32_t num_experts;     /* E (num_experts), 1..512 */
    int32_t top_k;           /* k (num_experts_per_tok), 1..32 */
    int32_t moe_inter;       /* I (moe_intermediate_size) */
    int32_t shared_inter;    /* Is (shared_expert_intermediate_size), 0 = none */
    int32_t scoring;         /* enum moe_scoring */
    int32_t norm_topk_prob;  /* renormalise the k selected weights to sum 1 */
    int32_t has_shared_gate; /* sigmoid shared_expert_gate [1, H] present */
    int32_t group_size;      /* quantization.group_size (64) */
    int32_t bits;            /* quantization.bits (4) */
} moe_block_config;

/* One quantized matrix (a quantized mlx_nn::Linear without bias, linear.rs:117-139). */
typedef struct moe_qweight {
    const uint32_t* w;
    const void* scales;
    const void* biases; /* may be NULL */
} moe_qweight;

/* Device weights of one block: the stacked SwitchLinear tensors
 * (qwen3_moe_python_port.rs:241-309, [E, N, K*bits/32]) or the pre-stacked
 * switch_mlp tensors (lfm2_moe_python_port.rs:426-460). */
typedef struct moe_block_weights {
    moe_qweight router;             /* gate / router Linear: [E, H] */
    const void* expert_bias;        /* [E] bf16, scoring modes 1 and 2 */
    moe_qweight gate;               /* switch_mlp.gate_proj [E, I, H] */
    moe_qweight up;                 /* switch_mlp.up_proj   [E, I, H] */
    moe_qweight down;               /* switch_mlp.down_proj [E, H, I] */
    moe_qweight shared_gate;        /* shared_expert.gate_proj [Is, H] */
    moe_qweight shared_up;          /* shared_expert.up_proj   [Is, H] */
    moe_qweight shared_down;        /* shared_expert.down_proj [H, Is] */
    moe_qweight shared_expert_gate; /* shared_expert_gate [1, H] */
} moe_block_weights;

typedef struct moe_ctx moe_ctx;

/* Context on a CUDA device and stream (cudaStream_t; NULL = the legacy default
 * stream). Replaces the implicit mlx default device/stream of
 * crates/mlx-core/src/array.rs:28-40 and stream.rs. */
int moe_ctx_create(int device, void* stream, moe_ctx** out);
void moe_ctx_destroy(moe_ctx* ctx);
int moe_ctx_set_stream(moe_ctx* ctx, void* stream);
/* Pre-size the context's scratch for blocks of this shape with up to max_tokens
 * tokens, so later calls allocate nothing. */
int moe_ctx_reserve(moe_ctx* ctx, const moe_block_config* cfg, int64_t max_tokens);
/* Message of the last failed call on ctx ("" if none); valid until the next call. */
const char* moe_last_error(const moe_ctx* ctx);
int moe_abi_version(void);

/*
 * out[M, N] (bf16) = x[M, K] (bf16) . dequant(w)^T
 * Replaces Array::quantized_matmul (crates/mlx-core/src/ops.rs:592-637), i.e.
 * mlx_quantized_matmul(&out, x, w, scales, biases, transpose, gs, bits, "affine", s)
 * at ops.rs:622-633, as called by Linear::forward (crates/mlx-nn/src/linear.rs:117-128).
 * transpose must be nonzero (the only form the reference calls). M >= 32 rows (with
 * N % 128 == 0) run on the tcgen05 GEMM, fewer on the GEMV; the tcgen05 path rounds each
 * dequantised weight to bf16 before the multiply (MLX's GPU qmm does the same).
 */
int moe_quantized_matmul(moe_ctx* ctx, const void* x, int64_t M, int64_t K, const uint32_t* w,
                         const void* scales, const void* biases, int64_t N, int transpose,
                         int group_size, int bits, void* out);

/*
 * out[i, N] (bf16) = x[row(i), K] . dequant(w[rhs_indices[i]])^T for i < batch,
 * row(i) = lhs_indices ? lhs_indices[i] : i / x_repeat.
 * Replaces Array::gather_qmm (crates/mlx-core/src/ops.rs:830-891), i.e.
 * mlx_gather_qmm(&out, x, w, scales, biases, lhs, rhs, transpose, gs, bits, "affine",
 * sorted_indices, s) at ops.rs:872-886, in the one-row-per-batch-element form that
 * SwitchLinear::forward uses (qwen3_moe_python_port.rs:311-324,
 * lfm2_moe_python_port.rs:462-479): x [T,1,1,K] against rhs [T,k] is x_rows = T,
 * x_repeat = k; the down projection's x [T,k,1,I] is x_rows = T*k, x_repeat = 1.
 * w is [num_experts, N, K*bits/32]. sorted_indices is accepted and ignored (the
 * kernels always group rows by expert themselves). transpose must be nonzero.
 * Each expert runs on the kernel its row count calls for, as in moe_block_forward:
 * experts with 32 rows or more on the tcgen05 GEMM (N % 128 == 0), the rest on the GEMV.
 */
int moe_gather_qmm(moe_ctx* ctx, const void* x, int64_t x_rows, int64_t K, int64_t x_repeat,
                   const uint32_t* lhs_indices, const uint32_t* w, const void* scales,
                   const void* biases, int64_t num_experts, int64_t N,
                   const uint32_t* rhs_indices, int64_t batch, int transpose, int group_size,
                   int bits, int sorted_indices, void* out);

/*
 * out[rows, dim] = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * weight)
 * Replaces Array::fast_rms_norm (crates/mlx-core/src/ops.rs:691-701) as called by
 * RmsNorm::forward (crates/mlx-nn/src/rms_norm.rs:30-34). dim % 8 == 0.
 */
int moe_fast_rms_norm(moe_ctx* ctx, const void* x, const void* weight, float eps, int64_t rows,
                      int64_t dim, void* out);

/*
 * The whole block: out[T, H] = MoE(x[T, H]) — router, scoring, top-k, SwitchGLU over
 * the selected experts, weighted combine and the optional sigmoid-gated shared
 * expert, on the context's stream.
 * Replaces SparseMoeBlock::forward (qwen3_moe_python_port.rs:420-488) and
 * MoeFeedForward::forward (lfm2_moe_python_port.rs:541-740), which are private in the
 * reference and reach mlx-c through quantized_matmul / softmax / argpartition /
 * take_along_axis / gather_qmm / multiply / sum_axis.
 */
int moe_block_forward(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts,
                      const void* x, int64_t T, void* out);

/*
 * The MoE half of a decoder layer: out[T, H] = x + MoE(RMSNorm(x; norm_weight, eps)),
 * the RMSNorm as moe_fast_rms_norm and the residual add fused into the combine
 * (out = bf16(x + bf16(moe)), the bf16 add of the reference). Replaces the FFN half of
 * MoeBlock::forward (qwen3_moe_python_port.rs:736-739: post_attention_layernorm,
 * ff.forward, residual.add) and of Lfm2Layer::forward (lfm2_moe_python_port.rs:856-868:
 * ffn_norm, ffn.forward, residual.add). normed[T, H] (optional) receives the RMSNorm
 * output; NULL keeps it in the context's scratch. x, normed and out must not overlap.
 */
int moe_layer_ffn_forward(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts,
                          const void* x, int64_t T, const void* norm_weight, float eps, void* normed,
                          void* out);

/*
 * The Gemma4 MoE block: out[T, H] (f32) = SparseMoeBlock::forward of
 * crates/mlx-models/src/gemma4.rs:1063-1085 with its Router (:906-936) and its GELU SwitchGlu
 * (:1045-1052). The router normalises x (RMSNorm with a unit weight, eps 1e-6), multiplies
 * by hidden^-0.5 and router_scale [H] (bf16) in f32, takes f32 logits through
 * wts->router, selects the top_k experts by logit, and weights them by
 * softmax(logits)[idx] / sum * per_expert_scale[idx] ([E] bf16), all in f32; the experts
 * compute down(gelu_approx(gate(x)) * up(x)); the block output is the f32 weighted sum.
 * cfg->scoring, norm_topk_prob and has_shared_gate are ignored; shared_inter must be 0.
 * idx_out [T, k] and weights_out [T, k] (f32) optional. Differences from the reference,
 * all inside the parity tolerance: the expert hidden h = gelu(gate) * up is rounded to
 * bf16 before the down projection and the expert outputs are rounded to bf16 before the
 * combine (the kernels' MMA operands and outputs are bf16; the reference keeps both f32).
 * The reference's block is private; SparseMoeBlock::forward in gemma4.rs is what this
 * replaces.
 */
int moe_gemma4_block_forward(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts,
                             const void* router_scale, const void* per_expert_scale, const void* x, int64_t T,
                             float* out, uint32_t* idx_out, float* weights_out);

/*
 * Routing only (R1-R4 plus the per-expert grouping gather_qmm forms internally):
 *   idx[T, k] uint32      selected experts, by (score desc, index asc);
 *   weights[T, k] bf16    combine weights (renormalised when norm_topk_prob);
 *   offsets[E + 1] int32  exclusive prefix sum of per-expert pair counts;
 *   perm[T * k] uint32    pairs p = t*k + j grouped by expert, ascending p within one.
 * Any output pointer may be NULL. Replaces the router half of the block
 * (qwen3_moe_python_port.rs:436-445, lfm2_moe_python_port.rs:559-586) and is what the
 * reference's MLX_VALIDATE_MOE_DEVICE_ROUTER shadow check reads back (:449-464).
 */
int moe_block_route(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts,
                    const void* x, int64_t T, uint32_t* idx, void* weights, int32_t* offsets,
                    uint32_t* perm);

/*
 * The router linear of a block alone: logits[T, n] (bf16, n = num_experts, plus one
 * column for the shared_expert_gate row when shared_inter > 0 and has_shared_gate), the
 * quantized_matmul of Linear::forward (crates/mlx-nn/src/linear.rs:117-128) on the gate
 * weight (qwen3_moe_python_port.rs:436, lfm2_moe_python_port.rs:559) and on
 * shared_expert_gate (qwen3_moe_python_port.rs:475-476), with the same canonical fp32
 * order as the routing of moe_block_forward (bit-identical logits). Reads only
 * wts->router and wts->shared_expert_gate.
 */
int moe_block_router_logits(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts,
                            const void* x, int64_t T, void* logits);

/*
 * moe_block_forward with CUDA events between its stages; blocks until the block has
 * run. stage_ms[8] receives the device time of: router, top-k, grouping, gate/up,
 * down, shared gate/up, shared down, combine; n_active (optional) the number of
 * distinct experts the routing selected. When the block ran as the one-launch decode
 * kernel (the smallest batches), its whole time is the gate/up entry and the other seven
 * are zero. Replaces the per-stage timers of
 * MoeProfileStats (qwen3_moe_python_port.rs:53-158, lfm2_moe_python_port.rs trace
 * stats), which time graph construction on the host rather than device work.
 */
int moe_block_profile(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts,
                      const void* x, int64_t T, void* out, float* stage_ms, int32_t* n_active);

/*
 * Status word of the context's device work: nonzero after a bounded device-side wait
 * expired in a kernel launched on this context (the kernel then stopped early and its
 * outputs are invalid). Synchronises the context's stream. No counterpart in the
 * reference (MLX kernels do not wait on barriers with a time limit).
 */
int moe_ctx_status(moe_ctx* ctx, int32_t* status);

/*
 * Expert parallelism (EP) over `world` ranks, one process and one context per GPU.
 * Rank r holds the router, expert_bias and the experts [expert_begin, expert_begin +
 * num_local) of every block, and its own T_r tokens. One block on every rank is:
 *   1. moe_ep_route(x_r)                       -> packed_r [T_r, k]
 *   2. all-gather x_r -> x_all [T_all, H] and packed_r -> packed_all [T_all, k]
 *      (every rank's tokens in rank order; NCCL, by the host)
 *   3. moe_ep_experts(x_all, packed_all)       -> partial [T_all, H] fp32
 *   4. all-to-all of partial in equal parts of T_r rows: rank s sends rows
 *      [r*T_r, (r+1)*T_r) of its partial to rank r (NCCL, by the host)
 *   5. moe_ep_finish(received [world, T_r, H]) -> out_r [T_r, H] (+ next RMSNorm)
 * The block's routing is that of moe_block_forward, bit for bit; the output differs
 * from it only in the fp32 association of the k-term sum (ranks' partial sums are
 * added in rank order), i.e. by last-bit rounding. These replace
 * SparseMoeBlock::forward (qwen3_moe_python_port.rs:420-488) when its experts are
 * sharded; the reference runs on one device and has no EP, so the split itself has
 * no reference counterpart. Blocks with a shared expert are not supported here
 * (MOE_ERR_UNSUPPORTED).
 */

/* Routing of this rank's tokens: packed[T, k] = expert | bf16(weight) << 16, the
 * experts and weights of moe_block_route (qwen3_moe_python_port.rs:436-445,
 * lfm2_moe_python_port.rs:559-586). Reads only wts->router and wts->expert_bias. */
int moe_ep_route(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts,
                 const void* x, int64_t T, uint32_t* packed);

/* This rank's experts over every rank's tokens: partial[t, :] (fp32) = sum over
 * j = 0..k-1 in order, of the pairs (t, j) whose expert lies in [expert_begin,
 * expert_begin + num_local), of bf16(expert_out * weight) (the weighted combine of
 * qwen3_moe_python_port.rs:471-472 restricted to these experts, not rounded); zero
 * rows for tokens that chose none of them. cfg->num_experts is the global E; the
 * gate/up/down tensors of wts hold the num_local local experts, [num_local, N, K/8].
 * Scratch covers the worst case of every pair being local (T_all*k rows). */
int moe_ep_experts(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts,
                   const void* x_all, int64_t T_all, const uint32_t* packed_all,
                   int32_t expert_begin, int32_t num_local, float* partial);

/* moe_ep_experts with each partial sum rounded once to bf16 (round to nearest even) into
 * partial [T_all, hidden] bf16: half the bytes through the combine's all-to-all. The
 * owner's sum (moe_ep_finish_bf16) then adds bf16-rounded partials, which differs from
 * the fp32 form only for tokens whose experts lie on more than one rank, but there
 * partials of opposite sign that nearly cancel lose relative accuracy (the fp32 form is
 * the one held to the block's parity bound). */
int moe_ep_experts_bf16(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts,
                        const void* x_all, int64_t T_all, const uint32_t* packed_all,
                        int32_t expert_begin, int32_t num_local, void* partial);

/* moe_ep_finish over bf16 partials [world, rows, hidden] (widened exactly, summed in fp32
 * in rank order). */
int moe_ep_finish_bf16(moe_ctx* ctx, const void* partials, int32_t world, int64_t rows,
                       int64_t hidden, void* out, const void* norm_weight, float eps, void* normed);

/* out[r] = bf16(sum over s = 0..world-1 in order of partials[s, r, :]) for r < rows
 * (partials [world, rows, hidden] fp32, the all-to-all's output). With norm_weight
 * (and normed), also normed[r] = moe_fast_rms_norm(out[r], norm_weight, eps): the
 * RMSNorm before the next block of a stack, fused. */
int moe_ep_finish(moe_ctx* ctx, const float* partials, int32_t world, int64_t rows,
                  int64_t hidden, void* out, const void* norm_weight, float eps, void* normed);

/*
 * moe_gather_qmm without any device allocation. Same arguments, semantics and results
 * as moe_gather_qmm; no counterpart in the reference (mlx-c allocates through MLX's own
 * allocator). For callers that cannot let a library allocate GPU memory: a host
 * framework whose allocator already owns the device memory, or a latency-critical
 * loop where cudaMalloc/cudaFree (which may synchronise the device) are not allowed.
 * Its row-grouping scratch is a fixed 64 KiB array in the library's device image
 * (held by every GPU that loads the library until the process exits), so
 * batch <= MOE_NOALLOC_MAX_BATCH and num_experts <= MOE_NOALLOC_MAX_EXPERTS; larger
 * calls return MOE_ERR_INVALID. The context provides the device, the stream and the
 * error message; its own scratch is not used. All calls on a device share the array:
 * calls that overlap on the GPU race, so order them. The first call on each device
 * looks up the array's device address (with that device current); make it before any
 * stream capture. The arguments are checked as moe_gather_qmm checks them (same codes,
 * same order) before the size limits. An expired bounded wait inside the tcgen05 GEMM
 * is not reported through moe_ctx_status for this entry point (it has no status word).
 */
#define MOE_NOALLOC_MAX_BATCH 4096
#define MOE_NOALLOC_MAX_EXPERTS 512
int moe_gather_qmm_noalloc(moe_ctx* ctx, const void* x, int64_t x_rows, int64_t K,
                           int64_t x_repeat, const uint32_t* lhs_indices, const uint32_t* w,
                           const void* scales, const void* biases, int64_t num_experts,
                           int64_t N, const uint32_t* rhs_indices, int64_t batch,
                           int transpose, int group_size, int bits, int sorted_indices,
                           void* out);

#ifdef __cplusplus
}
#endif
#endif

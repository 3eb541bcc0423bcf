// kernels.cuh — argument blocks and launchers of the MoE kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

namespace moe {

// Launches kern with programmatic stream serialisation (the kernel may begin while its
// predecessor in the stream finishes; it calls pdl_wait() before reading the
// predecessor's outputs). MOE_B200_PDL=0 in the environment launches normally.
bool pdl_enabled();
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                     Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Router logits: logits[T, n_rows] = x[T, K] . dequant(W)^T in the canonical order.
// Rows 0..E-1 come from the router weight; row E (when n_rows == E + 1) is the
// shared_expert_gate row.
struct RouterArgs {
  const uint16_t* x;
  int T, K, E, n_rows, group_size;
  const uint32_t* w;
  const uint16_t* s;
  const uint16_t* b;
  const uint32_t* gate_w;
  const uint16_t* gate_s;
  const uint16_t* gate_b;
  uint16_t* logits;
  const float* xf;     // f32 token rows (stride K) in place of x (the Gemma4 router), or null
  float* logits_f32;   // f32 logits [T, n_rows], not rounded (with xf), or null
};

struct TopkArgs {
  const uint16_t* logits;  // [T, n_rows]
  int T, E, n_rows, k, scoring, norm_topk_prob;
  const uint16_t* expert_bias;  // [E] or null
  uint32_t* idx;                // [T, k]
  uint16_t* weights;            // [T, k] bf16
  uint16_t* gate_val;           // [T] bf16 = sigmoid(logits[:, E]) or null
  uint32_t* packed;             // [T, k] idx | bf16(weight) << 16, or null
  // scoring 3 (the Gemma4 router): f32 logits in, top-k by logit, f32 weights
  // softmax(logits)[idx] / sum * per_expert_scale[idx] out
  const float* logits_f32;      // [T, n_rows]
  const uint16_t* per_expert_scale;  // [E] bf16
  float* weights_f32;           // [T, k]
};

// Stable grouping of P pair ids by expert id. The expert of pair p is
// (key_packed ? key[p] & 0xffff : key[p]) - key_base; pairs whose expert falls
// outside [0, E) are left out (offsets[E] counts the pairs kept).
struct GroupArgs {
  const uint32_t* key;  // [P]
  int key_packed;
  uint32_t key_base;
  int64_t P;
  int E;
  int seg;          // pairs per segment
  int nseg;         // ceil(P / seg)
  int32_t* hist;    // [nseg, E] scratch
  int32_t* segbase; // [nseg, E] scratch
  int32_t* offsets; // [E + 1]
  int32_t* active;  // [E] experts with pairs, ascending
  int32_t* n_active;
  uint32_t* perm;   // [P] pos -> p
  uint32_t* inv;    // [P] p -> pos, may be null
  int32_t* tile_start;  // [E + 1] exclusive prefix of ceil(count_e / tile_rows), may be null
  int tile_rows;
  int tc_min_rows;      // experts with fewer pairs get no tiles (0: every expert)
};

// Grouped quantized GEMV/GEMM over expert-grouped rows (tensor cores via mma.sync,
// 4-bit weights dequantised in registers).
struct QgemvArgs {
  const uint16_t* x;    // activations, row stride K
  int x_mode;           // 0: row = pos, 1: row = perm[pos] / x_repeat, 2: row = lhs[perm[pos]]
  int x_repeat;
  const uint32_t* lhs;
  const uint32_t* perm;     // pos -> original index, null = identity
  const int32_t* offsets;   // [E+1], null = one expert (0) owning rows [0, n_identity)
  const int32_t* active;    // slot -> expert, null = slot is the expert id
  const int32_t* n_active;  // number of valid slots (device), null = all
  int n_identity;
  const uint32_t* w0;       // [E, N, K/8]
  const uint16_t* s0;       // [E, N, K/64]
  const uint16_t* b0;
  const uint32_t* w1;       // second matrix (up) for the gated form
  const uint16_t* s1;
  const uint16_t* b1;
  int N, K;
  uint16_t* out;            // [rows, N] bf16
  int out_mode;             // 0: row = pos, 1: row = perm[pos]
  int max_expert_rows;      // experts with this many rows or more are skipped (0: none)
  // split-K (set by launch_qgemv when the grid would be too small): fp32 partials
  // [ksplit][part_rows][N or 2N] in a caller-provided buffer, then a reduction launch.
  int ksplit;
  float* partial;           // null: never split
  size_t partial_bytes;
  int64_t part_rows;        // rows of the partial buffer (grouped positions; P or T)
  int num_experts_total;    // entries of offsets minus one (for the reduction's row check)
  int act;                  // gated form: 0 SiLU(gate) * up in bf16 ops, 1 GELU-tanh(gate) * up in f32
};

struct CombineArgs {
  const uint16_t* y;        // [P, H] expert outputs in grouped order
  const uint32_t* inv;      // [P] pair -> grouped row
  const uint16_t* weights;  // [T, k] bf16
  const float* weights_f32; // [T, k] f32 weights, f32 products and sum, f32 out_f32 (the Gemma4 block)
  float* out_f32;           // [T, H]
  const uint16_t* shared;   // [T, H] shared expert output or null
  const uint16_t* gate_val; // [T] bf16 shared gate or null
  const uint16_t* residual; // [T, H] added last (the decoder layer's residual) or null
  int T, k, H;
  uint16_t* out;            // [T, H]
};

// Segment length of the grouping for P pairs over E experts: short segments (more
// parallel scatter warps) while the [nseg, E] histogram fits the scan's shared memory.
constexpr size_t kGroupScanSmem = 192 * 1024;
inline int group_seg(int64_t P, int E) {
  int seg = 256;
  while ((size_t)((P + seg - 1) / seg) * (size_t)E * 4 > kGroupScanSmem) seg *= 2;
  return seg;
}

cudaError_t launch_router(const RouterArgs& a, cudaStream_t st);
// Router + top-k (+ grouping when ga is non-null) in one launch for T <= 64 tokens
// (route_fused_fits). counters: kFusedRouteCounters zero-initialised words, left zero.
constexpr int kFusedRouteMaxTokens = 64;
constexpr int kFusedRouteCounters = kFusedRouteMaxTokens / 4 + 1;
bool route_fused_fits(int T, int E, int64_t P);
cudaError_t launch_route_fused(const RouterArgs& ra, const TopkArgs& ta, const GroupArgs* ga, uint32_t* counters,
                               cudaStream_t st);
cudaError_t launch_topk(const TopkArgs& a, cudaStream_t st);
cudaError_t launch_group(const GroupArgs& a, cudaStream_t st);
// gated: out = swiglu(x.W0^T, x.W1^T); else out = x.W0^T. rows_per_expert (the expected
// rows of an expert) sets how many tokens one pass over the weights serves; slots = the
// number of expert slots of the grid.
cudaError_t launch_qgemv(const QgemvArgs& a, bool gated, int slots, int rows_per_expert,
                         cudaStream_t st);
// Grouped GEMM on tcgen05 tensor cores for the prefill regime (many rows per expert):
// one CTA = 128 weight rows x up to 256 rows (tokens) of one expert. Requires N % 128 == 0
// and K % 64 == 0. tile_start (from the grouping) maps CTAs to (expert, token tile).
struct TcGemmArgs {
  QgemvArgs q;                // operands, row mapping and output as for the GEMV
  const int32_t* tile_start;  // [E + 1] prefix of 256-row tiles per expert (null: identity)
  int num_experts;            // E (entries of tile_start minus one)
  int max_tiles;              // grid.y
  int32_t* status;            // device word: nonzero after a bounded wait expired
  int ksplit;                 // grid.z: K splits into q.partial [ksplit][rows][N or 2N], 0/1 none
  // TMA maps of the packed weights q.w0 / q.w1 ([num_experts * N rows][K / 8 words],
  // box [128 rows][8 words]); filled by launch_tc_gemm
  CUtensorMap wmap[2];
};
// Ordered reduction of split-K partials (q.partial, q.ksplit, q.part_rows) into q.out.
cudaError_t launch_gemv_reduce(const QgemvArgs& q, bool gated, cudaStream_t st);
constexpr int kTcTileRows = 256;
cudaError_t launch_tc_gemm(const TcGemmArgs& a, bool gated, cudaStream_t st);

cudaError_t launch_combine(const CombineArgs& a, cudaStream_t st);

// The whole block for decode-sized batches (T <= kDecodeMaxT tokens) in one persistent
// cooperative kernel (decode.cu): router logits -> grid barrier -> top-k and grouping
// (every CTA, in shared memory) -> gate/up + SwiGLU of the selected experts and the
// shared expert (down weights prefetched into L2 meanwhile) -> grid barrier -> down
// projection and weighted combine (+ gated shared expert, + residual) per tile of 16
// hidden rows.
constexpr int kDecodeMaxT = 8;
constexpr int kDecodeMaxP = 64;
constexpr int kDecodeWarps = 16;  // at most (8 or 16 by the number of units)
constexpr int kDecodeLogitReplicas = 16;
struct DecodeArgs {
  RouterArgs ra;             // logits into scratch [T, n_rows]
  TopkArgs ta;               // scoring / top-k / renorm options (output pointers unused)
  int T, H, I, Is, k;
  const uint32_t* wg; const uint16_t* sg; const uint16_t* bg;   // gate [E, I, H/8]
  const uint32_t* wu; const uint16_t* su; const uint16_t* bu;   // up   [E, I, H/8]
  const uint32_t* wd; const uint16_t* sd; const uint16_t* bd;   // down [E, H, I/8]
  const uint32_t* swg; const uint16_t* ssg; const uint16_t* sbg;  // shared gate [Is, H/8]
  const uint32_t* swu; const uint16_t* ssu; const uint16_t* sbu;  // shared up   [Is, H/8]
  const uint32_t* swd; const uint16_t* ssd; const uint16_t* sbd;  // shared down [H, Is/8]
  uint16_t* logits_rep;      // [kDecodeLogitReplicas][T, n_rows] scratch: the router's logits,
                             // replicated so that the CTAs' reads spread over many L2 lines
  uint16_t* hbuf;            // [T*k, I] scratch (pair order)
  uint16_t* hsbuf;           // [T, Is] scratch
  const uint16_t* residual;  // [T, H] added last, or null
  uint16_t* out;             // [T, H]
  uint32_t* barrier;         // grid barrier word (any value; left consistent after each call)
  int32_t* status;           // device status word (bounded waits)
  int32_t* n_active;         // receives the number of distinct experts selected (or null)
  int has_gate;              // the shared expert is gated by sigmoid(logit row E)
  int scale8;                // 1: every scale/bias row pair of 4 groups is one 8-byte copy
};
// Dynamic shared memory of the decode kernel (0: the shapes do not fit it).
size_t decode_smem_bytes(int T, int k, int E, int H, int I, int Is);
cudaError_t launch_decode_block(const DecodeArgs& a, cudaStream_t st);

// One gather_qmm (out[i] = x[row(i)] . dequant(w[rhs[i]])^T, out in the caller's row
// order): grouping by expert, then each expert on the kernel its row count calls for
// (tcgen05 for experts with many rows, the GEMV for the rest), as in the block. The
// scratch pointers of g (hist, segbase, offsets, active, n_active, perm, tile_start,
// seg, nseg) and status come from the caller; the rest of g is filled here.
struct GatherCall {
  const uint16_t* x;
  int x_mode;  // 1: x row = i / x_repeat, 2: x row = lhs[i]
  int x_repeat;
  const uint32_t* lhs;
  const uint32_t* w;
  const uint16_t* s;
  const uint16_t* b;
  int E, N, K;
  int64_t batch;
  const uint32_t* rhs;
  uint16_t* out;
  GroupArgs g;
  int32_t* status;
};
cudaError_t launch_gather_qmm(const GatherCall& c, cudaStream_t st);

// Expert parallelism. Partial combine of one rank's experts [e0, e0 + E_l):
// partial[t, :] (fp32) = sum over j = 0..k-1 in order, of the pairs p = t*k + j whose
// expert is local, of bf16(y[inv[p], :] * weight_p); zero for tokens with none.
struct EpPartialArgs {
  const uint16_t* y;        // [local pairs, H] expert outputs in grouped order
  const uint32_t* inv;      // [T*k] pair -> grouped row (written for local pairs only)
  const uint32_t* packed;   // [T, k] expert | bf16(weight) << 16
  uint32_t e0;
  int E_l, T, k, H;
  float* partial;           // [T, H] fp32, or null when partial_bf16 is given
  uint16_t* partial_bf16;   // [T, H] bf16 (round to nearest even), or null
};
cudaError_t launch_ep_partial(const EpPartialArgs& a, cudaStream_t st);
// out[r] = bf16(sum over ranks s = 0..world-1 in order of recv[s, r, :]) for r < rows;
// with norm_w, also normed[r] = RMSNorm(out[r]) * norm_w as launch_rms_norm computes it.
cudaError_t launch_ep_finish(const float* recv, int world, int64_t rows, int H, uint16_t* out,
                             const uint16_t* norm_w, float eps, uint16_t* normed, cudaStream_t st);
// The same over bf16 partials (each widened to fp32 exactly, then summed in rank order).
cudaError_t launch_ep_finish_bf16(const uint16_t* recv, int world, int64_t rows, int H, uint16_t* out,
                                  const uint16_t* norm_w, float eps, uint16_t* normed, cudaStream_t st);
cudaError_t launch_rms_norm(const uint16_t* x, const uint16_t* w, float eps, int64_t rows, int dim,
                            uint16_t* out, cudaStream_t st);
// The Gemma4 router's input: out[r] (f32) = f32(RMSNorm(x[r]) with unit weight, rounded to
// bf16) * root * f32(scale), as launch_rms_norm computes the norm.
cudaError_t launch_gemma_router_input(const uint16_t* x, const uint16_t* scale, float root, float eps, int64_t rows,
                                      int dim, float* out, cudaStream_t st);

}  // namespace moe

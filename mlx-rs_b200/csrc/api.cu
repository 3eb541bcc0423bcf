// api.cu — the extern "C" boundary declared in include/moe_b200.h.
//
// Validates arguments, owns the per-context scratch, and sequences the kernels of
// the block on the context's stream:
//   router logits (+ shared_expert_gate row) -> scoring / top-k / weights ->
//   grouping by expert -> gate/up grouped GEMV with SwiGLU epilogue -> down grouped
//   GEMV -> [shared expert gate/up, down] -> weighted combine (+ gated shared).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cmath>
#include <cstring>
#include <new>
#include <string>

#include "../../include/moe_b200.h"
#include "kernels.cuh"

struct moe_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  std::string last_error;
  bool last_block_fused = false;  // the last block call ran the one-launch decode kernel
  // side stream for the tcgen05 half of a hybrid expert step (created on first use
  // outside stream capture), with its fork / join events
  cudaStream_t side = nullptr;
  cudaEvent_t fork_ev = nullptr, join_ev = nullptr;
};

namespace {


int fail(moe_ctx* ctx, int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  if (ctx) ctx->last_error = buf;
  return code;
}

#define MOE_CUDA(ctx, expr)                                                                       \
  do {                                                                                            \
    cudaError_t _e = (expr);                                                                      \
    if (_e != cudaSuccess) return fail((ctx), MOE_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(_e)); \
  } while (0)

// Switches to the context's device for the duration of a call.
struct DeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Bump allocator over the context scratch (256-byte aligned slices).
struct Carve {
  char* base;
  size_t off = 0;
  explicit Carve(void* b) : base(static_cast<char*>(b)) {}
  template <class T>
  T* take(size_t count) {
    off = (off + 255) & ~size_t(255);
    T* p = reinterpret_cast<T*>(base ? base + off : nullptr);
    off += count * sizeof(T);
    return p;
  }
};

int ensure_scratch(moe_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->scratch_bytes) return MOE_OK;
  if (ctx->scratch) {
    // cudaFree waits for work in flight that may still use the old buffer.
    cudaFree(ctx->scratch);
    ctx->scratch = nullptr;
    ctx->scratch_bytes = 0;
  }
  size_t want = std::max<size_t>(bytes, size_t(1) << 20);
  cudaError_t e = cudaMalloc(&ctx->scratch, want);
  if (e != cudaSuccess) {
    ctx->scratch = nullptr;
    return fail(ctx, MOE_ERR_NO_MEMORY, "scratch cudaMalloc(%zu) failed: %s", want, cudaGetErrorString(e));
  }
  ctx->scratch_bytes = want;
  // the first word holds the device status (bounded waits that expired); start clean
  e = cudaMemset(ctx->scratch, 0, 256);
  if (e != cudaSuccess) return fail(ctx, MOE_ERR_CUDA, "scratch status reset failed: %s", cudaGetErrorString(e));
  return MOE_OK;
}

int check_quant(moe_ctx* ctx, const char* fn, int64_t K, int group_size, int bits) {
  if (!(bits == 2 || bits == 3 || bits == 4 || bits == 5 || bits == 6 || bits == 8))
    return fail(ctx, MOE_ERR_INVALID, "%s: bits=%d is not a valid MLX affine width", fn, bits);
  if (!(group_size == 32 || group_size == 64 || group_size == 128))
    return fail(ctx, MOE_ERR_INVALID, "%s: group_size=%d is not a valid MLX group size", fn, group_size);
  if (bits != 4 || group_size != 64)
    return fail(ctx, MOE_ERR_UNSUPPORTED, "%s: only bits=4, group_size=64 are implemented (got %d, %d)", fn,
                bits, group_size);
  if (K <= 0 || K % 64 != 0)
    return fail(ctx, MOE_ERR_INVALID, "%s: K=%lld must be a positive multiple of 64", fn, (long long)K);
  return MOE_OK;
}

// Workspace of a block call with T tokens (base == null: size only).
struct BlockWs {
  uint16_t* logits;
  uint32_t* idx;
  uint16_t* wsel;
  uint16_t* gate_val;
  int32_t* hist;
  int32_t* segbase;
  int32_t* offsets;
  int32_t* active;
  int32_t* n_active;
  uint32_t* perm;
  uint32_t* inv;
  uint16_t* hbuf;
  uint16_t* ybuf;
  uint16_t* hs;
  uint16_t* ys;
  int32_t* tile_start;
  int32_t* status;
  float* gemv_partial;  // split-K partials of small GEMVs (null when T is large)
  size_t gemv_partial_bytes;
  float* tc_partial;    // split-K partials of the shared expert's tcgen05 GEMMs
  size_t tc_partial_bytes;
  uint16_t* xnorm;      // RMSNorm(x) of the decoder-layer step
  uint16_t* logits_rep; // replicated router logits of the decode kernel (T <= kDecodeMaxT)
  size_t bytes;
};

// K splits of a single-matrix tcgen05 GEMM (the shared expert) whose ctas CTAs would
// leave SMs idle: up to 8, about two waves of CTAs, at least 4 K steps per split, and
// partials [splits][rows][N2] fp32 within cap bytes.
int tc_ksplit(int ctas, int ksteps, int64_t rows, int N2, size_t cap) {
  if (ctas >= 148 || cap == 0) return 1;
  int ks = 1;
  while (ks < 8 && (int64_t)ctas * ks * 2 <= 2 * 148 && ksteps / (2 * ks) >= 4) ks *= 2;
  while (ks > 1 && (size_t)ks * rows * N2 * sizeof(float) > cap) ks >>= 1;
  return ks;
}

// Split-K buffer of the shared expert's tcgen05 down projection at prefill sizes: at
// most 64 MiB.
size_t tc_partial_floats(const moe_block_config* c, int64_t T) {
  size_t want = 0;
  if (c->shared_inter > 0 && T >= 32) want = (size_t)8 * T * c->hidden;
  return std::min<size_t>(want, (size_t)16 << 20);
}

// Split-K partial buffer of a block call: up to 8 splits of the routed projections
// (P <= 256 pairs) and of the shared expert (T <= 64 tokens); 0 when neither applies.
size_t gemv_partial_floats(const moe_block_config* c, int64_t T) {
  const int64_t P = T * c->top_k;
  size_t n = 0;
  if (P <= 256) n = std::max<size_t>(n, (size_t)8 * P * std::max(2 * c->moe_inter, c->hidden));
  if (c->shared_inter > 0 && T <= 64)
    n = std::max<size_t>(n, (size_t)8 * T * std::max(2 * c->shared_inter, c->hidden));
  return n;
}

BlockWs carve_block(void* base, const moe_block_config* c, int64_t T) {
  Carve cv(base);
  BlockWs w{};
  const int64_t E = c->num_experts, P = T * c->top_k;
  const int64_t nseg = std::max<int64_t>(1, (P + moe::group_seg(P, (int)E) - 1) / moe::group_seg(P, (int)E));
  w.status = cv.take<int32_t>(64);  // first, at a fixed offset; zeroed when allocated
  w.logits = cv.take<uint16_t>(T * (E + 1));
  w.idx = cv.take<uint32_t>(P);
  w.wsel = cv.take<uint16_t>(P);
  w.gate_val = cv.take<uint16_t>(T);
  w.hist = cv.take<int32_t>(nseg * E);
  w.segbase = cv.take<int32_t>(nseg * E);
  w.offsets = cv.take<int32_t>(E + 1);
  w.active = cv.take<int32_t>(E);
  w.n_active = cv.take<int32_t>(1);
  w.perm = cv.take<uint32_t>(P);
  w.inv = cv.take<uint32_t>(P);
  w.tile_start = cv.take<int32_t>(E + 1);
  w.hbuf = cv.take<uint16_t>(P * c->moe_inter);
  w.ybuf = cv.take<uint16_t>(P * c->hidden);
  if (c->shared_inter > 0) {
    w.hs = cv.take<uint16_t>(T * c->shared_inter);
    w.ys = cv.take<uint16_t>(T * c->hidden);
  }
  const size_t npart = gemv_partial_floats(c, T);
  w.gemv_partial = npart ? cv.take<float>(npart) : nullptr;
  w.gemv_partial_bytes = npart * sizeof(float);
  const size_t ntc = tc_partial_floats(c, T);
  w.tc_partial = ntc ? cv.take<float>(ntc) : nullptr;
  w.tc_partial_bytes = ntc * sizeof(float);
  w.xnorm = cv.take<uint16_t>(T * c->hidden);
  if (T <= moe::kDecodeMaxT) w.logits_rep = cv.take<uint16_t>((size_t)moe::kDecodeLogitReplicas * T * (E + 1));
  w.bytes = cv.off + 256;
  return w;
}

int check_block(moe_ctx* ctx, const moe_block_config* c, const moe_block_weights* w, const char* fn) {
  if (!c) return fail(ctx, MOE_ERR_INVALID, "%s: null config", fn);
  int rc = check_quant(ctx, fn, c->hidden, c->group_size, c->bits);
  if (rc) return rc;
  if (c->num_experts <= 0 || c->num_experts > 512)
    return fail(ctx, MOE_ERR_UNSUPPORTED, "%s: num_experts=%d (supported 1..512)", fn, c->num_experts);
  if (c->top_k <= 0 || c->top_k > 32 || c->top_k > c->num_experts)
    return fail(ctx, MOE_ERR_INVALID, "%s: top_k=%d (1..min(32, num_experts))", fn, c->top_k);
  if (c->moe_inter <= 0 || c->moe_inter % 64 != 0)
    return fail(ctx, MOE_ERR_INVALID, "%s: moe_inter=%d must be a positive multiple of 64", fn, c->moe_inter);
  if (c->shared_inter < 0 || c->shared_inter % 64 != 0)
    return fail(ctx, MOE_ERR_INVALID, "%s: shared_inter=%d must be a multiple of 64", fn, c->shared_inter);
  if (c->scoring < 0 || c->scoring > 2) return fail(ctx, MOE_ERR_INVALID, "%s: scoring=%d", fn, c->scoring);
  if (!w) return fail(ctx, MOE_ERR_INVALID, "%s: null weights", fn);
  if (!w->router.w || !w->router.scales) return fail(ctx, MOE_ERR_INVALID, "%s: router weight missing", fn);
  if (c->scoring != MOE_SCORING_SOFTMAX && !w->expert_bias)
    return fail(ctx, MOE_ERR_INVALID, "%s: scoring mode %d needs expert_bias", fn, c->scoring);
  const moe_qweight* need[3] = {&w->gate, &w->up, &w->down};
  for (const moe_qweight* q : need)
    if (!q->w || !q->scales) return fail(ctx, MOE_ERR_INVALID, "%s: expert weights missing", fn);
  if (c->shared_inter > 0) {
    const moe_qweight* sh[3] = {&w->shared_gate, &w->shared_up, &w->shared_down};
    for (const moe_qweight* q : sh)
      if (!q->w || !q->scales) return fail(ctx, MOE_ERR_INVALID, "%s: shared expert weights missing", fn);
    if (c->has_shared_gate && (!w->shared_expert_gate.w || !w->shared_expert_gate.scales))
      return fail(ctx, MOE_ERR_INVALID, "%s: shared_expert_gate weight missing", fn);
  }
  const void* ptrs[] = {w->router.w, w->gate.w, w->up.w, w->down.w};
  for (const void* p : ptrs)
    if (!aligned16(p)) return fail(ctx, MOE_ERR_INVALID, "%s: weight pointers must be 16-byte aligned", fn);
  if (c->shared_inter > 0) {
    const void* sp[] = {w->shared_gate.w, w->shared_up.w, w->shared_down.w};
    for (const void* p : sp)
      if (!aligned16(p)) return fail(ctx, MOE_ERR_INVALID, "%s: weight pointers must be 16-byte aligned", fn);
    if (c->has_shared_gate && !aligned16(w->shared_expert_gate.w))
      return fail(ctx, MOE_ERR_INVALID, "%s: weight pointers must be 16-byte aligned", fn);
  }
  return MOE_OK;
}

// Router-side checks only (the expert-parallel route needs no expert weights).
int check_route(moe_ctx* ctx, const moe_block_config* c, const moe_block_weights* w, const char* fn) {
  if (!c) return fail(ctx, MOE_ERR_INVALID, "%s: null config", fn);
  int rc = check_quant(ctx, fn, c->hidden, c->group_size, c->bits);
  if (rc) return rc;
  if (c->num_experts <= 0 || c->num_experts > 512)
    return fail(ctx, MOE_ERR_UNSUPPORTED, "%s: num_experts=%d (supported 1..512)", fn, c->num_experts);
  if (c->top_k <= 0 || c->top_k > 32 || c->top_k > c->num_experts)
    return fail(ctx, MOE_ERR_INVALID, "%s: top_k=%d (1..min(32, num_experts))", fn, c->top_k);
  if (c->scoring < 0 || c->scoring > 2) return fail(ctx, MOE_ERR_INVALID, "%s: scoring=%d", fn, c->scoring);
  if (c->shared_inter != 0)
    return fail(ctx, MOE_ERR_UNSUPPORTED, "%s: the expert-parallel path has no shared expert (shared_inter=%d)", fn,
                c->shared_inter);
  if (!w || !w->router.w || !w->router.scales) return fail(ctx, MOE_ERR_INVALID, "%s: router weight missing", fn);
  if (c->scoring != MOE_SCORING_SOFTMAX && !w->expert_bias)
    return fail(ctx, MOE_ERR_INVALID, "%s: scoring mode %d needs expert_bias", fn, c->scoring);
  if (!aligned16(w->router.w)) return fail(ctx, MOE_ERR_INVALID, "%s: weight pointers must be 16-byte aligned", fn);
  return MOE_OK;
}

// Expert-side checks of the expert-parallel experts call (the router is not read).
int check_experts(moe_ctx* ctx, const moe_block_config* c, const moe_block_weights* w, const char* fn) {
  if (!c) return fail(ctx, MOE_ERR_INVALID, "%s: null config", fn);
  int rc = check_quant(ctx, fn, c->hidden, c->group_size, c->bits);
  if (rc) return rc;
  if (c->num_experts <= 0 || c->num_experts > 512)
    return fail(ctx, MOE_ERR_UNSUPPORTED, "%s: num_experts=%d (supported 1..512)", fn, c->num_experts);
  if (c->top_k <= 0 || c->top_k > 32 || c->top_k > c->num_experts)
    return fail(ctx, MOE_ERR_INVALID, "%s: top_k=%d (1..min(32, num_experts))", fn, c->top_k);
  if (c->moe_inter <= 0 || c->moe_inter % 64 != 0)
    return fail(ctx, MOE_ERR_INVALID, "%s: moe_inter=%d must be a positive multiple of 64", fn, c->moe_inter);
  if (c->shared_inter != 0)
    return fail(ctx, MOE_ERR_UNSUPPORTED, "%s: the expert-parallel path has no shared expert (shared_inter=%d)", fn,
                c->shared_inter);
  if (!w) return fail(ctx, MOE_ERR_INVALID, "%s: null weights", fn);
  const moe_qweight* need[3] = {&w->gate, &w->up, &w->down};
  for (const moe_qweight* q : need) {
    if (!q->w || !q->scales) return fail(ctx, MOE_ERR_INVALID, "%s: expert weights missing", fn);
    if (!aligned16(q->w)) return fail(ctx, MOE_ERR_INVALID, "%s: weight pointers must be 16-byte aligned", fn);
  }
  return MOE_OK;
}

// Routing workspace of T tokens: the status word, the logits and the top-k scratch.
BlockWs carve_route(void* base, const moe_block_config* c, int64_t T) {
  Carve cv(base);
  BlockWs w{};
  const int64_t E = c->num_experts, P = T * c->top_k;
  w.status = cv.take<int32_t>(64);
  w.logits = cv.take<uint16_t>(T * (E + 1));
  w.idx = cv.take<uint32_t>(P);
  w.wsel = cv.take<uint16_t>(P);
  w.gate_val = cv.take<uint16_t>(T);
  w.bytes = cv.off + 256;
  return w;
}

// Workspace of an expert-parallel experts call over T tokens (every rank's tokens)
// with El local experts; sized for the worst case of every pair being local.
struct EpWs {
  int32_t* status;
  int32_t *hist, *segbase, *offsets, *active, *n_active, *tile_start;
  uint32_t *perm, *inv;
  uint16_t *hbuf, *ybuf;
  float* gemv_partial;
  size_t gemv_partial_bytes;
  size_t bytes;
};

EpWs carve_ep(void* base, const moe_block_config* c, int64_t T, int El) {
  Carve cv(base);
  EpWs w{};
  const int64_t P = T * c->top_k;
  const int64_t nseg = std::max<int64_t>(1, (P + moe::group_seg(P, El) - 1) / moe::group_seg(P, El));
  w.status = cv.take<int32_t>(64);  // first, at the fixed offset every workspace shares
  w.hist = cv.take<int32_t>(nseg * El);
  w.segbase = cv.take<int32_t>(nseg * El);
  w.offsets = cv.take<int32_t>(El + 1);
  w.active = cv.take<int32_t>(El);
  w.n_active = cv.take<int32_t>(1);
  w.tile_start = cv.take<int32_t>(El + 1);
  w.perm = cv.take<uint32_t>(P);
  w.inv = cv.take<uint32_t>(P);
  w.hbuf = cv.take<uint16_t>(P * c->moe_inter);
  w.ybuf = cv.take<uint16_t>(P * c->hidden);
  const size_t npart = P <= 256 ? (size_t)8 * P * std::max(2 * c->moe_inter, c->hidden) : 0;
  w.gemv_partial = npart ? cv.take<float>(npart) : nullptr;
  w.gemv_partial_bytes = npart * sizeof(float);
  w.bytes = cv.off + 256;
  return w;
}

// Stage boundaries recorded by moe_block_profile (ev == null: not recorded).
enum Stage { kRouter = 0, kTopk, kGroup, kGateUp, kDown, kSharedGateUp, kSharedDown, kCombine, kStages };

#define MOE_MARK(ev, i, st) \
  do {                        \
    if (ev) MOE_CUDA(ctx, cudaEventRecord((ev)[i], st)); \
  } while (0)

// The status block (first 256 bytes of the scratch, zeroed when allocated): word 0 is
// the device status (bounded waits that expired); words from kFusedCounterWord are the
// ticket counters of the fused routing kernel, which leaves them zero.
constexpr int kFusedCounterWord = 32;
static_assert(kFusedCounterWord + moe::kFusedRouteCounters <= 64, "status block");

// Opt-in (MOE_B200_FUSED_ROUTE=1): on the B200 the three launches chained by
// programmatic dependent launch finish sooner at decode sizes than the fused kernel,
// whose top-k and grouping run on the last CTAs only.
bool fused_route_enabled() {
  const char* v = std::getenv("MOE_B200_FUSED_ROUTE");
  return v && v[0] == '1';
}

// Routing + grouping of one block call into ws.
// With `packed`, routing writes [T, k] expert | bf16(weight) << 16 there and stops
// before the grouping (the expert-parallel route).
// Router and top-k arguments of a block call (logits into ws.logits).
void route_args(const moe_block_config* c, const moe_block_weights* w, const void* x, int64_t T, const BlockWs& ws,
                moe::RouterArgs& ra, moe::TopkArgs& ta) {
  const int E = c->num_experts;
  const bool gate_row = c->shared_inter > 0 && c->has_shared_gate;
  ra = moe::RouterArgs{};
  ra.x = static_cast<const uint16_t*>(x);
  ra.T = (int)T;
  ra.K = c->hidden;
  ra.E = E;
  ra.n_rows = E + (gate_row ? 1 : 0);
  ra.group_size = c->group_size;
  ra.w = w->router.w;
  ra.s = static_cast<const uint16_t*>(w->router.scales);
  ra.b = static_cast<const uint16_t*>(w->router.biases);
  ra.gate_w = w->shared_expert_gate.w;
  ra.gate_s = static_cast<const uint16_t*>(w->shared_expert_gate.scales);
  ra.gate_b = static_cast<const uint16_t*>(w->shared_expert_gate.biases);
  ra.logits = ws.logits;
  ta = moe::TopkArgs{};
  ta.logits = ws.logits;
  ta.T = (int)T;
  ta.E = E;
  ta.n_rows = ra.n_rows;
  ta.k = c->top_k;
  ta.scoring = c->scoring;
  ta.norm_topk_prob = c->norm_topk_prob;
  ta.expert_bias = static_cast<const uint16_t*>(w->expert_bias);
  ta.gate_val = gate_row ? ws.gate_val : nullptr;
}

int run_route(moe_ctx* ctx, const moe_block_config* c, const moe_block_weights* w, const void* x, int64_t T,
              const BlockWs& ws, cudaEvent_t* ev = nullptr, uint32_t* packed = nullptr, int tc_min_rows = 0) {
  const int E = c->num_experts;
  const bool gate_row = c->shared_inter > 0 && c->has_shared_gate;
  moe::RouterArgs ra{};
  ra.x = static_cast<const uint16_t*>(x);
  ra.T = (int)T;
  ra.K = c->hidden;
  ra.E = E;
  ra.n_rows = E + (gate_row ? 1 : 0);
  ra.group_size = c->group_size;
  ra.w = w->router.w;
  ra.s = static_cast<const uint16_t*>(w->router.scales);
  ra.b = static_cast<const uint16_t*>(w->router.biases);
  ra.gate_w = w->shared_expert_gate.w;
  ra.gate_s = static_cast<const uint16_t*>(w->shared_expert_gate.scales);
  ra.gate_b = static_cast<const uint16_t*>(w->shared_expert_gate.biases);
  ra.logits = ws.logits;
  MOE_MARK(ev, kRouter, ctx->stream);

  moe::TopkArgs ta{};
  ta.logits = ws.logits;
  ta.T = (int)T;
  ta.E = E;
  ta.n_rows = ra.n_rows;
  ta.k = c->top_k;
  ta.scoring = c->scoring;
  ta.norm_topk_prob = c->norm_topk_prob;
  ta.expert_bias = static_cast<const uint16_t*>(w->expert_bias);
  ta.idx = packed ? nullptr : ws.idx;
  ta.weights = packed ? nullptr : ws.wsel;
  ta.packed = packed;
  ta.gate_val = gate_row ? ws.gate_val : nullptr;

  moe::GroupArgs ga{};
  ga.key = ws.idx;
  ga.P = T * c->top_k;
  ga.E = E;
  ga.seg = moe::group_seg(ga.P, E);
  ga.nseg = (int)std::max<int64_t>(1, (ga.P + ga.seg - 1) / ga.seg);
  ga.hist = ws.hist;
  ga.segbase = ws.segbase;
  ga.offsets = ws.offsets;
  ga.active = ws.active;
  ga.n_active = ws.n_active;
  ga.perm = ws.perm;
  ga.inv = ws.inv;
  ga.tile_start = ws.tile_start;
  ga.tile_rows = moe::kTcTileRows;
  ga.tc_min_rows = tc_min_rows;

  // Decode-sized batches, when enabled: one launch (router, top-k and grouping; the
  // stage split of moe_block_profile then books all of it as "router").
  if (moe::route_fused_fits((int)T, E, ga.P) && fused_route_enabled()) {
    MOE_CUDA(ctx, moe::launch_route_fused(ra, ta, packed ? nullptr : &ga,
                                          reinterpret_cast<uint32_t*>(ws.status) + kFusedCounterWord, ctx->stream));
    MOE_MARK(ev, kTopk, ctx->stream);
    MOE_MARK(ev, kGroup, ctx->stream);
    return MOE_OK;
  }
  MOE_CUDA(ctx, moe::launch_router(ra, ctx->stream));
  MOE_MARK(ev, kTopk, ctx->stream);
  MOE_CUDA(ctx, moe::launch_topk(ta, ctx->stream));
  if (packed) return MOE_OK;
  MOE_MARK(ev, kGroup, ctx->stream);
  MOE_CUDA(ctx, moe::launch_group(ga, ctx->stream));
  return MOE_OK;
}

// The smallest batches (T <= kDecodeFusedDefaultT tokens) run the whole block in one
// cooperative kernel when the shapes fit its shared memory and every scale / bias array
// is 4-byte aligned: measured on the B200 with the L2 flushed, a Qwen3-30B-A3B block at
// T = 1 takes 34.8 us against 41.0 us for the launch chain (Qwen1.5-MoE 53 against 59 us),
// while at T = 8 the chain is faster (72 against 103 us: the kernel's gate/up phase, one
// 16-row unit per warp, streams at ~3 TB/s). MOE_B200_DECODE=1 takes the kernel for every
// T <= kDecodeMaxT, =0 never.
constexpr int kDecodeFusedDefaultT = 2;
constexpr int kDecodeBarrierWord = 60;  // grid barrier word of the decode kernel, in the status block
static_assert(kDecodeBarrierWord >= kFusedCounterWord + moe::kFusedRouteCounters && kDecodeBarrierWord < 64,
              "status block");
bool decode_fused_ok(const moe_block_config* c, const moe_block_weights* w, int64_t T) {
  const char* v = std::getenv("MOE_B200_DECODE");
  if (v && v[0] == '0') return false;
  if (!(v && v[0] == '1') && T > kDecodeFusedDefaultT) return false;
  if (T > moe::kDecodeMaxT || !moe::decode_smem_bytes((int)T, c->top_k, c->num_experts, c->hidden, c->moe_inter, c->shared_inter))
    return false;
  const moe_qweight* m[6] = {&w->gate, &w->up, &w->down, &w->shared_gate, &w->shared_up, &w->shared_down};
  for (int i = 0; i < (c->shared_inter > 0 ? 6 : 3); ++i)
    if ((reinterpret_cast<uintptr_t>(m[i]->scales) | reinterpret_cast<uintptr_t>(m[i]->biases)) & 3) return false;
  return true;
}
// 1 when every scale / bias row of every projection moves as 8-byte pieces (groups per
// row a multiple of 4, arrays 8-byte aligned); else the kernel copies 4 bytes at a time.
int decode_scale8(const moe_block_config* c, const moe_block_weights* w) {
  if ((c->hidden / 64) % 4 || (c->moe_inter / 64) % 4 || (c->shared_inter / 64) % 4) return 0;
  const moe_qweight* m[6] = {&w->gate, &w->up, &w->down, &w->shared_gate, &w->shared_up, &w->shared_down};
  for (int i = 0; i < (c->shared_inter > 0 ? 6 : 3); ++i)
    if ((reinterpret_cast<uintptr_t>(m[i]->scales) | reinterpret_cast<uintptr_t>(m[i]->biases)) & 7) return 0;
  return 1;
}

// Tensor-core (tcgen05) GEMM for many rows per expert, GEMV (mma.sync) for few.
// MOE_B200_TC=0 / =1 in the environment forces one path (where the shape allows tc).
bool use_tc(int64_t rows, int64_t experts, int N, int K) {
  if (N % 128 != 0 || K % 64 != 0) return false;
  const char* v = std::getenv("MOE_B200_TC");
  if (v && v[0] == '0') return false;
  if (v && v[0] == '1') return true;
  // (grid.y of the tcgen05 launch holds the token tiles: at most 65535)
  return rows >= 32 * experts && rows <= (int64_t)65535 * moe::kTcTileRows;
}

// Routed experts: each expert takes the path its own row count calls for, decided on
// the device. Experts with at least kTcMinRows rows run on the tcgen05 GEMM (the
// grouping gives only them tiles); the others on the GEMV, which skips the large ones.
// (Measured alternatives that were slower: keeping experts of up to three GEMV passes on
// the GEMV — Qwen1.5-MoE prefill at T=512 fell from 1.14 M to 0.87 M tokens/s — and
// splitting K of the tcgen05 launches when few experts are local — 8-GPU expert-parallel
// decode went from 0.265 to 0.300 ms per step.) MOE_B200_TC=0 puts every expert on the
// GEMV, =1 every expert on tcgen05.
constexpr int kTcMinRows = 32;
// Expected rows per expert from which every expert runs on tcgen05. Measured on the B200
// (CUDA-graph blocks, L2 flushed), against the previous 128: Qwen1.5-MoE T=512 (34 rows
// per expert) 400 -> 356 us, Qwen3-30B-A3B T=384 (24) 375 -> 331 us and T=512 (32) 371
// -> 342 us, LFM2-8B-A1B T=256 (32) 161 -> 129 us; at 16 rows per expert the GEMV, the
// hybrid and all-tcgen05 are level (Qwen3 T=256: 338 us).
constexpr int kTcAllRows = 24;
struct ExpertPlan {
  bool tc_gu = false, tc_dn = false;      // launch the tcgen05 kernel
  bool gemv_gu = true, gemv_dn = true;    // launch the GEMV
  int min_rows = 0;                       // tile threshold of the grouping
  int gemv_skip_gu = 0, gemv_skip_dn = 0; // GEMV max_expert_rows
  int max_tiles = 0;                      // tcgen05 grid.y
};

// max_rows: the most rows one expert can receive (the block: T, since a token selects an
// expert at most once; gather_qmm: every row). Below kTcMinRows no expert can reach the
// tcgen05 threshold and its launches (whose CTAs would all leave at once) are skipped.
ExpertPlan plan_experts(int64_t P, int E, int I, int H, int64_t max_rows) {
  ExpertPlan p;
  const bool shape_gu = I % 128 == 0 && H % 64 == 0, shape_dn = H % 128 == 0 && I % 64 == 0;
  const char* v = std::getenv("MOE_B200_TC");
  if (v && v[0] == '0') return p;
  if (v && v[0] == '1') {
    p.tc_gu = shape_gu;
    p.tc_dn = shape_dn;
    p.gemv_gu = !shape_gu;
    p.gemv_dn = !shape_dn;
  } else if (max_rows < kTcMinRows) {
    return p;  // GEMV only
  } else if (P >= (int64_t)kTcAllRows * E) {
    // prefill, and expert-parallel decode at 8 GPUs: most experts are large, all go to
    // tcgen05 (no GEMV launch)
    p.tc_gu = shape_gu;
    p.tc_dn = shape_dn;
    p.gemv_gu = !shape_gu;
    p.gemv_dn = !shape_dn;
  } else if (P >= kTcMinRows) {
    p.tc_gu = shape_gu;
    p.tc_dn = shape_dn;
    p.min_rows = kTcMinRows;
    p.gemv_skip_gu = shape_gu ? kTcMinRows : 0;
    p.gemv_skip_dn = shape_dn ? kTcMinRows : 0;
  }
  const int64_t big = p.min_rows ? std::min<int64_t>(E, P / p.min_rows) : std::min<int64_t>(E, P);
  p.max_tiles = (int)(P / moe::kTcTileRows + big + 1);
  if (P / moe::kTcTileRows + big + 1 > 65535) {  // beyond grid.y: every expert on the GEMV
    ExpertPlan g;
    return g;
  }
  return p;
}

}  // namespace

// gather_qmm as one hybrid launch sequence (declared in kernels.cuh); shared by
// moe_gather_qmm and moe_gather_qmm_noalloc, which differ only in where the scratch lives.
cudaError_t moe::launch_gather_qmm(const moe::GatherCall& c, cudaStream_t st) {
  // one matrix: the gate/up fields of the plan with I = N, H = K
  const ExpertPlan plan = plan_experts(c.batch, c.E, c.N, c.K, c.batch);
  moe::GroupArgs ga = c.g;
  ga.key = c.rhs;
  ga.key_packed = 0;
  ga.key_base = 0;
  ga.P = c.batch;
  ga.E = c.E;
  ga.inv = nullptr;
  ga.tile_rows = moe::kTcTileRows;
  ga.tc_min_rows = plan.min_rows;
  if (!plan.tc_gu) ga.tile_start = nullptr;
  cudaError_t e = moe::launch_group(ga, st);
  if (e != cudaSuccess) return e;
  moe::QgemvArgs q{};
  q.x = c.x;
  q.x_mode = c.x_mode;
  q.x_repeat = c.x_repeat;
  q.lhs = c.lhs;
  q.perm = ga.perm;
  q.offsets = ga.offsets;
  q.active = ga.active;
  q.n_active = ga.n_active;
  q.w0 = c.w;
  q.s0 = c.s;
  q.b0 = c.b;
  q.N = c.N;
  q.K = c.K;
  q.out = c.out;
  q.out_mode = 1;
  q.num_experts_total = c.E;
  const int slots = (int)std::min<int64_t>(c.batch, c.E);
  const int rows_pe = (int)std::min<int64_t>((c.batch + slots - 1) / slots, 1 << 20);
  if (plan.gemv_gu) {
    q.max_expert_rows = plan.gemv_skip_gu;
    e = moe::launch_qgemv(q, false, slots, rows_pe, st);
    if (e != cudaSuccess) return e;
  }
  if (plan.tc_gu) {
    q.max_expert_rows = 0;
    moe::TcGemmArgs ta{q, ga.tile_start, c.E, plan.max_tiles, c.status};
    e = moe::launch_tc_gemm(ta, false, st);
  }
  return e;
}

namespace {

moe::QgemvArgs qgemv_args(const moe_qweight& m0, const moe_qweight* m1, int N, int K) {
  moe::QgemvArgs q{};
  q.w0 = m0.w;
  q.s0 = static_cast<const uint16_t*>(m0.scales);
  q.b0 = static_cast<const uint16_t*>(m0.biases);
  if (m1) {
    q.w1 = m1->w;
    q.s1 = static_cast<const uint16_t*>(m1->scales);
    q.b1 = static_cast<const uint16_t*>(m1->biases);
  }
  q.N = N;
  q.K = K;
  return q;
}

}  // namespace

namespace {

// The routed experts of a block call after its routing and grouping: SwitchGLU gate/up
// (SiLU * up, act 0; GELU-tanh * up, act 1) and down over the grouped pairs, each expert
// on the GEMV or the tcgen05 GEMM as plan says; expert outputs into ws.ybuf.
// The context's side stream and events, created on first use; false (run everything on
// the context's stream) while the stream is being captured and they do not exist yet, or
// when creating them fails.
bool ensure_side(moe_ctx* ctx) {
  if (ctx->side) return true;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(ctx->stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return false;
  cudaStream_t s = nullptr;
  cudaEvent_t f = nullptr, j = nullptr;
  if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) return false;
  if (cudaEventCreateWithFlags(&f, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&j, cudaEventDisableTiming) != cudaSuccess) {
    if (f) cudaEventDestroy(f);
    cudaStreamDestroy(s);
    return false;
  }
  ctx->side = s;
  ctx->fork_ev = f;
  ctx->join_ev = j;
  return true;
}

// The GEMV chain and the tcgen05 chain own disjoint experts from gate/up through down
// (both kernels on both projections, with one row threshold): only then may they run on
// two streams. With one projection on a single kernel for all experts, that projection
// reads rows the other chain's first projection writes, so the steps run in order.
bool split_chains(const ExpertPlan& p) {
  return p.tc_gu && p.tc_dn && p.gemv_gu && p.gemv_dn && p.gemv_skip_gu == p.gemv_skip_dn;
}

int run_routed_experts(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts, const void* x,
                       int64_t T, const BlockWs& ws, const ExpertPlan& plan, cudaEvent_t* ev, int act) {
  const int E = cfg->num_experts, H = cfg->hidden, I = cfg->moe_inter, k = cfg->top_k;
  const int64_t P = T * k;
  const int slots = (int)std::min<int64_t>(P, E);
  // Expected rows per expert: how many tokens one GEMV pass over the weights serves.
  const int rows_pe = (int)std::min<int64_t>((P + E - 1) / E, 1 << 20);
  // SwitchGLU gate/up + SiLU*up over grouped rows (x row = pair / k).
  moe::QgemvArgs gu = qgemv_args(wts->gate, &wts->up, I, H);
  gu.x = static_cast<const uint16_t*>(x);
  gu.x_mode = 1;
  gu.x_repeat = k;
  gu.perm = ws.perm;
  gu.offsets = ws.offsets;
  gu.active = ws.active;
  gu.n_active = ws.n_active;
  gu.out = ws.hbuf;
  gu.out_mode = 0;
  gu.partial = ws.gemv_partial;
  gu.partial_bytes = ws.gemv_partial_bytes;
  gu.part_rows = P;
  gu.num_experts_total = E;
  gu.act = act;
  MOE_MARK(ev, kGateUp, ctx->stream);
  // Hybrid step (both paths): the GEMV chain (gate/up -> down) and the tcgen05 chain own
  // disjoint experts and rows, so the tcgen05 chain runs on the side stream, joined back
  // before anything reads its outputs, and its launches (mostly idle CTAs at decode
  // sizes) stay off the GEMV's dependency chain: measured 4-6 us per Qwen3 block at
  // T = 16..96. Sequential under moe_block_profile (stage events) and until the side
  // stream exists.
  const bool fork = ev == nullptr && split_chains(plan) && ensure_side(ctx);
  cudaStream_t tcs = fork ? ctx->side : ctx->stream;
  if (fork) {
    MOE_CUDA(ctx, cudaEventRecord(ctx->fork_ev, ctx->stream));
    MOE_CUDA(ctx, cudaStreamWaitEvent(ctx->side, ctx->fork_ev, 0));
  }
  // GEMV first: at decode sizes it carries the work (sequential form: the mostly idle
  // tcgen05 launch behind it overlaps its tail under programmatic dependent launch).
  if (plan.gemv_gu) {
    gu.max_expert_rows = plan.gemv_skip_gu;
    MOE_CUDA(ctx, moe::launch_qgemv(gu, true, slots, rows_pe, ctx->stream));
  }
  if (plan.tc_gu) {
    moe::TcGemmArgs ta{gu, ws.tile_start, E, plan.max_tiles, ws.status};
    MOE_CUDA(ctx, moe::launch_tc_gemm(ta, true, tcs));
  }

  // down projection over the same grouped rows.
  moe::QgemvArgs dn = qgemv_args(wts->down, nullptr, H, I);
  dn.x = ws.hbuf;
  dn.x_mode = 0;
  dn.perm = ws.perm;
  dn.offsets = ws.offsets;
  dn.active = ws.active;
  dn.n_active = ws.n_active;
  dn.out = ws.ybuf;
  dn.out_mode = 0;
  dn.partial = ws.gemv_partial;
  dn.partial_bytes = ws.gemv_partial_bytes;
  dn.part_rows = P;
  dn.num_experts_total = E;
  MOE_MARK(ev, kDown, ctx->stream);
  if (plan.gemv_dn) {
    dn.max_expert_rows = plan.gemv_skip_dn;
    MOE_CUDA(ctx, moe::launch_qgemv(dn, false, slots, rows_pe, ctx->stream));
  }
  if (plan.tc_dn) {
    moe::TcGemmArgs ta{dn, ws.tile_start, E, plan.max_tiles, ws.status};
    MOE_CUDA(ctx, moe::launch_tc_gemm(ta, false, tcs));
  }
  if (fork) {
    MOE_CUDA(ctx, cudaEventRecord(ctx->join_ev, ctx->side));
    MOE_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, ctx->join_ev, 0));
  }
  return MOE_OK;
}

int run_block(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts, const void* x, int64_t T,
              void* out, cudaEvent_t* ev, const void* residual = nullptr) {
  if (!ctx) return MOE_ERR_INVALID;
  ctx->last_error.clear();
  const char* fn = "moe_block_forward";
  int rc = check_block(ctx, cfg, wts, fn);
  if (rc) return rc;
  if (T < 0 || T > (INT32_MAX / 64)) return fail(ctx, MOE_ERR_INVALID, "%s: bad T", fn);
  if (T == 0) return MOE_OK;
  if (!x || !out || !aligned16(x) || !aligned16(out))
    return fail(ctx, MOE_ERR_INVALID, "%s: x and out must be non-null and 16-byte aligned", fn);
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(ctx, MOE_ERR_CUDA, "cudaSetDevice(%d) failed", ctx->device);
  rc = ensure_scratch(ctx, carve_block(nullptr, cfg, T).bytes);
  if (rc) return rc;
  BlockWs ws = carve_block(ctx->scratch, cfg, T);
  const int E = cfg->num_experts, H = cfg->hidden, I = cfg->moe_inter, k = cfg->top_k;
  const int64_t P = T * k;
  if (decode_fused_ok(cfg, wts, T)) {
    // decode-sized batch: the whole block in one cooperative kernel (decode.cu); under
    // moe_block_profile its time is booked as the gate/up stage
    moe::DecodeArgs d{};
    route_args(cfg, wts, x, T, ws, d.ra, d.ta);
    d.T = (int)T;
    d.H = H;
    d.I = I;
    d.Is = cfg->shared_inter;
    d.k = k;
    auto q = [](const moe_qweight& m, const uint32_t*& w, const uint16_t*& s, const uint16_t*& b) {
      w = m.w;
      s = static_cast<const uint16_t*>(m.scales);
      b = static_cast<const uint16_t*>(m.biases);
    };
    q(wts->gate, d.wg, d.sg, d.bg);
    q(wts->up, d.wu, d.su, d.bu);
    q(wts->down, d.wd, d.sd, d.bd);
    if (d.Is) {
      q(wts->shared_gate, d.swg, d.ssg, d.sbg);
      q(wts->shared_up, d.swu, d.ssu, d.sbu);
      q(wts->shared_down, d.swd, d.ssd, d.sbd);
    }
    d.logits_rep = ws.logits_rep;
    d.hbuf = ws.hbuf;
    d.hsbuf = ws.hs;
    d.residual = static_cast<const uint16_t*>(residual);
    d.out = static_cast<uint16_t*>(out);
    d.barrier = reinterpret_cast<uint32_t*>(ws.status) + kDecodeBarrierWord;
    d.status = ws.status;
    d.n_active = ws.n_active;
    d.has_gate = cfg->shared_inter > 0 && cfg->has_shared_gate;
    d.scale8 = decode_scale8(cfg, wts);
    for (int i = kRouter; i <= kGateUp; ++i) MOE_MARK(ev, i, ctx->stream);
    MOE_CUDA(ctx, moe::launch_decode_block(d, ctx->stream));
    for (int i = kDown; i <= kStages; ++i) MOE_MARK(ev, i, ctx->stream);
    ctx->last_block_fused = true;
    return MOE_OK;
  }
  ctx->last_block_fused = false;
  const ExpertPlan plan = plan_experts(P, E, I, H, T);
  rc = run_route(ctx, cfg, wts, x, T, ws, ev, nullptr, plan.min_rows);
  if (rc) return rc;

  rc = run_routed_experts(ctx, cfg, wts, x, T, ws, plan, ev, 0);
  if (rc) return rc;

  const bool shared = cfg->shared_inter > 0;
  if (!shared) {
    MOE_MARK(ev, kSharedGateUp, ctx->stream);
    MOE_MARK(ev, kSharedDown, ctx->stream);
  }
  if (shared) {
    const int Is = cfg->shared_inter;
    moe::QgemvArgs sgu = qgemv_args(wts->shared_gate, &wts->shared_up, Is, H);
    sgu.x = static_cast<const uint16_t*>(x);
    sgu.x_mode = 0;
    sgu.n_identity = (int)T;
    sgu.out = ws.hs;
    sgu.partial = ws.gemv_partial;
    sgu.partial_bytes = ws.gemv_partial_bytes;
    sgu.part_rows = T;
    MOE_MARK(ev, kSharedGateUp, ctx->stream);
    const int stiles = (int)((T + moe::kTcTileRows - 1) / moe::kTcTileRows);
    if (use_tc(T, 1, Is, H)) {
      moe::TcGemmArgs ta{sgu, nullptr, 1, stiles, ws.status};
      // (not split: the gated partials are twice as wide and measured slower split,
      // 84 us against 49 us for Qwen1.5-MoE at T=512)
      MOE_CUDA(ctx, moe::launch_tc_gemm(ta, true, ctx->stream));
    } else {
      MOE_CUDA(ctx, moe::launch_qgemv(sgu, true, 1, (int)T, ctx->stream));
    }
    moe::QgemvArgs sdn = qgemv_args(wts->shared_down, nullptr, H, Is);
    sdn.x = ws.hs;
    sdn.x_mode = 0;
    sdn.n_identity = (int)T;
    sdn.out = ws.ys;
    sdn.partial = ws.gemv_partial;
    sdn.partial_bytes = ws.gemv_partial_bytes;
    sdn.part_rows = T;
    MOE_MARK(ev, kSharedDown, ctx->stream);
    if (use_tc(T, 1, H, Is)) {
      moe::TcGemmArgs ta{sdn, nullptr, 1, stiles, ws.status};
      ta.q.partial = ws.tc_partial;
      ta.q.partial_bytes = ws.tc_partial_bytes;
      ta.ksplit = tc_ksplit((H % 256 == 0 ? H / 256 : H / 128) * stiles, Is / 64, T, H, ws.tc_partial_bytes);
      MOE_CUDA(ctx, moe::launch_tc_gemm(ta, false, ctx->stream));
    } else {
      MOE_CUDA(ctx, moe::launch_qgemv(sdn, false, 1, (int)T, ctx->stream));
    }
  }

  moe::CombineArgs ca{};
  ca.y = ws.ybuf;
  ca.inv = ws.inv;
  ca.weights = ws.wsel;
  ca.shared = shared ? ws.ys : nullptr;
  ca.gate_val = (shared && cfg->has_shared_gate) ? ws.gate_val : nullptr;
  ca.residual = static_cast<const uint16_t*>(residual);
  ca.T = (int)T;
  ca.k = k;
  ca.H = H;
  ca.out = static_cast<uint16_t*>(out);
  MOE_MARK(ev, kCombine, ctx->stream);
  MOE_CUDA(ctx, moe::launch_combine(ca, ctx->stream));
  MOE_MARK(ev, kStages, ctx->stream);
  return MOE_OK;
}

}  // namespace

// Argument checks shared by moe_gather_qmm and moe_gather_qmm_noalloc (same codes and
// order: quantization, transpose, shapes, pointers); MOE_OK for a valid call, including
// batch == 0, which computes nothing.
namespace moe_internal {
int check_gather(moe_ctx* ctx, const char* fn, const void* x, int64_t K, int64_t x_repeat,
                 const uint32_t* lhs_indices, const uint32_t* w, const void* scales, int64_t num_experts,
                 int64_t N, const uint32_t* rhs_indices, int64_t batch, int transpose, int group_size, int bits,
                 const void* out) {
  int rc = check_quant(ctx, fn, K, group_size, bits);
  if (rc) return rc;
  if (!transpose) return fail(ctx, MOE_ERR_UNSUPPORTED, "%s: transpose=false is not implemented", fn);
  if (batch < 0 || N <= 0 || N > INT32_MAX || num_experts <= 0 || num_experts > 4096 || batch > INT32_MAX)
    return fail(ctx, MOE_ERR_INVALID, "%s: bad batch/N/num_experts", fn);
  if (!lhs_indices && x_repeat <= 0) return fail(ctx, MOE_ERR_INVALID, "%s: x_repeat must be positive", fn);
  if (batch == 0) return MOE_OK;
  if (!x || !w || !scales || !rhs_indices || !out) return fail(ctx, MOE_ERR_INVALID, "%s: null pointer", fn);
  if (!aligned16(x) || !aligned16(w)) return fail(ctx, MOE_ERR_INVALID, "%s: x and w must be 16-byte aligned", fn);
  return MOE_OK;
}
}  // namespace moe_internal

extern "C" {

int moe_abi_version(void) { return MOE_B200_ABI_VERSION; }

int moe_ctx_create(int device, void* stream, moe_ctx** out) {
  if (!out) return MOE_ERR_INVALID;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return MOE_ERR_CUDA;
  moe_ctx* c = new (std::nothrow) moe_ctx();
  if (!c) return MOE_ERR_NO_MEMORY;
  c->device = device;
  c->stream = static_cast<cudaStream_t>(stream);
  *out = c;
  return MOE_OK;
}

void moe_ctx_destroy(moe_ctx* ctx) {
  if (!ctx) return;
  if (ctx->scratch || ctx->side) {
    DeviceGuard g(ctx->device);
    if (ctx->scratch) cudaFree(ctx->scratch);
    if (ctx->side) cudaStreamDestroy(ctx->side);
    if (ctx->fork_ev) cudaEventDestroy(ctx->fork_ev);
    if (ctx->join_ev) cudaEventDestroy(ctx->join_ev);
  }
  delete ctx;
}

int moe_ctx_set_stream(moe_ctx* ctx, void* stream) {
  if (!ctx) return MOE_ERR_INVALID;
  ctx->stream = static_cast<cudaStream_t>(stream);
  return MOE_OK;
}

const char* moe_last_error(const moe_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

int moe_ctx_reserve(moe_ctx* ctx, const moe_block_config* cfg, int64_t max_tokens) {
  if (!ctx) return MOE_ERR_INVALID;
  ctx->last_error.clear();
  if (!cfg || max_tokens < 0) return fail(ctx, MOE_ERR_INVALID, "moe_ctx_reserve: bad arguments");
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(ctx, MOE_ERR_CUDA, "cudaSetDevice(%d) failed", ctx->device);
  return ensure_scratch(ctx, carve_block(nullptr, cfg, max_tokens).bytes);
}

int moe_quantized_matmul(moe_ctx* ctx, const void* x, int64_t M, int64_t K, const uint32_t* w,
                         const void* scales, const void* biases, int64_t N, int transpose, int group_size,
                         int bits, void* out) {
  if (!ctx) return MOE_ERR_INVALID;
  ctx->last_error.clear();
  const char* fn = "moe_quantized_matmul";
  int rc = check_quant(ctx, fn, K, group_size, bits);
  if (rc) return rc;
  if (!transpose) return fail(ctx, MOE_ERR_UNSUPPORTED, "%s: transpose=false is not implemented", fn);
  if (M < 0 || N <= 0 || N > INT32_MAX || M > INT32_MAX) return fail(ctx, MOE_ERR_INVALID, "%s: bad M/N", fn);
  if (M == 0) return MOE_OK;
  if (!x || !w || !scales || !out) return fail(ctx, MOE_ERR_INVALID, "%s: null pointer", fn);
  if (!aligned16(x) || !aligned16(w)) return fail(ctx, MOE_ERR_INVALID, "%s: x and w must be 16-byte aligned", fn);
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(ctx, MOE_ERR_CUDA, "cudaSetDevice(%d) failed", ctx->device);
  moe_qweight m{w, scales, biases};
  moe::QgemvArgs q = qgemv_args(m, nullptr, (int)N, (int)K);
  q.x = static_cast<const uint16_t*>(x);
  q.x_mode = 0;
  q.n_identity = (int)M;
  q.out = static_cast<uint16_t*>(out);
  if (use_tc(M, 1, (int)N, (int)K)) {
    // many rows: the tcgen05 GEMM, as the block's shared expert (one "expert", token
    // tiles in order); the context's status word records an expired bounded wait
    rc = ensure_scratch(ctx, 256);
    if (rc) return rc;
    moe::TcGemmArgs ta{q, nullptr, 1, (int)((M + moe::kTcTileRows - 1) / moe::kTcTileRows),
                       static_cast<int32_t*>(ctx->scratch)};
    MOE_CUDA(ctx, moe::launch_tc_gemm(ta, false, ctx->stream));
    return MOE_OK;
  }
  MOE_CUDA(ctx, moe::launch_qgemv(q, false, 1, (int)std::min<int64_t>(M, 1 << 20), ctx->stream));
  return MOE_OK;
}

int moe_gather_qmm(moe_ctx* ctx, const void* x, int64_t x_rows, int64_t K, int64_t x_repeat,
                   const uint32_t* lhs_indices, const uint32_t* w, const void* scales, const void* biases,
                   int64_t num_experts, int64_t N, const uint32_t* rhs_indices, int64_t batch, int transpose,
                   int group_size, int bits, int sorted_indices, void* out) {
  (void)sorted_indices;
  (void)x_rows;
  if (!ctx) return MOE_ERR_INVALID;
  ctx->last_error.clear();
  int rc = moe_internal::check_gather(ctx, "moe_gather_qmm", x, K, x_repeat, lhs_indices, w, scales, num_experts, N,
                                      rhs_indices, batch, transpose, group_size, bits, out);
  if (rc || batch == 0) return rc;
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(ctx, MOE_ERR_CUDA, "cudaSetDevice(%d) failed", ctx->device);

  const int E = (int)num_experts;
  const int seg = moe::group_seg(batch, E);
  const int64_t nseg = std::max<int64_t>(1, (batch + seg - 1) / seg);
  auto carve = [&](void* base, moe::GroupArgs& ga, int32_t*& status) {
    Carve cv(base);
    status = cv.take<int32_t>(64);  // the context's status word, at offset 0
    ga.hist = cv.take<int32_t>(nseg * E);
    ga.segbase = cv.take<int32_t>(nseg * E);
    ga.offsets = cv.take<int32_t>(E + 1);
    ga.active = cv.take<int32_t>(E);
    ga.n_active = cv.take<int32_t>(1);
    ga.tile_start = cv.take<int32_t>(E + 1);
    ga.perm = cv.take<uint32_t>(batch);
    return cv.off + 256;
  };
  moe::GatherCall gc{};
  rc = ensure_scratch(ctx, carve(nullptr, gc.g, gc.status));
  if (rc) return rc;
  carve(ctx->scratch, gc.g, gc.status);
  gc.g.seg = seg;
  gc.g.nseg = (int)nseg;
  gc.x = static_cast<const uint16_t*>(x);
  gc.x_mode = lhs_indices ? 2 : 1;
  gc.x_repeat = (int)std::max<int64_t>(1, x_repeat);
  gc.lhs = lhs_indices;
  gc.w = w;
  gc.s = static_cast<const uint16_t*>(scales);
  gc.b = static_cast<const uint16_t*>(biases);
  gc.E = E;
  gc.N = (int)N;
  gc.K = (int)K;
  gc.batch = batch;
  gc.rhs = rhs_indices;
  gc.out = static_cast<uint16_t*>(out);
  MOE_CUDA(ctx, moe::launch_gather_qmm(gc, ctx->stream));
  return MOE_OK;
}

int moe_fast_rms_norm(moe_ctx* ctx, const void* x, const void* weight, float eps, int64_t rows, int64_t dim,
                      void* out) {
  if (!ctx) return MOE_ERR_INVALID;
  ctx->last_error.clear();
  if (rows < 0 || dim <= 0 || dim % 8 != 0 || dim > INT32_MAX)
    return fail(ctx, MOE_ERR_INVALID, "moe_fast_rms_norm: dim=%lld must be a positive multiple of 8", (long long)dim);
  if (rows == 0) return MOE_OK;
  if (!x || !weight || !out || !aligned16(x) || !aligned16(weight) || !aligned16(out))
    return fail(ctx, MOE_ERR_INVALID, "moe_fast_rms_norm: pointers must be non-null and 16-byte aligned");
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(ctx, MOE_ERR_CUDA, "cudaSetDevice(%d) failed", ctx->device);
  MOE_CUDA(ctx, moe::launch_rms_norm(static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(weight), eps, rows,
                                     (int)dim, static_cast<uint16_t*>(out), ctx->stream));
  return MOE_OK;
}

int moe_block_route(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts, const void* x,
                    int64_t T, uint32_t* idx, void* weights, int32_t* offsets, uint32_t* perm) {
  if (!ctx) return MOE_ERR_INVALID;
  ctx->last_error.clear();
  int rc = check_block(ctx, cfg, wts, "moe_block_route");
  if (rc) return rc;
  if (T < 0 || T > (INT32_MAX / 64)) return fail(ctx, MOE_ERR_INVALID, "moe_block_route: bad T");
  if (T == 0) return MOE_OK;
  if (!x || !aligned16(x)) return fail(ctx, MOE_ERR_INVALID, "moe_block_route: x must be 16-byte aligned");
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(ctx, MOE_ERR_CUDA, "cudaSetDevice(%d) failed", ctx->device);
  rc = ensure_scratch(ctx, carve_block(nullptr, cfg, T).bytes);
  if (rc) return rc;
  BlockWs ws = carve_block(ctx->scratch, cfg, T);
  rc = run_route(ctx, cfg, wts, x, T, ws);
  if (rc) return rc;
  const int64_t P = T * cfg->top_k;
  if (idx) MOE_CUDA(ctx, cudaMemcpyAsync(idx, ws.idx, P * 4, cudaMemcpyDeviceToDevice, ctx->stream));
  if (weights) MOE_CUDA(ctx, cudaMemcpyAsync(weights, ws.wsel, P * 2, cudaMemcpyDeviceToDevice, ctx->stream));
  if (offsets)
    MOE_CUDA(ctx, cudaMemcpyAsync(offsets, ws.offsets, (cfg->num_experts + 1) * 4, cudaMemcpyDeviceToDevice,
                                  ctx->stream));
  if (perm) MOE_CUDA(ctx, cudaMemcpyAsync(perm, ws.perm, P * 4, cudaMemcpyDeviceToDevice, ctx->stream));
  return MOE_OK;
}

int moe_block_router_logits(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts,
                            const void* x, int64_t T, void* logits) {
  if (!ctx) return MOE_ERR_INVALID;
  ctx->last_error.clear();
  const char* fn = "moe_block_router_logits";
  if (!cfg) return fail(ctx, MOE_ERR_INVALID, "%s: null config", fn);
  int rc = check_quant(ctx, fn, cfg->hidden, cfg->group_size, cfg->bits);
  if (rc) return rc;
  if (cfg->num_experts <= 0 || cfg->num_experts > 512)
    return fail(ctx, MOE_ERR_UNSUPPORTED, "%s: num_experts=%d (supported 1..512)", fn, cfg->num_experts);
  if (!wts || !wts->router.w || !wts->router.scales || !aligned16(wts->router.w))
    return fail(ctx, MOE_ERR_INVALID, "%s: router weight missing or not 16-byte aligned", fn);
  const bool gate_row = cfg->shared_inter > 0 && cfg->has_shared_gate;
  if (gate_row && (!wts->shared_expert_gate.w || !wts->shared_expert_gate.scales ||
                   !aligned16(wts->shared_expert_gate.w)))
    return fail(ctx, MOE_ERR_INVALID, "%s: shared_expert_gate weight missing or not 16-byte aligned", fn);
  if (T < 0 || T > (INT32_MAX / 64)) return fail(ctx, MOE_ERR_INVALID, "%s: bad T", fn);
  if (T == 0) return MOE_OK;
  if (!x || !logits || !aligned16(x)) return fail(ctx, MOE_ERR_INVALID, "%s: x (16-byte aligned) and logits required", fn);
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(ctx, MOE_ERR_CUDA, "cudaSetDevice(%d) failed", ctx->device);
  BlockWs ws{};
  ws.logits = static_cast<uint16_t*>(logits);
  moe::RouterArgs ra;
  moe::TopkArgs ta;
  route_args(cfg, wts, x, T, ws, ra, ta);
  MOE_CUDA(ctx, moe::launch_router(ra, ctx->stream));
  return MOE_OK;
}

int moe_block_forward(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts, const void* x,
                      int64_t T, void* out) {
  return run_block(ctx, cfg, wts, x, T, out, nullptr);
}

int moe_gemma4_block_forward(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts,
                             const void* router_scale, const void* per_expert_scale, const void* x, int64_t T,
                             float* out, uint32_t* idx_out, float* weights_out) {
  if (!ctx) return MOE_ERR_INVALID;
  ctx->last_error.clear();
  const char* fn = "moe_gemma4_block_forward";
  if (!cfg) return fail(ctx, MOE_ERR_INVALID, "%s: null config", fn);
  moe_block_config c = *cfg;  // scoring, renormalisation and gate are fixed by the variant
  c.scoring = MOE_SCORING_SOFTMAX;
  c.norm_topk_prob = 1;
  c.has_shared_gate = 0;
  if (c.shared_inter != 0)
    return fail(ctx, MOE_ERR_UNSUPPORTED, "%s: the Gemma4 block has no shared expert (shared_inter=%d)", fn,
                c.shared_inter);
  int rc = check_block(ctx, &c, wts, fn);
  if (rc) return rc;
  if (T < 0 || T > (INT32_MAX / 64)) return fail(ctx, MOE_ERR_INVALID, "%s: bad T", fn);
  if (T == 0) return MOE_OK;
  if (!x || !out || !router_scale || !per_expert_scale || !aligned16(x) || !aligned16(out) ||
      !aligned16(router_scale))
    return fail(ctx, MOE_ERR_INVALID, "%s: x, out, router_scale (16-byte aligned) and per_expert_scale required",
                fn);
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(ctx, MOE_ERR_CUDA, "cudaSetDevice(%d) failed", ctx->device);
  const int E = c.num_experts, H = c.hidden, k = c.top_k;
  // the block workspace, then the router's f32 input rows, f32 logits and f32 weights
  auto carve = [&](void* base, BlockWs& ws, float*& hf, float*& lf, float*& wf) {
    ws = carve_block(base, &c, T);
    Carve cv(base);
    cv.off = ws.bytes;
    hf = cv.take<float>((size_t)T * H);
    lf = cv.take<float>((size_t)T * E);
    wf = cv.take<float>((size_t)T * k);
    return cv.off + 256;
  };
  BlockWs ws;
  float *hf, *lf, *wf;
  rc = ensure_scratch(ctx, carve(nullptr, ws, hf, lf, wf));
  if (rc) return rc;
  carve(ctx->scratch, ws, hf, lf, wf);
  const int64_t P = T * k;
  // router input: RMSNorm(x) (unit weight, eps 1e-6) * hidden^-0.5 * scale, in f32
  const float root = (float)(1.0 / std::sqrt((double)H));
  MOE_CUDA(ctx, moe::launch_gemma_router_input(static_cast<const uint16_t*>(x),
                                               static_cast<const uint16_t*>(router_scale), root, 1e-6f, T, H, hf,
                                               ctx->stream));
  moe::RouterArgs ra{};
  moe::TopkArgs ta{};
  route_args(&c, wts, x, T, ws, ra, ta);
  ra.xf = hf;
  ra.logits_f32 = lf;
  MOE_CUDA(ctx, moe::launch_router(ra, ctx->stream));
  ta.scoring = 3;
  ta.logits_f32 = lf;
  ta.per_expert_scale = static_cast<const uint16_t*>(per_expert_scale);
  ta.weights_f32 = wf;
  ta.idx = ws.idx;
  ta.weights = nullptr;
  MOE_CUDA(ctx, moe::launch_topk(ta, ctx->stream));
  const ExpertPlan plan = plan_experts(P, E, c.moe_inter, H, T);
  moe::GroupArgs ga{};
  ga.key = ws.idx;
  ga.P = P;
  ga.E = E;
  ga.seg = moe::group_seg(P, E);
  ga.nseg = (int)std::max<int64_t>(1, (P + ga.seg - 1) / ga.seg);
  ga.hist = ws.hist;
  ga.segbase = ws.segbase;
  ga.offsets = ws.offsets;
  ga.active = ws.active;
  ga.n_active = ws.n_active;
  ga.perm = ws.perm;
  ga.inv = ws.inv;
  ga.tile_start = ws.tile_start;
  ga.tile_rows = moe::kTcTileRows;
  ga.tc_min_rows = plan.min_rows;
  MOE_CUDA(ctx, moe::launch_group(ga, ctx->stream));
  rc = run_routed_experts(ctx, &c, wts, x, T, ws, plan, nullptr, 1);
  if (rc) return rc;
  moe::CombineArgs ca{};
  ca.y = ws.ybuf;
  ca.inv = ws.inv;
  ca.weights_f32 = wf;
  ca.out_f32 = out;
  ca.T = (int)T;
  ca.k = k;
  ca.H = H;
  MOE_CUDA(ctx, moe::launch_combine(ca, ctx->stream));
  if (idx_out) MOE_CUDA(ctx, cudaMemcpyAsync(idx_out, ws.idx, P * 4, cudaMemcpyDeviceToDevice, ctx->stream));
  if (weights_out) MOE_CUDA(ctx, cudaMemcpyAsync(weights_out, wf, P * 4, cudaMemcpyDeviceToDevice, ctx->stream));
  return MOE_OK;
}

int moe_layer_ffn_forward(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts,
                          const void* x, int64_t T, const void* norm_weight, float eps, void* normed,
                          void* out) {
  if (!ctx) return MOE_ERR_INVALID;
  ctx->last_error.clear();
  const char* fn = "moe_layer_ffn_forward";
  int rc = check_block(ctx, cfg, wts, fn);
  if (rc) return rc;
  if (T < 0 || T > (INT32_MAX / 64)) return fail(ctx, MOE_ERR_INVALID, "%s: bad T", fn);
  if (T == 0) return MOE_OK;
  if (!x || !out || !norm_weight || !aligned16(x) || !aligned16(out) || !aligned16(norm_weight) ||
      (normed && !aligned16(normed)))
    return fail(ctx, MOE_ERR_INVALID, "%s: x, norm_weight, out (and normed) must be non-null and 16-byte aligned",
                fn);
  const size_t row_bytes = (size_t)T * cfg->hidden * 2;
  auto overlaps = [](const void* a, const void* b, size_t n) {
    const char* p = static_cast<const char*>(a);
    const char* q = static_cast<const char*>(b);
    return p < q + n && q < p + n;
  };
  if (overlaps(x, out, row_bytes) || (normed && (overlaps(normed, out, row_bytes) || overlaps(normed, x, row_bytes))))
    return fail(ctx, MOE_ERR_INVALID, "%s: x, normed and out must not overlap", fn);
  if (!(eps >= 0.0f)) return fail(ctx, MOE_ERR_INVALID, "%s: eps must be >= 0", fn);
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(ctx, MOE_ERR_CUDA, "cudaSetDevice(%d) failed", ctx->device);
  rc = ensure_scratch(ctx, carve_block(nullptr, cfg, T).bytes);
  if (rc) return rc;
  uint16_t* h = normed ? static_cast<uint16_t*>(normed) : carve_block(ctx->scratch, cfg, T).xnorm;
  MOE_CUDA(ctx, moe::launch_rms_norm(static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(norm_weight),
                                     eps, T, cfg->hidden, h, ctx->stream));
  return run_block(ctx, cfg, wts, h, T, out, nullptr, x);
}

int moe_block_profile(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts, const void* x,
                      int64_t T, void* out, float* stage_ms, int32_t* n_active) {
  if (!ctx) return MOE_ERR_INVALID;
  if (!stage_ms) return fail(ctx, MOE_ERR_INVALID, "moe_block_profile: stage_ms is null");
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(ctx, MOE_ERR_CUDA, "cudaSetDevice(%d) failed", ctx->device);
  cudaEvent_t ev[kStages + 1] = {};
  for (int i = 0; i <= kStages; ++i) MOE_CUDA(ctx, cudaEventCreate(&ev[i]));
  int rc = run_block(ctx, cfg, wts, x, T, out, T > 0 ? ev : nullptr);
  if (rc == MOE_OK && T > 0) {
    cudaError_t e = cudaEventSynchronize(ev[kStages]);
    if (ctx->last_block_fused) {
      // one launch: its whole device time is the gate/up stage, the others are zero
      for (int i = 0; i < kStages; ++i) stage_ms[i] = 0.0f;
      e = cudaEventElapsedTime(&stage_ms[kGateUp], ev[kRouter], ev[kStages]);
    } else {
      for (int i = 0; i < kStages && e == cudaSuccess; ++i) e = cudaEventElapsedTime(&stage_ms[i], ev[i], ev[i + 1]);
    }
    if (e != cudaSuccess) rc = fail(ctx, MOE_ERR_CUDA, "moe_block_profile: %s", cudaGetErrorString(e));
    if (rc == MOE_OK) {
      BlockWs ws = carve_block(ctx->scratch, cfg, T);
      int32_t st = 0;
      e = cudaMemcpy(&st, ws.status, sizeof(int32_t), cudaMemcpyDeviceToHost);
      if (e == cudaSuccess && n_active) e = cudaMemcpy(n_active, ws.n_active, sizeof(int32_t), cudaMemcpyDeviceToHost);
      if (e != cudaSuccess) rc = fail(ctx, MOE_ERR_CUDA, "moe_block_profile: %s", cudaGetErrorString(e));
      else if (st != 0) rc = fail(ctx, MOE_ERR_TIMEOUT, "moe_block_profile: a bounded device wait expired (status %d)", st);
    }
  } else if (rc == MOE_OK) {
    for (int i = 0; i < kStages; ++i) stage_ms[i] = 0.0f;
    if (n_active) *n_active = 0;
  }
  for (int i = 0; i <= kStages; ++i) cudaEventDestroy(ev[i]);
  return rc;
}

// ---------------------------------------------------------------------------------
// Expert parallelism
// ---------------------------------------------------------------------------------

int moe_ep_route(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts, const void* x,
                 int64_t T, uint32_t* packed) {
  if (!ctx) return MOE_ERR_INVALID;
  ctx->last_error.clear();
  const char* fn = "moe_ep_route";
  int rc = check_route(ctx, cfg, wts, fn);
  if (rc) return rc;
  if (T < 0 || T > (INT32_MAX / 64)) return fail(ctx, MOE_ERR_INVALID, "%s: bad T", fn);
  if (T == 0) return MOE_OK;
  if (!x || !packed || !aligned16(x)) return fail(ctx, MOE_ERR_INVALID, "%s: x must be 16-byte aligned, packed non-null", fn);
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(ctx, MOE_ERR_CUDA, "cudaSetDevice(%d) failed", ctx->device);
  rc = ensure_scratch(ctx, carve_route(nullptr, cfg, T).bytes);
  if (rc) return rc;
  return run_route(ctx, cfg, wts, x, T, carve_route(ctx->scratch, cfg, T), nullptr, packed);
}

namespace {
// moe_ep_experts / moe_ep_experts_bf16: partial sums into partial (fp32) or partial_bf16.
int ep_experts(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts, const void* x_all,
               int64_t T_all, const uint32_t* packed_all, int32_t expert_begin, int32_t num_local, float* partial_f32,
               uint16_t* partial_bf16, const char* fn) {
  void* partial = partial_f32 ? static_cast<void*>(partial_f32) : static_cast<void*>(partial_bf16);
  if (!ctx) return MOE_ERR_INVALID;
  ctx->last_error.clear();
  int rc = check_experts(ctx, cfg, wts, fn);
  if (rc) return rc;
  if (num_local <= 0 || expert_begin < 0 || (int64_t)expert_begin + num_local > cfg->num_experts)
    return fail(ctx, MOE_ERR_INVALID, "%s: experts [%d, %d + %d) outside [0, %d)", fn, expert_begin, expert_begin,
                num_local, cfg->num_experts);
  if (T_all < 0 || T_all > (INT32_MAX / 64)) return fail(ctx, MOE_ERR_INVALID, "%s: bad T_all", fn);
  if (T_all == 0) return MOE_OK;
  if (!x_all || !packed_all || !partial || !aligned16(x_all) || !aligned16(partial))
    return fail(ctx, MOE_ERR_INVALID, "%s: x_all and partial must be non-null and 16-byte aligned", fn);
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(ctx, MOE_ERR_CUDA, "cudaSetDevice(%d) failed", ctx->device);
  rc = ensure_scratch(ctx, carve_ep(nullptr, cfg, T_all, num_local).bytes);
  if (rc) return rc;
  const EpWs ws = carve_ep(ctx->scratch, cfg, T_all, num_local);
  const int E = cfg->num_experts, El = num_local, H = cfg->hidden, I = cfg->moe_inter, k = cfg->top_k;
  const int64_t P = T_all * k;

  moe::GroupArgs ga{};
  ga.key = packed_all;
  ga.key_packed = 1;
  ga.key_base = (uint32_t)expert_begin;
  ga.P = P;
  ga.E = El;
  ga.seg = moe::group_seg(P, El);
  ga.nseg = (int)std::max<int64_t>(1, (P + ga.seg - 1) / ga.seg);
  ga.hist = ws.hist;
  ga.segbase = ws.segbase;
  ga.offsets = ws.offsets;
  ga.active = ws.active;
  ga.n_active = ws.n_active;
  ga.perm = ws.perm;
  ga.inv = ws.inv;
  // Path choice per expert as in moe_block_forward, on the expected rows per expert of
  // all pairs over all E experts; the grids cover every local pair in the worst case
  // and idle CTAs leave at once.
  ExpertPlan plan = plan_experts(P, E, I, H, T_all);
  plan.max_tiles = (int)(P / moe::kTcTileRows +
                         std::min<int64_t>(El, plan.min_rows ? P / plan.min_rows : P) + 1);
  ga.tile_start = ws.tile_start;
  ga.tile_rows = moe::kTcTileRows;
  ga.tc_min_rows = plan.min_rows;
  MOE_CUDA(ctx, moe::launch_group(ga, ctx->stream));
  const int slots = (int)std::min<int64_t>(P, El);
  const int rows_pe = (int)std::min<int64_t>((P + E - 1) / E, 1 << 20);
  moe::QgemvArgs gu = qgemv_args(wts->gate, &wts->up, I, H);
  gu.x = static_cast<const uint16_t*>(x_all);
  gu.x_mode = 1;
  gu.x_repeat = k;
  gu.perm = ws.perm;
  gu.offsets = ws.offsets;
  gu.active = ws.active;
  gu.n_active = ws.n_active;
  gu.out = ws.hbuf;
  gu.partial = ws.gemv_partial;
  gu.partial_bytes = ws.gemv_partial_bytes;
  gu.part_rows = P;
  gu.num_experts_total = El;
  // hybrid step: the tcgen05 chain on the side stream, as in run_routed_experts
  const bool fork = split_chains(plan) && ensure_side(ctx);
  cudaStream_t tcs = fork ? ctx->side : ctx->stream;
  if (fork) {
    MOE_CUDA(ctx, cudaEventRecord(ctx->fork_ev, ctx->stream));
    MOE_CUDA(ctx, cudaStreamWaitEvent(ctx->side, ctx->fork_ev, 0));
  }
  if (plan.gemv_gu) {
    gu.max_expert_rows = plan.gemv_skip_gu;
    MOE_CUDA(ctx, moe::launch_qgemv(gu, true, slots, rows_pe, ctx->stream));
  }
  if (plan.tc_gu) {
    moe::TcGemmArgs ta{gu, ws.tile_start, El, plan.max_tiles, ws.status};
    MOE_CUDA(ctx, moe::launch_tc_gemm(ta, true, tcs));
  }
  moe::QgemvArgs dn = qgemv_args(wts->down, nullptr, H, I);
  dn.x = ws.hbuf;
  dn.x_mode = 0;
  dn.perm = ws.perm;
  dn.offsets = ws.offsets;
  dn.active = ws.active;
  dn.n_active = ws.n_active;
  dn.out = ws.ybuf;
  dn.partial = ws.gemv_partial;
  dn.partial_bytes = ws.gemv_partial_bytes;
  dn.part_rows = P;
  dn.num_experts_total = El;
  if (plan.gemv_dn) {
    dn.max_expert_rows = plan.gemv_skip_dn;
    MOE_CUDA(ctx, moe::launch_qgemv(dn, false, slots, rows_pe, ctx->stream));
  }
  if (plan.tc_dn) {
    moe::TcGemmArgs ta{dn, ws.tile_start, El, plan.max_tiles, ws.status};
    MOE_CUDA(ctx, moe::launch_tc_gemm(ta, false, tcs));
  }
  if (fork) {
    MOE_CUDA(ctx, cudaEventRecord(ctx->join_ev, ctx->side));
    MOE_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, ctx->join_ev, 0));
  }
  moe::EpPartialArgs pa{};
  pa.y = ws.ybuf;
  pa.inv = ws.inv;
  pa.packed = packed_all;
  pa.e0 = (uint32_t)expert_begin;
  pa.E_l = El;
  pa.T = (int)T_all;
  pa.k = k;
  pa.H = H;
  pa.partial = partial_f32;
  pa.partial_bf16 = partial_bf16;
  MOE_CUDA(ctx, moe::launch_ep_partial(pa, ctx->stream));
  return MOE_OK;
}
}  // namespace

int moe_ep_experts(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts, const void* x_all,
                   int64_t T_all, const uint32_t* packed_all, int32_t expert_begin, int32_t num_local,
                   float* partial) {
  return ep_experts(ctx, cfg, wts, x_all, T_all, packed_all, expert_begin, num_local, partial, nullptr,
                    "moe_ep_experts");
}

int moe_ep_experts_bf16(moe_ctx* ctx, const moe_block_config* cfg, const moe_block_weights* wts, const void* x_all,
                        int64_t T_all, const uint32_t* packed_all, int32_t expert_begin, int32_t num_local,
                        void* partial) {
  return ep_experts(ctx, cfg, wts, x_all, T_all, packed_all, expert_begin, num_local, nullptr,
                    static_cast<uint16_t*>(partial), "moe_ep_experts_bf16");
}

namespace {
int ep_finish(moe_ctx* ctx, const void* partials, bool bf16, int32_t world, int64_t rows, int64_t hidden, void* out,
              const void* norm_weight, float eps, void* normed, const char* fn) {
  if (!ctx) return MOE_ERR_INVALID;
  ctx->last_error.clear();
  if (world <= 0 || rows < 0 || hidden <= 0 || hidden % 8 != 0 || hidden > INT32_MAX)
    return fail(ctx, MOE_ERR_INVALID, "%s: bad world/rows/hidden (hidden a positive multiple of 8)", fn);
  if (rows == 0) return MOE_OK;
  if (!partials || !out || !aligned16(partials) || !aligned16(out))
    return fail(ctx, MOE_ERR_INVALID, "%s: partials and out must be non-null and 16-byte aligned", fn);
  if ((norm_weight == nullptr) != (normed == nullptr))
    return fail(ctx, MOE_ERR_INVALID, "%s: norm_weight and normed go together", fn);
  if (norm_weight && (!aligned16(norm_weight) || !aligned16(normed)))
    return fail(ctx, MOE_ERR_INVALID, "%s: norm_weight and normed must be 16-byte aligned", fn);
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(ctx, MOE_ERR_CUDA, "cudaSetDevice(%d) failed", ctx->device);
  if (bf16)
    MOE_CUDA(ctx, moe::launch_ep_finish_bf16(static_cast<const uint16_t*>(partials), world, rows, (int)hidden,
                                             static_cast<uint16_t*>(out), static_cast<const uint16_t*>(norm_weight),
                                             eps, static_cast<uint16_t*>(normed), ctx->stream));
  else
    MOE_CUDA(ctx, moe::launch_ep_finish(static_cast<const float*>(partials), world, rows, (int)hidden,
                                        static_cast<uint16_t*>(out), static_cast<const uint16_t*>(norm_weight), eps,
                                        static_cast<uint16_t*>(normed), ctx->stream));
  return MOE_OK;
}
}  // namespace

int moe_ep_finish(moe_ctx* ctx, const float* partials, int32_t world, int64_t rows, int64_t hidden, void* out,
                  const void* norm_weight, float eps, void* normed) {
  return ep_finish(ctx, partials, false, world, rows, hidden, out, norm_weight, eps, normed, "moe_ep_finish");
}

int moe_ep_finish_bf16(moe_ctx* ctx, const void* partials, int32_t world, int64_t rows, int64_t hidden, void* out,
                       const void* norm_weight, float eps, void* normed) {
  return ep_finish(ctx, partials, true, world, rows, hidden, out, norm_weight, eps, normed, "moe_ep_finish_bf16");
}

int moe_ctx_status(moe_ctx* ctx, int32_t* status) {
  if (!ctx || !status) return MOE_ERR_INVALID;
  *status = 0;
  if (!ctx->scratch) return MOE_OK;
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(ctx, MOE_ERR_CUDA, "cudaSetDevice(%d) failed", ctx->device);
  MOE_CUDA(ctx, cudaMemcpyAsync(status, ctx->scratch, sizeof(int32_t), cudaMemcpyDeviceToHost, ctx->stream));
  MOE_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  return MOE_OK;
}

}  // extern "C"

namespace moe {
bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("MOE_B200_PDL");
    return !(v && std::strcmp(v, "0") == 0);
  }();
  return on;
}
}  // namespace moe

// Accessors for moe_gather_qmm_noalloc (api_noalloc.cu), which must not reach the
// context's scratch.
namespace moe_internal {
int ctx_device(const moe_ctx* ctx) { return ctx->device; }
void* ctx_stream(const moe_ctx* ctx) { return ctx->stream; }
void ctx_set_error(moe_ctx* ctx, const char* msg) { ctx->last_error = msg; }
}  // namespace moe_internal

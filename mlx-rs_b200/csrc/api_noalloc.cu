// api_noalloc.cu — moe_gather_qmm_noalloc: gather_qmm without any device allocation.
//
// moe_gather_qmm groups its rows by expert in scratch memory that the context
// allocates with cudaMalloc on first use. Some callers cannot let a library allocate
// device memory: a host framework whose own allocator has already reserved the GPU's
// memory (a caching allocator or an MLX-style heap that owns HBM, where a foreign
// cudaMalloc either fails or fragments it), or a latency-critical decode loop in which
// cudaMalloc/cudaFree, which may synchronise the device, are not allowed. This entry
// point serves them: its scratch is a fixed array in the library's device image, so
// the call allocates nothing; the caller still passes x, the weights, the indices and
// the output buffer.
//
// Limits: batch <= MOE_NOALLOC_MAX_BATCH rows and num_experts <= MOE_NOALLOC_MAX_EXPERTS
// (the array below is sized for exactly that, 64 KiB per GPU that loads the library,
// held until the process exits); larger calls are rejected with MOE_ERR_INVALID.
//
// Kernels: the same launch sequence as moe_gather_qmm (moe::launch_gather_qmm: the
// grouping, then the GEMV and, for experts with many rows, the tcgen05 GEMM, with the
// same per-call choices), so both entry points give bit-identical outputs. The one
// difference: the tcgen05 kernel gets no status word here, so a bounded wait that
// expires inside it (a kernel that ended early and left its outputs invalid) is not
// reported through moe_ctx_status for this entry point.
//
// Shared state: every call on a device uses the same array and the array keeps the
// previous call's contents. Nothing in it needs to start at zero: each grouping kernel
// writes every element that a later kernel of the same call reads. Calls whose work
// overlaps on the GPU (two streams, or two host threads) race on the array; callers
// must order them (one stream, or events between streams).
//
// Set-up: the device address of the array is looked up once per device, with that
// device current, by the first call on that device (cudaGetSymbolAddress; the host
// symbol itself is only a stand-in and must never be handed to a kernel). Make that
// first call on each device before any stream capture.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/moe_b200.h"
#include "kernels.cuh"

namespace {

constexpr int kSeg = 1024;  // pairs per grouping segment (as moe_gather_qmm)
constexpr int kMaxDevices = 64;
constexpr size_t kScratchBytes = 64 * 1024;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

struct Layout {
  size_t hist, segbase, offsets, active, n_active, tile_start, perm, end;
};

Layout layout(int64_t batch, int E) {
  const int64_t nseg = std::max<int64_t>(1, (batch + kSeg - 1) / kSeg);
  Layout l{};
  size_t o = 0;
  l.hist = o;       o = align256(o + sizeof(int32_t) * nseg * E);
  l.segbase = o;    o = align256(o + sizeof(int32_t) * nseg * E);
  l.offsets = o;    o = align256(o + sizeof(int32_t) * (E + 1));
  l.active = o;     o = align256(o + sizeof(int32_t) * E);
  l.n_active = o;   o = align256(o + sizeof(int32_t));
  l.tile_start = o; o = align256(o + sizeof(int32_t) * (E + 1));
  l.perm = o;       o = align256(o + sizeof(uint32_t) * batch);
  l.end = o;
  return l;
}

}  // namespace

// Accessors of the context (its type is private to api.cu). The context supplies the
// device, the stream and the error message; its own scratch is never touched here.
namespace moe_internal {
int ctx_device(const moe_ctx* ctx);
void* ctx_stream(const moe_ctx* ctx);
void ctx_set_error(moe_ctx* ctx, const char* msg);
int check_gather(moe_ctx* ctx, const char* fn, const void* x, int64_t K, int64_t x_repeat,
                 const uint32_t* lhs_indices, const uint32_t* w, const void* scales, int64_t num_experts,
                 int64_t N, const uint32_t* rhs_indices, int64_t batch, int transpose, int group_size, int bits,
                 const void* out);
}  // namespace moe_internal
using moe_internal::check_gather;
using moe_internal::ctx_device;
using moe_internal::ctx_set_error;
using moe_internal::ctx_stream;

static int noalloc_fail(moe_ctx* ctx, int code, const char* msg) {
  ctx_set_error(ctx, msg);
  return code;
}

extern "C" int moe_gather_qmm_noalloc(moe_ctx* ctx, const void* x, int64_t x_rows, int64_t K,
                                      int64_t x_repeat, const uint32_t* lhs_indices, const uint32_t* w,
                                      const void* scales, const void* biases, int64_t num_experts,
                                      int64_t N, const uint32_t* rhs_indices, int64_t batch, int transpose,
                                      int group_size, int bits, int sorted_indices, void* out) {
  (void)x_rows;
  (void)sorted_indices;
  if (!ctx) return MOE_ERR_INVALID;
  char msg[256];
  ctx_set_error(ctx, "");
  // the same checks, codes and order as moe_gather_qmm; then the fixed-scratch limits
  int rc = check_gather(ctx, "moe_gather_qmm_noalloc", x, K, x_repeat, lhs_indices, w, scales, num_experts, N,
                        rhs_indices, batch, transpose, group_size, bits, out);
  if (rc || batch == 0) return rc;
  if (batch > MOE_NOALLOC_MAX_BATCH || num_experts > MOE_NOALLOC_MAX_EXPERTS) {
    snprintf(msg, sizeof(msg),
             "moe_gather_qmm_noalloc: batch=%lld / num_experts=%lld exceed the fixed scratch "
             "(at most %d rows and %d experts); use moe_gather_qmm",
             (long long)batch, (long long)num_experts, MOE_NOALLOC_MAX_BATCH, MOE_NOALLOC_MAX_EXPERTS);
    return noalloc_fail(ctx, MOE_ERR_INVALID, msg);
  }

  const int dev = ctx_device(ctx);
  if (dev < 0 || dev >= kMaxDevices) return noalloc_fail(ctx, MOE_ERR_INVALID, "moe_gather_qmm_noalloc: device");
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
  if (prev != dev && cudaSetDevice(dev) != cudaSuccess)
    return noalloc_fail(ctx, MOE_ERR_CUDA, "moe_gather_qmm_noalloc: cudaSetDevice failed");
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_ptr[dev]) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || !p) {
        snprintf(msg, sizeof(msg), "moe_gather_qmm_noalloc: cudaGetSymbolAddress failed: %s",
                 cudaGetErrorString(e));
        rc = noalloc_fail(ctx, MOE_ERR_CUDA, msg);
      } else {
        g_scratch_ptr[dev] = p;
      }
    }
    base = g_scratch_ptr[dev];
  }
  if (rc == MOE_OK) {
    const int E = (int)num_experts;
    const Layout l = layout(batch, E);
    if (l.end > kScratchBytes) {
      if (prev >= 0 && prev != dev) cudaSetDevice(prev);
      return noalloc_fail(ctx, MOE_ERR_INVALID, "moe_gather_qmm_noalloc: fixed scratch too small");
    }
    char* s = static_cast<char*>(base);
    moe::GatherCall gc{};
    gc.g.seg = kSeg;
    gc.g.nseg = (int)std::max<int64_t>(1, (batch + kSeg - 1) / kSeg);
    gc.g.hist = reinterpret_cast<int32_t*>(s + l.hist);
    gc.g.segbase = reinterpret_cast<int32_t*>(s + l.segbase);
    gc.g.offsets = reinterpret_cast<int32_t*>(s + l.offsets);
    gc.g.active = reinterpret_cast<int32_t*>(s + l.active);
    gc.g.n_active = reinterpret_cast<int32_t*>(s + l.n_active);
    gc.g.tile_start = reinterpret_cast<int32_t*>(s + l.tile_start);
    gc.g.perm = reinterpret_cast<uint32_t*>(s + l.perm);
    gc.status = nullptr;  // no status word: see the header comment
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
    const cudaError_t e = moe::launch_gather_qmm(gc, static_cast<cudaStream_t>(ctx_stream(ctx)));
    if (e != cudaSuccess) {
      snprintf(msg, sizeof(msg), "moe_gather_qmm_noalloc: launch failed: %s", cudaGetErrorString(e));
      rc = noalloc_fail(ctx, MOE_ERR_CUDA, msg);
    }
  }
  if (prev >= 0 && prev != dev) cudaSetDevice(prev);
  return rc;
}

static_assert(sizeof(int32_t) * 4 * MOE_NOALLOC_MAX_EXPERTS * 2 + sizeof(int32_t) * (3 * MOE_NOALLOC_MAX_EXPERTS + 3) +
                      sizeof(uint32_t) * MOE_NOALLOC_MAX_BATCH + 7 * 256 <=
                  kScratchBytes,
              "fixed scratch too small for the stated limits");

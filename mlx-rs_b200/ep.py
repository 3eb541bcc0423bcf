"""Expert parallelism (EP) of the MoE block over torch.distributed ranks, one GPU each.

The reference runs a block on one device (SparseMoeBlock::forward,
qwen3_moe_python_port.rs:420-488). Its experts shard naturally: rank r of `world`
holds the router (replicated) and experts [r*E/world, (r+1)*E/world) of every block,
and owns T_r tokens of the batch (the same T_r on every rank). One block is

    x_all     = all_gather(x_r)                     NCCL              [world*T_r, H]
    pk_all    = route(x_all)                        moe_ep_route      [world*T_r, k] u32
    partial   = experts(x_all, pk_all)              moe_ep_experts    [world*T_r, H] fp32 (or bf16)
    received  = all_to_all(partial)                 NCCL, equal parts [world, T_r, H]
    out_r     = finish(received) (+ next RMSNorm)   moe_ep_finish     [T_r, H] bf16

Dispatch is an all-gather rather than a variable all-to-all: with top-8 of 128 experts
a token reaches 5.3 of 8 ranks on average (1.6 of 2 at world 2), so the gather moves at
most 1.6x the rows a deduplicated all-to-all would, and it needs no per-step counts on
the host. Every rank routes every gathered token itself (the router is replicated and
its logits are bit-exact, so every rank computes the same routing): one router pass over
world*T_r tokens costs less than a second collective for the routing. Nothing in a block
waits for the host, so a whole stack of blocks, the
collectives included, can be captured in one CUDA graph. The combine all-to-all returns
per-rank partial sums, which the owner adds in fp32 in rank order: fp32 partials by
default (outputs differ from the single-device block only by the fp32 association of
the k-term sum), or, with partials="bf16", bf16 partials (half the bytes through the
all-to-all; each partial rounded once, so a token whose experts lie on several ranks
sees one more rounding, and partials of opposite sign that nearly cancel lose relative
accuracy: a 3-layer stack of small synthetic blocks measured mean-rel 0.02 against the
single-device oracle, twice the parity bound). Routing is bit-identical to the
single-device block.

The compute steps are supplied by an `ops` object so that the same orchestration runs
on the CUDA library (CudaEpOps, the default and the only product implementation) or,
in tests, on any other implementation of the three steps with the gloo backend.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import replace
from typing import Optional, Sequence

import torch
import torch.distributed as dist

from ._lib import MlxError, library
from .block import _Block
from .ops import _ctx, _ptr
from .synth import BlockWeights, MoeConfig, QWeight


def expert_range(num_experts: int, world: int, rank: int):
    """(expert_begin, num_local) of `rank`: equal contiguous shares of the experts."""
    if world <= 0 or not 0 <= rank < world:
        raise MlxError("expert_range", 1, f"rank {rank} of world {world}")
    if num_experts % world:
        raise MlxError("expert_range", 1, f"{num_experts} experts do not split evenly over {world} ranks")
    n = num_experts // world
    return rank * n, n


def local_weights(full: BlockWeights, expert_begin: int, num_local: int) -> BlockWeights:
    """The rank's share of a block: router and expert_bias whole, experts sliced."""
    def sl(q: QWeight) -> QWeight:
        e0, e1 = expert_begin, expert_begin + num_local
        return QWeight(q.w[e0:e1].contiguous(), q.scales[e0:e1].contiguous(),
                       None if q.biases is None else q.biases[e0:e1].contiguous())
    if full.config.shared_inter:
        raise MlxError("moe_ep_experts", 2, "the expert-parallel path has no shared expert")
    return BlockWeights(full.config, full.router, sl(full.gate), sl(full.up), sl(full.down), full.expert_bias)


class CudaEpOps:
    """The three EP compute steps on libmoe_b200.so (moe_ep_route / _experts / _finish)."""

    def bind(self, weights: BlockWeights, config: MoeConfig):
        return _Block(weights, config)

    def route(self, blk: _Block, x: torch.Tensor, packed: torch.Tensor):
        ctx = _ctx(x)
        T = x.shape[0]
        ctx.check("moe_ep_route", library().moe_ep_route(ctx.handle, C.byref(blk._cfg), C.byref(blk._wts),
                                                          _ptr(x), T, _ptr(packed)))

    def experts(self, blk: _Block, x_all, packed_all, expert_begin: int, num_local: int, partial):
        """partial: fp32 (moe_ep_experts) or bf16 (moe_ep_experts_bf16) [T_all, H]."""
        ctx = _ctx(x_all)
        name = "moe_ep_experts_bf16" if partial.dtype == torch.bfloat16 else "moe_ep_experts"
        ctx.check(name, getattr(library(), name)(
            ctx.handle, C.byref(blk._cfg), C.byref(blk._wts), _ptr(x_all), x_all.shape[0], _ptr(packed_all),
            expert_begin, num_local, _ptr(partial)))

    def finish(self, received, world: int, out, norm_weight=None, eps: float = 1e-6, normed=None):
        """received: [world, rows, H] fp32 or bf16 partials (moe_ep_finish / _bf16)."""
        ctx = _ctx(received)
        rows, H = out.shape
        name = "moe_ep_finish_bf16" if received.dtype == torch.bfloat16 else "moe_ep_finish"
        ctx.check(name, getattr(library(), name)(ctx.handle, _ptr(received), world, rows, H, _ptr(out),
                                                 _ptr(norm_weight), C.c_float(eps), _ptr(normed)))


class _Buffers:
    """Per-(tokens per rank) exchange buffers, reused by every block of a stack. With C
    chunks the gathered / partial / received tensors are C consecutive [world*T/C, ...]
    (or [world, T/C, H]) pieces of the same storage."""

    def __init__(self, T: int, H: int, k: int, world: int, device, partial_dtype=torch.float32):
        self.T = T
        self.x_all = torch.empty(world * T, H, dtype=torch.bfloat16, device=device)
        self.packed_all = torch.empty(world * T, k, dtype=torch.int32, device=device)
        self.partial = torch.empty(world * T, H, dtype=partial_dtype, device=device)
        self.received = torch.empty(world, T, H, dtype=partial_dtype, device=device)

    def chunk(self, C: int, c: int, world: int):
        Tc = self.T // C
        H = self.x_all.shape[1]
        k = self.packed_all.shape[1]
        return (self.x_all.view(C, world * Tc, H)[c], self.packed_all.view(C, world * Tc, k)[c],
                self.partial.view(C, world * Tc, H)[c], self.received.view(C, world, Tc, H)[c])


def default_chunks(T: int) -> int:
    """Token chunks per block when the caller does not choose: one. Splitting the batch
    lets the collectives of one chunk overlap the expert GEMMs of the next, but on 2 B200s
    with 4096 tokens per GPU four chunks measured slower (1.38 ms per block against 1.12):
    the smaller chunks give the tensor-core GEMM fewer rows per expert tile and the NCCL
    kernels take SMs from it."""
    del T
    return 1


class ExpertParallelBlock:
    """One rank's share of an expert-parallel MoE block (see the module docstring)."""

    def __init__(self, weights: BlockWeights, config: Optional[MoeConfig] = None, *, expert_begin: int,
                 num_local: int, group=None, ops=None, chunks: Optional[int] = None,
                 partials: str = "f32"):
        self.config = config or weights.config
        if self.config.shared_inter:
            raise MlxError("moe_ep_experts", 2, "the expert-parallel path has no shared expert")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.expert_begin, self.num_local = expert_begin, num_local
        self.ops = ops if ops is not None else CudaEpOps()
        self.bound = self.ops.bind(weights, self.config)
        self.chunks = chunks
        if partials not in ("bf16", "f32"):
            raise MlxError("moe_ep_experts", 1, f"partials must be 'bf16' or 'f32', not {partials!r}")
        self.partial_dtype = torch.bfloat16 if partials == "bf16" else torch.float32
        self._buf: dict = {}

    def buffers(self, T: int, device) -> _Buffers:
        b = self._buf.get((T, str(device)))
        if b is None:
            c = self.config
            b = _Buffers(T, c.hidden, c.top_k, self.world, device, self.partial_dtype)
            self._buf[(T, str(device))] = b
        return b

    def forward(self, x: torch.Tensor, out: Optional[torch.Tensor] = None, *, norm_weight=None,
                eps: float = 1e-6, normed: Optional[torch.Tensor] = None, buffers: Optional[_Buffers] = None):
        """out[T_r, H] = this rank's rows of the block applied to every rank's tokens.
        With norm_weight, normed = RMSNorm(out) * norm_weight is written as well."""
        c = self.config
        if x.dim() != 2 or x.shape[1] != c.hidden or x.dtype != torch.bfloat16 or not x.is_contiguous():
            raise MlxError("moe_ep_route", 1, f"x must be contiguous bf16 [T, {c.hidden}]")
        T = x.shape[0]
        b = buffers if buffers is not None else self.buffers(T, x.device)
        if out is None:
            out = torch.empty_like(x)
        g = self.group
        C = self.chunks if self.chunks is not None else default_chunks(T)
        if C < 1 or T % C:
            raise MlxError("moe_ep_route", 1, f"{T} tokens do not split into {C} chunks")
        if C == 1:
            dist.all_gather_into_tensor(b.x_all.view(torch.uint8), x.view(torch.uint8), group=g)
            self.ops.route(self.bound, b.x_all, b.packed_all)
            self.ops.experts(self.bound, b.x_all, b.packed_all, self.expert_begin, self.num_local, b.partial)
            dist.all_to_all_single(b.received.view(-1), b.partial.view(-1), group=g)
            self.ops.finish(b.received, self.world, out, norm_weight, eps, normed)
            return out
        # C chunks of T/C tokens: the gathers of chunk c+1 and the all-to-all of chunk c
        # run on the communication stream while the experts of the next chunk compute.
        Tc = T // C
        rows = [slice(c * Tc, (c + 1) * Tc) for c in range(C)]

        def gather(c):
            xa, _, _, _ = b.chunk(C, c, self.world)
            return (dist.all_gather_into_tensor(xa.view(torch.uint8), x[rows[c]].view(torch.uint8), group=g,
                                                async_op=True),)

        pending = gather(0)
        combines = []
        for c in range(C):
            for w in pending:
                w.wait()
            if c + 1 < C:
                pending = gather(c + 1)
            xa, pa, part, recv = b.chunk(C, c, self.world)
            self.ops.route(self.bound, xa, pa)
            self.ops.experts(self.bound, xa, pa, self.expert_begin, self.num_local, part)
            combines.append(dist.all_to_all_single(recv.view(-1), part.view(-1), group=g, async_op=True))
        for c in range(C):
            combines[c].wait()
            _, _, _, recv = b.chunk(C, c, self.world)
            self.ops.finish(recv, self.world, out[rows[c]], norm_weight, eps,
                            None if normed is None else normed[rows[c]])
        return out

    __call__ = forward


class ExpertParallelStack:
    """h = x; for each layer l: if l > 0: h = RmsNorm_l(h); h = block_l(h), every block
    expert-parallel; the RMSNorm runs fused into the previous block's finish step."""

    def __init__(self, blocks: Sequence[ExpertParallelBlock], norm_weights: Sequence[Optional[torch.Tensor]],
                 eps: float = 1e-6):
        self.blocks, self.norm_weights, self.eps = list(blocks), list(norm_weights), eps
        c0 = self.blocks[0].config
        if any((b.config.hidden, b.config.top_k) != (c0.hidden, c0.top_k) for b in self.blocks):
            raise MlxError("ExpertParallelStack", 1, "blocks must share hidden size and top_k")
        self._h: dict = {}

    def forward(self, x: torch.Tensor, out: Optional[torch.Tensor] = None):
        T, H = x.shape
        key = (T, str(x.device))
        if key not in self._h:
            self._h[key] = torch.empty_like(x)
        h = self._h[key]
        if out is None:
            out = torch.empty_like(x)
        buf = self.blocks[0].buffers(T, x.device)
        cur = x
        L = len(self.blocks)
        for l, blk in enumerate(self.blocks):
            last = l == L - 1
            nw = None if last else self.norm_weights[l + 1]
            normed = h if nw is not None else None
            # x and out may alias: the block reads x (route, all-gather) before it writes out
            blk.forward(cur, out, norm_weight=nw, eps=self.eps, normed=normed, buffers=buf)
            cur = h if normed is not None else out
        return out

    __call__ = forward


__all__ = ["expert_range", "local_weights", "default_chunks", "CudaEpOps", "ExpertParallelBlock",
           "ExpertParallelStack"]

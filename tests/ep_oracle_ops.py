"""The three expert-parallel compute steps (route / experts / finish) on the CPU oracle,
for running mlx_rs_b200.ep's orchestration over gloo ranks on CPU tensors. Test
infrastructure only: the product's ExpertParallelBlock uses CudaEpOps."""
from __future__ import annotations

from dataclasses import replace

import numpy as np
import torch

import oracle as O
import mlx_rs_b200.synth as S


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)


def from_bits(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def local_block(bw: S.BlockWeights, e0: int, n: int) -> S.BlockWeights:
    def sl(q):
        return S.QWeight(q.w[e0:e0 + n], q.scales[e0:e0 + n], q.biases[e0:e0 + n])
    return replace(bw, gate=sl(bw.gate), up=sl(bw.up), down=sl(bw.down))


class OracleEpOps:
    def bind(self, weights, config):
        return weights  # numpy BlockWeights holding the local experts

    def route(self, blk, x, packed):
        idx, w, _, _ = O.route(blk, bits(x), nthreads=1)
        packed.copy_(torch.from_numpy(O.pack_routing(idx, w).view(np.int32)))

    def experts(self, blk, x_all, packed_all, expert_begin, num_local, partial):
        p = O.ep_partials(blk, bits(x_all), packed_all.numpy().view(np.uint32), expert_begin, num_local,
                          nthreads=1)
        if partial.dtype == torch.bfloat16:  # the partial sums rounded once (to nearest even)
            partial.copy_(from_bits(S.f32_to_bf16_bits(p)))
        else:
            partial.copy_(torch.from_numpy(p))

    def finish(self, received, world, out, norm_weight=None, eps=1e-6, normed=None):
        nw = None if norm_weight is None else bits(norm_weight)
        o, n = O.ep_finish(received.float().numpy(), nw, eps)  # bf16 partials widen exactly
        out.copy_(from_bits(o))
        if normed is not None:
            normed.copy_(from_bits(n))

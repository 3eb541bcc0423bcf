"""GPU test of moe_gather_qmm_noalloc, the gather_qmm entry point that allocates nothing.

It exists for callers that cannot let this library allocate GPU memory (a host whose
own allocator already owns the device memory, or a latency-critical loop where an
allocation's device synchronisation is not allowed). Called straight through the C ABI,
twice in a row with different inputs, its output must match the regular moe_gather_qmm
within the parity tolerance; a call beyond its fixed scratch must be refused with an
error code. Collected last on purpose (file name) so that a run stopping at the first
failure has already run every other test; it also passes alone in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

import mlx_rs_b200.synth as S
from parity import assert_close

pytestmark = pytest.mark.gpu


def _case(rng, torch, T, k, E, N, K, with_lhs):
    q = S._stack(S._qweight(rng, E * N, K, 64, 4), E, N)
    x = S.f32_to_bf16_bits(rng.standard_normal((T, K), dtype=np.float32))
    dev = "cuda"
    tw = torch.from_numpy(q.w.view(np.int32)).to(dev)
    ts = torch.from_numpy(q.scales.view(np.int16)).to(dev).view(torch.bfloat16)
    tb = torch.from_numpy(q.biases.view(np.int16)).to(dev).view(torch.bfloat16)
    tx = torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16)
    if with_lhs:
        batch = T * k
        lhs = torch.from_numpy(rng.integers(0, T, size=batch).astype(np.int32)).to(dev)
        rhs = torch.from_numpy(rng.integers(0, E, size=batch).astype(np.int32)).to(dev)
        x_repeat = 1
    else:
        batch = T * k
        lhs = None
        rhs = torch.from_numpy(np.stack([rng.choice(E, size=k, replace=False) for _ in range(T)])
                               .astype(np.int32).reshape(-1)).to(dev)
        x_repeat = k
    return tx, tw, ts, tb, lhs, rhs, batch, x_repeat


def _call(fn_name, ctx, torch, tx, tw, ts, tb, lhs, rhs, batch, x_repeat, E, N, K):
    import mlx_rs_b200
    out = torch.empty(batch, N, dtype=torch.bfloat16, device="cuda")
    p = lambda t: None if t is None else C.c_void_p(t.data_ptr())  # noqa: E731
    rc = getattr(mlx_rs_b200.library(), fn_name)(
        ctx.handle, p(tx), tx.shape[0], K, x_repeat, p(lhs), p(tw), p(ts), p(tb), E, N, p(rhs),
        batch, 1, 64, 4, 0, p(out))
    return rc, out


def test_noalloc_gather_qmm_matches_regular_entry_point_twice():
    import torch
    from mlx_rs_b200._lib import context_for
    from gpu_util import dev_bits
    ctx = context_for(0)
    ctx.bind_stream(torch.cuda.current_stream().cuda_stream)
    rng = np.random.default_rng(2024)
    cases = [dict(T=40, k=8, E=64, N=384, K=1024, with_lhs=False),
             dict(T=9, k=3, E=16, N=128, K=512, with_lhs=True)]
    for c in cases:
        tx, tw, ts, tb, lhs, rhs, batch, xr = _case(rng, torch, c["T"], c["k"], c["E"], c["N"], c["K"],
                                                    c["with_lhs"])
        rc0, ref = _call("moe_gather_qmm", ctx, torch, tx, tw, ts, tb, lhs, rhs, batch, xr, c["E"], c["N"], c["K"])
        ctx.check("moe_gather_qmm", rc0)
        rc1, got = _call("moe_gather_qmm_noalloc", ctx, torch, tx, tw, ts, tb, lhs, rhs, batch, xr, c["E"],
                         c["N"], c["K"])
        ctx.check("moe_gather_qmm_noalloc", rc1)
        torch.cuda.synchronize()
        assert_close(dev_bits(got), dev_bits(ref), f"noalloc {c}")


def test_noalloc_rejects_sizes_beyond_its_fixed_scratch():
    import torch
    import mlx_rs_b200
    from mlx_rs_b200._lib import MOE_ERR_INVALID, context_for
    ctx = context_for(0)
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    p = C.c_void_p(dummy.data_ptr())
    rc = mlx_rs_b200.library().moe_gather_qmm_noalloc(ctx.handle, p, 1, 64, 1, None, p, p, None, 8, 64, p,
                                                      4097, 1, 64, 4, 0, p)
    assert rc == MOE_ERR_INVALID
    assert b"fixed scratch" in mlx_rs_b200.library().moe_last_error(ctx.handle)
    rc = mlx_rs_b200.library().moe_gather_qmm_noalloc(ctx.handle, p, 1, 64, 1, None, p, p, None, 513, 64, p,
                                                      16, 1, 64, 4, 0, p)
    assert rc == MOE_ERR_INVALID

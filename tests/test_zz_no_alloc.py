"""GPU test of moe_gather_qmm_noalloc, the gather_qmm entry point that allocates nothing.

It exists for callers that cannot let this library allocate GPU memory (a host whose
own allocator already owns the device memory, or a latency-critical loop where an
allocation's device synchronisation is not allowed). Called straight through the C ABI,
twice in a row with different inputs, its output must be bit-identical to the regular
moe_gather_qmm (both run the same kernel sequence with the same per-call choices) and
within the parity tolerance of the CPU oracle; a call beyond its fixed scratch must be
refused with an error code. Collected last on purpose (file name) so that a run
stopping at the first failure has already run every other test; it also passes alone
in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

import mlx_rs_b200.synth as S
from parity import ULP_TOL, ULP_TOL_TC, assert_close

pytestmark = pytest.mark.gpu


def _case(rng, torch, T, k, E, N, K, with_lhs):
    q = S._stack(S._qweight(rng, E * N, K, 64, 4), E, N)
    x = S.f32_to_bf16_bits(rng.standard_normal((T, K), dtype=np.float32))
    dev = "cuda"
    tw = torch.from_numpy(q.w.view(np.int32)).to(dev)
    ts = torch.from_numpy(q.scales.view(np.int16)).to(dev).view(torch.bfloat16)
    tb = torch.from_numpy(q.biases.view(np.int16)).to(dev).view(torch.bfloat16)
    tx = torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16)
    batch = T * k
    if with_lhs:
        lhs_h = rng.integers(0, T, size=batch).astype(np.uint32)
        rhs_h = rng.integers(0, E, size=batch).astype(np.uint32)
        x_repeat = 1
    else:
        lhs_h = None
        rhs_h = np.stack([rng.choice(E, size=k, replace=False) for _ in range(T)]).astype(np.uint32).reshape(-1)
        x_repeat = k
    lhs = None if lhs_h is None else torch.from_numpy(lhs_h.view(np.int32)).to(dev)
    rhs = torch.from_numpy(rhs_h.view(np.int32)).to(dev)
    host = (x, q, lhs_h, rhs_h)
    return (tx, tw, ts, tb, lhs, rhs, batch, x_repeat), host


def _call(fn_name, ctx, torch, dev_args, E, N, K):
    import mlx_rs_b200
    tx, tw, ts, tb, lhs, rhs, batch, x_repeat = dev_args
    out = torch.empty(batch, N, dtype=torch.bfloat16, device="cuda")
    p = lambda t: None if t is None else C.c_void_p(t.data_ptr())  # noqa: E731
    rc = getattr(mlx_rs_b200.library(), fn_name)(
        ctx.handle, p(tx), tx.shape[0], K, x_repeat, p(lhs), p(tw), p(ts), p(tb), E, N, p(rhs),
        batch, 1, 64, 4, 0, p(out))
    return rc, out


@pytest.mark.parametrize("case", [
    # few rows per expert: the GEMV only
    dict(T=40, k=8, E=64, N=384, K=1024, with_lhs=False, tc=False),
    dict(T=9, k=3, E=16, N=128, K=512, with_lhs=True, tc=False),
    # hundreds of rows per expert (4096 rows over 8 experts): the tcgen05 branch
    dict(T=512, k=8, E=8, N=256, K=512, with_lhs=False, tc=True),
])
def test_noalloc_gather_qmm_bit_identical_to_regular_entry_point_twice(case):
    import oracle as O
    import torch
    from gpu_util import dev_bits
    from mlx_rs_b200._lib import context_for
    ctx = context_for(0)
    ctx.bind_stream(torch.cuda.current_stream().cuda_stream)
    rng = np.random.default_rng(2024 + case["T"])
    E, N, K = case["E"], case["N"], case["K"]
    # two calls in a row with different inputs: the shared fixed scratch keeps the first
    # call's contents, which must not leak into the second
    for rep in range(2):
        dev_args, (xh, q, lhs_h, rhs_h) = _case(rng, torch, case["T"], case["k"], E, N, K, case["with_lhs"])
        rc0, ref = _call("moe_gather_qmm", ctx, torch, dev_args, E, N, K)
        ctx.check("moe_gather_qmm", rc0)
        rc1, got = _call("moe_gather_qmm_noalloc", ctx, torch, dev_args, E, N, K)
        ctx.check("moe_gather_qmm_noalloc", rc1)
        torch.cuda.synchronize()
        assert np.array_equal(dev_bits(got), dev_bits(ref)), f"noalloc differs from moe_gather_qmm ({case}, call {rep})"
        want = O.gather_qmm(xh, q.w, q.scales, q.biases, rhs_h, x_repeat=dev_args[7], lhs=lhs_h)
        assert_close(dev_bits(got), want, f"noalloc vs oracle {case}", ULP_TOL_TC if case["tc"] else ULP_TOL)


def test_noalloc_rejects_sizes_beyond_its_fixed_scratch():
    import torch
    import mlx_rs_b200
    from mlx_rs_b200._lib import MOE_ERR_INVALID, MOE_ERR_UNSUPPORTED, context_for
    ctx = context_for(0)
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    p = C.c_void_p(dummy.data_ptr())
    L = mlx_rs_b200.library()
    rc = L.moe_gather_qmm_noalloc(ctx.handle, p, 1, 64, 1, None, p, p, None, 8, 64, p, 4097, 1, 64, 4, 0, p)
    assert rc == MOE_ERR_INVALID
    assert b"fixed scratch" in L.moe_last_error(ctx.handle)
    rc = L.moe_gather_qmm_noalloc(ctx.handle, p, 1, 64, 1, None, p, p, None, 513, 64, p, 16, 1, 64, 4, 0, p)
    assert rc == MOE_ERR_INVALID
    # argument errors come first, with the codes moe_gather_qmm gives: a valid MLX width
    # that is not implemented is UNSUPPORTED even when the size is also beyond the limit
    for fn in ("moe_gather_qmm", "moe_gather_qmm_noalloc"):
        rc = getattr(L, fn)(ctx.handle, p, 1, 64, 1, None, p, p, None, 8, 64, p, 5000, 1, 64, 3, 0, p)
        assert rc == MOE_ERR_UNSUPPORTED, fn

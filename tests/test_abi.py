"""CPU checks of the C-ABI library: it builds, loads, and exports every symbol that
include/moe_b200.h declares; argument validation answers with error codes (no GPU work)."""
import ctypes as C
import os
import re

import mlx_rs_b200
from mlx_rs_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "moe_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(moe_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for n in ("moe_gather_qmm", "moe_quantized_matmul", "moe_block_forward", "moe_block_route",
              "moe_fast_rms_norm", "moe_ctx_create", "moe_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = mlx_rs_b200.library()
    assert os.path.dirname(os.path.abspath(mlx_rs_b200.library_path)).endswith("mlx-rs_b200")
    for n in declared_functions():
        assert hasattr(lib, n), f"missing export {n}"
        assert n in _lib.SIGNATURES, f"no ctypes signature for {n}"


def test_abi_version():
    assert mlx_rs_b200.library().moe_abi_version() == 1


def test_null_context_is_rejected_without_crashing():
    lib = mlx_rs_b200.library()
    assert lib.moe_quantized_matmul(None, None, 1, 64, None, None, None, 1, 1, 64, 4, None) == _lib.MOE_ERR_INVALID
    assert lib.moe_block_forward(None, None, None, None, 1, None) == _lib.MOE_ERR_INVALID
    assert lib.moe_layer_ffn_forward(None, None, None, None, 1, None, 1e-6, None, None) == _lib.MOE_ERR_INVALID
    assert lib.moe_ctx_create(0, None, None) == _lib.MOE_ERR_INVALID
    assert lib.moe_last_error(None) == b"null context"


def test_ctx_create_reports_missing_device():
    import torch
    if torch.cuda.is_available():
        return
    h = C.c_void_p()
    assert mlx_rs_b200.library().moe_ctx_create(0, None, C.byref(h)) == _lib.MOE_ERR_CUDA
    assert not h.value

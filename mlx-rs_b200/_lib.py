"""ctypes binding of libmoe_b200.so (the C ABI in include/moe_b200.h).

The library is loaded from this package directory. If it is missing it is built
with nvcc (``build.py``); if that is impossible the import of any compute entry point
raises — there is no fallback implementation.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
library_path = os.path.join(_HERE, "libmoe_b200.so")

MOE_OK = 0
MOE_ERR_INVALID = 1
MOE_ERR_UNSUPPORTED = 2
MOE_ERR_CUDA = 3
MOE_ERR_NO_MEMORY = 4
MOE_ERR_TIMEOUT = 5

SCORING_SOFTMAX = 0
SCORING_SOFTMAX_BIAS = 1
SCORING_SIGMOID_BIAS_SELECT = 2


class MlxError(RuntimeError):
    """Error::Mlx("<fn> failed (rc=N)") of crates/mlx-core/src/error.rs, plus the
    library's one-line reason."""

    def __init__(self, fn: str, rc: int, detail: str = ""):
        self.fn, self.rc, self.detail = fn, rc, detail
        msg = f"{fn} failed (rc={rc})"
        if detail:
            msg += f": {detail}"
        super().__init__(msg)


class QWeight(C.Structure):
    _fields_ = [("w", C.c_void_p), ("scales", C.c_void_p), ("biases", C.c_void_p)]


class BlockConfig(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "hidden", "num_experts", "top_k", "moe_inter", "shared_inter", "scoring",
        "norm_topk_prob", "has_shared_gate", "group_size", "bits")]


class BlockWeights(C.Structure):
    _fields_ = [("router", QWeight), ("expert_bias", C.c_void_p), ("gate", QWeight),
                ("up", QWeight), ("down", QWeight), ("shared_gate", QWeight),
                ("shared_up", QWeight), ("shared_down", QWeight),
                ("shared_expert_gate", QWeight)]


_lib = None
_lock = threading.Lock()

# Every symbol include/moe_b200.h declares, with its ctypes signature.
SIGNATURES = {
    "moe_abi_version": (C.c_int, []),
    "moe_ctx_create": (C.c_int, [C.c_int, C.c_void_p, C.POINTER(C.c_void_p)]),
    "moe_ctx_destroy": (None, [C.c_void_p]),
    "moe_ctx_set_stream": (C.c_int, [C.c_void_p, C.c_void_p]),
    "moe_ctx_reserve": (C.c_int, [C.c_void_p, C.POINTER(BlockConfig), C.c_int64]),
    "moe_last_error": (C.c_char_p, [C.c_void_p]),
    "moe_quantized_matmul": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p,
                                       C.c_void_p, C.c_void_p, C.c_int64, C.c_int, C.c_int,
                                       C.c_int, C.c_void_p]),
    "moe_gather_qmm": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int64,
                                 C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64,
                                 C.c_int64, C.c_void_p, C.c_int64, C.c_int, C.c_int, C.c_int,
                                 C.c_int, C.c_void_p]),
    "moe_gather_qmm_noalloc": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int64,
                                         C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64,
                                         C.c_int64, C.c_void_p, C.c_int64, C.c_int, C.c_int, C.c_int,
                                         C.c_int, C.c_void_p]),
    "moe_fast_rms_norm": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_float, C.c_int64,
                                    C.c_int64, C.c_void_p]),
    "moe_block_forward": (C.c_int, [C.c_void_p, C.POINTER(BlockConfig), C.POINTER(BlockWeights),
                                    C.c_void_p, C.c_int64, C.c_void_p]),
    "moe_layer_ffn_forward": (C.c_int, [C.c_void_p, C.POINTER(BlockConfig), C.POINTER(BlockWeights),
                                        C.c_void_p, C.c_int64, C.c_void_p, C.c_float, C.c_void_p,
                                        C.c_void_p]),
    "moe_gemma4_block_forward": (C.c_int, [C.c_void_p, C.POINTER(BlockConfig), C.POINTER(BlockWeights),
                                           C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p,
                                           C.c_void_p, C.c_void_p]),
    "moe_block_profile": (C.c_int, [C.c_void_p, C.POINTER(BlockConfig), C.POINTER(BlockWeights),
                                    C.c_void_p, C.c_int64, C.c_void_p, C.POINTER(C.c_float),
                                    C.POINTER(C.c_int32)]),
    "moe_block_router_logits": (C.c_int, [C.c_void_p, C.POINTER(BlockConfig), C.POINTER(BlockWeights),
                                          C.c_void_p, C.c_int64, C.c_void_p]),
    "moe_block_route": (C.c_int, [C.c_void_p, C.POINTER(BlockConfig), C.POINTER(BlockWeights),
                                  C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p,
                                  C.c_void_p]),
    "moe_ctx_status": (C.c_int, [C.c_void_p, C.POINTER(C.c_int32)]),
    "moe_ep_route": (C.c_int, [C.c_void_p, C.POINTER(BlockConfig), C.POINTER(BlockWeights),
                               C.c_void_p, C.c_int64, C.c_void_p]),
    "moe_ep_experts": (C.c_int, [C.c_void_p, C.POINTER(BlockConfig), C.POINTER(BlockWeights),
                                 C.c_void_p, C.c_int64, C.c_void_p, C.c_int32, C.c_int32,
                                 C.c_void_p]),
    "moe_ep_finish": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int64, C.c_int64,
                                C.c_void_p, C.c_void_p, C.c_float, C.c_void_p]),
    "moe_ep_experts_bf16": (C.c_int, [C.c_void_p, C.POINTER(BlockConfig), C.POINTER(BlockWeights),
                                      C.c_void_p, C.c_int64, C.c_void_p, C.c_int32, C.c_int32,
                                      C.c_void_p]),
    "moe_ep_finish_bf16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int64, C.c_int64,
                                     C.c_void_p, C.c_void_p, C.c_float, C.c_void_p]),
}


def library():
    """Load (building first if needed) and return the ctypes handle."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(library_path):
                from . import build as _build
                _build.build()
            L = C.CDLL(library_path)
            for name, (res, args) in SIGNATURES.items():
                f = getattr(L, name)
                f.restype = res
                f.argtypes = args
            _lib = L
    return _lib


class Context:
    """A moe_ctx on one CUDA device; follows torch's current stream per call."""

    def __init__(self, device: int):
        self.device = device
        h = C.c_void_p()
        rc = library().moe_ctx_create(device, None, C.byref(h))
        if rc != MOE_OK:
            raise MlxError("moe_ctx_create", rc, f"device {device}")
        self.handle = h

    def bind_stream(self, stream_handle: int):
        library().moe_ctx_set_stream(self.handle, C.c_void_p(stream_handle))

    def check(self, fn: str, rc: int):
        if rc != MOE_OK:
            msg = library().moe_last_error(self.handle)
            raise MlxError(fn, rc, msg.decode() if msg else "")

    def close(self):
        if self.handle:
            library().moe_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_contexts: dict[int, Context] = {}


def context_for(device_index: int) -> Context:
    ctx = _contexts.get(device_index)
    if ctx is None:
        ctx = Context(device_index)
        _contexts[device_index] = ctx
    return ctx

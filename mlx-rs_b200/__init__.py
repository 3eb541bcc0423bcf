"""B200 (sm_100a) implementation of the mlx-rs device-side MoE / SwitchGLU block.

Host-side mirror of the reference's Rust interface for this path:
  ops.quantized_matmul / ops.gather_qmm / ops.fast_rms_norm
      <- Array::quantized_matmul / Array::gather_qmm / Array::fast_rms_norm
         (crates/mlx-core/src/ops.rs:592-637, 830-891, 691-701)
  block.SparseMoeBlock, block.MoeFeedForward, block.RmsNorm, block.MoeStack
      <- SparseMoeBlock::forward (qwen3_moe_python_port.rs:420-488),
         MoeFeedForward::forward (lfm2_moe_python_port.rs:541-740),
         RmsNorm::forward (crates/mlx-nn/src/rms_norm.rs:30-34)
  graph.GraphedForward
      <- the per-step MoE work of the decode loop (generate.rs:811-880), one graph replay
  checkpoint.load_blocks / load_device_blocks
      <- VarBuilder::from_safetensors + SparseMoeBlock::load / MoeFeedForward::load
         (crates/mlx-nn/src/var_builder.rs:31-46, qwen3_moe_python_port.rs:394-418,
         lfm2_moe_python_port.rs:524-540)
Every call goes through the C ABI of libmoe_b200.so (include/moe_b200.h); there is no
other compute path. torch supplies device memory and streams only.
"""
from ._lib import MlxError, library, library_path  # noqa: F401
from . import ops  # noqa: F401
from . import block  # noqa: F401
from . import synth  # noqa: F401
from . import checkpoint  # noqa: F401
from . import graph  # noqa: F401

__all__ = ["MlxError", "library", "library_path", "ops", "block", "synth", "checkpoint", "graph"]

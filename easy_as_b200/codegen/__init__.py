"""IR -> CUDA C++ lowering for sm_100a (generic emitter plus native pattern plans)."""

from .cuda import Lowered, infer_block_and_mode, ir_to_cuda

__all__ = ["Lowered", "infer_block_and_mode", "ir_to_cuda"]

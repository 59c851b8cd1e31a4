"""Which buffer arguments a kernel writes (easy_as ``eas/analysis.py:8-27``).

The result marks written buffers: the emitter declares the others ``const``,
and the runtime copies written host (numpy) buffers back after a launch.
"""

from __future__ import annotations

from .ir import IRModule


def infer_writes(ir: IRModule) -> frozenset[str]:
    arg_name = {i.out.id: str(i.args[0]) for i in ir.insts if i.op == "arg" and i.out is not None}
    return frozenset(arg_name[i.args[0].id] for i in ir.insts
                     if i.op in ("store", "mma_store") and i.args[0].id in arg_name)

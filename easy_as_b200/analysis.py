"""Which buffer arguments a kernel writes (easy_as ``eas/analysis.py:8-27``).

The result marks written buffers: the emitter declares the others ``const``,
and the runtime copies written host (numpy) buffers back after a launch.
"""

from __future__ import annotations

from .ir import IRModule


def infer_reads(ir: IRModule) -> frozenset[str]:
    """Buffer arguments the kernel may read: every use of a buffer other than as the target of a
    store counts (loads, dot and mma operands, ...), so the set can only be too large."""
    arg_name = {i.out.id: str(i.args[0]) for i in ir.insts if i.op == "arg" and i.out is not None}
    out = set()
    for i in ir.insts:
        for k, x in enumerate(i.args):
            if hasattr(x, "id") and x.id in arg_name and not (i.op in ("store", "mma_store") and k == 0):
                out.add(arg_name[x.id])
    return frozenset(out)


def infer_writes(ir: IRModule) -> frozenset[str]:
    arg_name = {i.out.id: str(i.args[0]) for i in ir.insts if i.op == "arg" and i.out is not None}
    return frozenset(arg_name[i.args[0].id] for i in ir.insts
                     if i.op in ("store", "mma_store") and i.args[0].id in arg_name)

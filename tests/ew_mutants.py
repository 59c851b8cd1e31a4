"""Variants of an elementwise kernel for soundness tests of the elementwise analysis behind the
pipelined host-buffer path (``elementwise_info`` in easy_as_b200/codegen/cuda.py): that path copies
in only the buffers a kernel loads and copies back only the elements below each store's mask
bound, so a wrong analysis would corrupt host arrays.  ``EW_MUTANTS`` lists (MUT, what changes,
is the kernel still elementwise)."""

from __future__ import annotations

import eas
from eas import mk

EW_MUTANTS = [
    (0, "c = a + b, masked offs < N", True),
    (1, "store one element to the right", False),
    (2, "load a at a permuted offset", False),
    (3, "store masked by offs < M (a smaller scalar bound)", True),
    (4, "c read and written: c = c + a", True),
    (5, "store masked by a data-dependent condition", False),
    (6, "store masked by a constant bound (offs < 1000)", True),
    (7, "two outputs with different bounds (c below N, d below M)", True),
]


@eas.kernel
def ew_mut(a, b, c, d, N, M, MUT: eas.constexpr, BLOCK: eas.constexpr):
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    m = offs < N
    x = mk.load(a, offs, m)
    y = mk.load(b, offs, m)
    if MUT == 2:
        x = mk.load(a, (offs * 7) % N, m)
    v = x + y
    if MUT == 4:
        v = mk.load(c, offs, m) + x
    if MUT == 1:
        mk.store(c, offs + 1, v, offs + 1 < N)
    elif MUT == 3:
        mk.store(c, offs, v, offs < M)
    elif MUT == 5:
        mk.store(c, offs, v, m & (mk.to_u32(x + 1000.0) < 1000))
    elif MUT == 6:
        mk.store(c, offs, v, offs < 1000)
    elif MUT == 7:
        mk.store(c, offs, v, m)
        mk.store(d, offs, x * y, offs < M)
    else:
        mk.store(c, offs, v, m)
    if MUT != 7:
        mk.store(d, offs, x, offs < 1)   # d touched at element 0 only

"""Near-miss variants of a simdgroup-MMA matmul written with this repository's DSL, for soundness tests
of the simdgroup-MMA GEMM proof (easy_as_b200/codegen/mma_gemm.py).

``mma_mm`` stages f16 tiles of A (BM x BK) and B (BK x BN) in threadgroup memory, lets each
simdgroup accumulate one 8x8 C subtile with ``mk.mma`` over the K tile, stores the fragments to a
threadgroup C tile and copies it out with bounds checks.  ``MUT`` selects one change;
``MMA_MUTANTS`` lists (MUT, what changes, must the proof decline)."""

from __future__ import annotations

import eas
from eas import mk

MMA_MUTANTS = [
    (0, "unchanged", False),
    (1, "B tile staged transposed but read as row-major", True),
    (2, "second mma step reads A one column to the left (columns 7..14)", True),
    (3, "B columns unmasked (reads past N; those outputs are never stored)", False),
    (4, "K loop skips the last tile", False),
    (5, "1.0 added to every output", True),
    (6, "C tile read back one column to the right", True),
    (7, "A rows unmasked past M (rows past M are never stored)", False),
]

BM, BN, BK = 16, 16, 16
NT = (BM // 8) * (BN // 8) * 32


@eas.kernel
def mma_mm(a, b, c, M, N, K: eas.constexpr, MUT: eas.constexpr):
    t = mk.tid(0, NT)
    sg = mk.sg_id()
    row0 = mk.program_id(1) * BM
    col0 = mk.program_id(0) * BN
    sg_r = sg // (BN // 8)
    sg_c = sg % (BN // 8)
    lda, ldb, ldc = BK + 1, BN + 1, BN + 1
    sa = mk.alloc_tg_f16(BM * lda)
    sb = mk.alloc_tg_f16(BK * ldb)
    sc = mk.alloc_tg(BM * ldc)
    acc = mk.mma_zero()
    k_end = K - BK if MUT == 4 else K
    for k0 in range(0, k_end, BK):
        for i in range(0, BM * BK, NT):
            e = t + i
            ar, ak = e // BK, e % BK
            row_ok = True if MUT == 7 else row0 + ar < M
            ok = mk.where(e < BM * BK, mk.where(row_ok, k0 + ak < K, False), False)
            mk.store(sa, ar * lda + ak, mk.to_f16(mk.load(a, (row0 + ar) * K + k0 + ak, ok)), e < BM * BK)
        for i in range(0, BK * BN, NT):
            e = t + i
            bk, bc = e // BN, e % BN
            col_ok = True if MUT == 3 else col0 + bc < N
            ok = mk.where(e < BK * BN, mk.where(k0 + bk < K, col_ok, False), False)
            slot = bc * ldb + bk if MUT == 1 else bk * ldb + bc
            mk.store(sb, slot, mk.to_f16(mk.load(b, (k0 + bk) * N + col0 + bc, ok)), e < BK * BN)
        mk.barrier()
        for kk in range(0, BK, 8):
            a_col = 7 if (MUT == 2 and kk == 8) else kk
            acc = mk.mma(sa, (sg_r * 8) * lda + a_col, lda, sb, kk * ldb + sg_c * 8, ldb, acc)
        mk.barrier()
    mk.mma_store(sc, (sg_r * 8) * ldc + sg_c * 8, ldc, acc)
    mk.barrier()
    for i in range(0, BM * BN, NT):
        e = t + i
        r, cc = e // BN, e % BN
        row, col = row0 + r, col0 + cc
        src = r * ldc + (cc + 1) % BN if MUT == 6 else r * ldc + cc
        v = mk.load(sc, src, True)
        if MUT == 5:
            v = v + 1.0
        mk.store(c, row * N + col, v, mk.where(row < M, col < N, False))


def grid(M: int, N: int) -> tuple[int, int, int]:
    return (-(-N // BN), -(-M // BM), 1)


def sizes(M: int, N: int, K: int) -> dict[str, int]:
    """Buffer elements: A and B are padded by a tile so unmasked mutants stay inside."""
    return {"a": (M + BM) * K, "b": K * N + BN, "c": M * N}

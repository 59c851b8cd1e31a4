"""A family of tiled fp32 matmul kernels written with this repository's DSL (not the reference's
code): tile shape TM x TN, K tiles of TK, NT threads, threadgroup padding PAD, each thread owning
TM*TN/NT consecutive outputs of one row.  Used to check that the tiled-GEMM proof handles kernels
beyond the reference's own IR."""

from __future__ import annotations

import eas
from eas import mk


@eas.kernel
def tile_mm(a, b, c, M, N, K: eas.constexpr, TM: eas.constexpr, TN: eas.constexpr, TK: eas.constexpr,
            NT: eas.constexpr, PAD: eas.constexpr):
    t = mk.tid(0, NT)
    row0 = mk.program_id(1) * TM
    col0 = mk.program_id(0) * TN
    lda_s = TK + PAD
    ldb_s = TN + PAD
    sa = mk.alloc_tg(TM * lda_s)
    sb = mk.alloc_tg(TK * ldb_s)
    per = TM * TN // NT            # outputs per thread, along a row
    r = t // (TN // per)
    cq = (t % (TN // per)) * per
    acc = [0.0] * per
    for k0 in range(0, K, TK):
        for i in range(0, TM * TK, NT):
            e = t + i
            inb = e < TM * TK              # threads past the tile copy nothing
            ar, ak = e // TK, e % TK
            ok = (row0 + ar < M) & (k0 + ak < K) & inb
            mk.store(sa, ar * lda_s + ak, mk.load(a, (row0 + ar) * K + k0 + ak, ok), inb)
        for i in range(0, TK * TN, NT):
            e = t + i
            inb = e < TK * TN
            bk, bc = e // TN, e % TN
            ok = (k0 + bk < K) & (col0 + bc < N) & inb
            mk.store(sb, bk * ldb_s + bc, mk.load(b, (k0 + bk) * N + col0 + bc, ok), inb)
        mk.barrier()
        for j in range(per):
            acc[j] = acc[j] + mk.dot(sa, r * lda_s, 1, sb, cq + j, ldb_s, TK)
        mk.barrier()
    for j in range(per):
        mk.store(c, (row0 + r) * N + col0 + cq + j, acc[j], (row0 + r < M) & (col0 + cq + j < N))


# (TM, TN, TK, NT, PAD)
VARIANTS = [(16, 64, 16, 256, 1), (32, 32, 32, 256, 1), (64, 64, 16, 256, 0), (8, 128, 8, 128, 4),
            (32, 64, 24, 128, 2)]


def grid(M, N, TM, TN):
    return (-(-N // TN), -(-M // TM), 1)


@eas.kernel
def tile_mm_batched(a, b, c, M, N, K: eas.constexpr, TM: eas.constexpr, TN: eas.constexpr,
                    TK: eas.constexpr, NT: eas.constexpr):
    """Batch on program_id(2): A[z] at z*M*K, B[z] at z*K*N, C[z] at z*M*N."""
    t = mk.tid(0, NT)
    z = mk.program_id(2)
    row0 = mk.program_id(1) * TM
    col0 = mk.program_id(0) * TN
    sa = mk.alloc_tg(TM * TK)
    sb = mk.alloc_tg(TK * TN)
    per = TM * TN // NT
    r = t // (TN // per)
    cq = (t % (TN // per)) * per
    acc = [0.0] * per
    for k0 in range(0, K, TK):
        for i in range(0, TM * TK, NT):
            e = t + i
            ar, ak = e // TK, e % TK
            ok = (row0 + ar < M) & (k0 + ak < K)
            mk.store(sa, ar * TK + ak, mk.load(a, z * M * K + (row0 + ar) * K + k0 + ak, ok))
        for i in range(0, TK * TN, NT):
            e = t + i
            bk, bc = e // TN, e % TN
            ok = (k0 + bk < K) & (col0 + bc < N)
            mk.store(sb, bk * TN + bc, mk.load(b, z * K * N + (k0 + bk) * N + col0 + bc, ok))
        mk.barrier()
        for j in range(per):
            acc[j] = acc[j] + mk.dot(sa, r * TK, 1, sb, cq + j, TN, TK)
        mk.barrier()
    for j in range(per):
        mk.store(c, z * M * N + (row0 + r) * N + col0 + cq + j, acc[j], (row0 + r < M) & (col0 + cq + j < N))

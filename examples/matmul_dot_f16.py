"""fp16 GEMM written with one ``mk.dot`` per output element (configs C4 and C5).

``C[b][m][n] = sum_k A[b][m][k] * B[b][k][n]`` with f16 inputs, f32
accumulation and an f32 output; A is ``[batch, M, K]`` and B ``[batch, K, N]``,
both row-major and contiguous, K is a runtime scalar.  Each DSL thread owns one
output element; ``program_id(0)`` tiles N, ``program_id(1)`` is the row and
``program_id(2)`` the batch.  The CUDA backend recognises this shape and runs
it on the tcgen05 tensor-core GEMM (``eas_gemm_f16_tile``).  ``BLOCK_N`` is
the N tile of a CTA; ``BLOCK_M`` 128 runs the 1-SM kernel (128 x BLOCK_N
tiles) and 256 a CTA pair (256 x 2 BLOCK_N tiles); ``BLOCK_K`` 64 or 128 is
the K depth of one pipeline stage.  The default ``BLOCK_M = BLOCK_K = 0``
leaves the M tile and stage depth to the library.  ``CONFIGS`` is the
autotune space of benchmark configuration C4: eight distinct kernels.

Run as a script for a quick check against torch (needs a GPU).
"""

import argparse

import eas
from eas import mk

CONFIGS = [eas.Config(meta={"BLOCK_M": bm, "BLOCK_N": bn, "BLOCK_K": bk})
           for bm in (128, 256) for bn in (128, 256) for bk in (64, 128)]


def _cdiv(a, b):
    return -(-a // b)


@eas.kernel
def matmul_dot_f16(a, b, c, M, N, K, BLOCK_M: eas.constexpr = 0, BLOCK_N: eas.constexpr = 256,
                   BLOCK_K: eas.constexpr = 0):
    col = mk.program_id(0) * BLOCK_N + mk.tid(0, BLOCK_N)
    row = mk.program_id(1)
    bat = mk.program_id(2)
    inside = (row < M) & (col < N)
    # threads outside C take a zero-length dot, so they read nothing past a or b
    acc = mk.dot(a, bat * (M * K) + row * K, 1, b, bat * (K * N) + col, N, mk.where(inside, K, 0))
    mk.store(c, bat * (M * N) + row * N + col, acc, inside)


matmul_dot_f16_tuned = eas.autotune(configs=CONFIGS, key=["M", "N", "K"], warmup=2, repeat=5)(
    eas.kernel(matmul_dot_f16.fn))


def grid(batch):
    return lambda meta, args: (_cdiv(int(args["N"]), int(meta["BLOCK_N"])), int(args["M"]), int(batch))


def matmul(a, b, c, batch, M, N, K, *, block_n=256, tuned=False, sync=True):
    """Launch on flat buffers a [batch*M*K], b [batch*K*N], c [batch*M*N]."""
    if tuned:
        matmul_dot_f16_tuned(a, b, c, M, N, K, _grid=grid(batch), _sync=sync)
    else:
        matmul_dot_f16(a, b, c, M, N, K, BLOCK_N=block_n, _grid=grid(batch), _sync=sync)


def main():
    import torch

    ap = argparse.ArgumentParser()
    ap.add_argument("--m", type=int, default=1024)
    ap.add_argument("--n", type=int, default=1024)
    ap.add_argument("--k", type=int, default=1024)
    ap.add_argument("--batch", type=int, default=1)
    args = ap.parse_args()
    g = torch.Generator(device="cuda").manual_seed(0)
    a = (torch.randn(args.batch, args.m, args.k, device="cuda", generator=g) / args.k ** 0.5).half()
    b = (torch.randn(args.batch, args.k, args.n, device="cuda", generator=g) / args.k ** 0.5).half()
    c = torch.empty(args.batch, args.m, args.n, device="cuda")
    matmul(a.reshape(-1), b.reshape(-1), c.reshape(-1), args.batch, args.m, args.n, args.k)
    ref = torch.bmm(a.double(), b.double())
    err = (c.double() - ref).abs().max().item() / ref.abs().max().item()
    print(f"max |C - ref| / max |ref| = {err:.3e}")


if __name__ == "__main__":
    main()

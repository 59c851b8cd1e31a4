"""GPU: a grid split into program-id ranges (as each rank of a multi-GPU run launches
it) reproduces the single launch bit for bit, with full-size buffers and with
slice-only buffers (pointer rebasing)."""

import pytest

import eas
from eas import mk
from easy_as_b200.shard import element_range, run_shard

pytestmark = pytest.mark.gpu


@eas.kernel
def add_kernel(a, b, c, N, BLOCK: eas.constexpr):
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    m = offs < N
    mk.store(c, offs, mk.load(a, offs, m) + mk.load(b, offs, m), m)


@eas.kernel
def rows_kernel(out, H, W, BLOCK: eas.constexpr):
    col = mk.program_id(0) * BLOCK + mk.tid(0, BLOCK)
    row = mk.program_id(1)
    mk.store(out, row * W + col, mk.to_f32(row * W + col), (row < H) & (col < W))


@pytest.mark.parametrize("world", [2, 3, 8])
def test_ranges_cover_the_launch(cuda_rt, world):
    import torch

    n = 1 << 20 | 37
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(n, device="cuda", generator=g)
    b = torch.randn(n, device="cuda", generator=g)
    c = torch.zeros(n, device="cuda")
    for r in range(world):
        run_shard(add_kernel, a, b, c, n, BLOCK=1024, _rank=r, _world=world)
    assert torch.equal(c, a + b)


def test_slice_only_buffers(cuda_rt):
    import torch

    n, world = 100_003, 4
    g = torch.Generator(device="cuda").manual_seed(1)
    a = torch.randn(n, device="cuda", generator=g)
    b = torch.randn(n, device="cuda", generator=g)
    pieces = []
    for r in range(world):
        lo, hi = element_range(n, 256, r, world)
        al, bl, cl = a[lo:hi].clone(), b[lo:hi].clone(), torch.zeros(hi - lo, device="cuda")
        run_shard(add_kernel, al, bl, cl, n, BLOCK=256, _rank=r, _world=world,
                  _buffer_base={"a": lo, "b": lo, "c": lo})
        pieces.append(cl)
    assert torch.equal(torch.cat(pieces), a + b)


def test_axis1_split_thread_mode(cuda_rt):
    import torch

    H, W = 37, 300
    out = torch.full((H * W,), -1.0, device="cuda")
    for r in range(3):
        run_shard(rows_kernel, out, H, W, BLOCK=128, _rank=r, _world=3, _axis=1)
    assert torch.equal(out, torch.arange(H * W, device="cuda", dtype=torch.float32))


def test_repeated_slice_calls_reuse_the_prepared_launch(cuda_rt):
    """Later identical run_shard calls take the prepared range launch (buffer pointers patched in,
    moved back by the buffer base) and stay bit-exact as the data changes."""
    import torch

    n, world = 1 << 20 | 5, 4
    shard_keys = lambda: {k for k in add_kernel._fast if k[0] == "shard"}  # noqa: E731
    before = shard_keys()
    for step in range(3):
        g = torch.Generator(device="cuda").manual_seed(10 + step)
        a = torch.randn(n, device="cuda", generator=g)
        b = torch.randn(n, device="cuda", generator=g)
        pieces = []
        for r in range(world):
            lo, hi = element_range(n, 1024, r, world)
            al, bl, cl = a[lo:hi].clone(), b[lo:hi].clone(), torch.zeros(hi - lo, device="cuda")
            run_shard(add_kernel, al, bl, cl, n, BLOCK=1024, _rank=r, _world=world,
                      _buffer_base={"a": lo, "b": lo, "c": lo}, _sync=False)
            pieces.append(cl)
        torch.cuda.synchronize()
        assert torch.equal(torch.cat(pieces), a + b)
    assert len(shard_keys() - before) == world      # one prepared launch per rank, reused by steps 2 and 3

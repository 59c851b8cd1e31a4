"""CPU: the fp16 GEMM launcher's choices (``eas_gemm_f16_plan``: CTA pair or 1-SM kernel, tile,
stages, split-K), computed without a device from the same rules the launcher applies, for the
benchmark shapes and their per-GPU shards on a 148-SM B200 with 74 resident pairs."""

from __future__ import annotations

import ctypes

import pytest

from easy_as_b200.runtime import cuda_ext


def plan(M, N, K, batch=1, block_n=256, tma=True, sms=148, pairs=74, tile_m=0, block_k=0, with_bk=False):
    lib = cuda_ext.load()
    vals = [ctypes.c_int() for _ in range(6)]
    cuda_ext.check(lib.eas_gemm_f16_plan(M, N, K, batch, block_n, tile_m, block_k, int(tma), sms, pairs,
                                         *(ctypes.byref(v) for v in vals)), "plan")
    tm, tn, st, ks, pair, bk = (v.value for v in vals)
    out = {"pair": bool(pair), "tile": (tm, tn), "stages": st, "ksplit": ks}
    if with_bk:
        out["block_k"] = bk
    return out


@pytest.mark.parametrize("shape,want", [
    # C4 on 1, 2, 4, 8 GPUs (M split across ranks)
    ((8192, 8192, 8192), {"pair": True, "tile": (256, 512), "stages": 4, "ksplit": 1}),
    ((4096, 8192, 8192), {"pair": True, "tile": (256, 256), "stages": 6, "ksplit": 1}),   # wide adds a round
    ((2048, 8192, 8192), {"pair": True, "tile": (256, 512), "stages": 4, "ksplit": 1}),
    ((1024, 8192, 8192), {"pair": True, "tile": (256, 512), "stages": 4, "ksplit": 1}),
    # C5 on 1 GPU (batch 64) and on 8 (batch 8): K = 2088 is too short a loop for wide tiles
    ((4096, 4096, 2088, 64), {"pair": True, "tile": (256, 256), "stages": 6, "ksplit": 1}),
    ((4096, 4096, 2088, 8), {"pair": True, "tile": (256, 256), "stages": 6, "ksplit": 1}),
    # launches that leave most SMs idle split K, into at most 2 parts (bit-reproducible sums)
    ((512, 512, 4096), {"pair": True, "tile": (256, 256), "stages": 6, "ksplit": 2}),
    ((128, 8192, 8192), {"pair": False, "tile": (128, 256), "stages": 4, "ksplit": 2}),
    ((64, 4096, 2048, 1, 128), {"pair": False, "tile": (128, 128), "stages": 6, "ksplit": 2}),
    # few k-blocks: no split below 8 k-blocks per part
    ((512, 512, 1024), {"pair": True, "tile": (256, 256), "stages": 6, "ksplit": 2}),   # 16 k-blocks
    ((512, 512, 256), {"pair": True, "tile": (256, 256), "stages": 6, "ksplit": 1}),    # 4 k-blocks
])
def test_launch_choices(shape, want):
    M, N, K, *rest = shape
    batch = rest[0] if rest else 1
    block_n = rest[1] if len(rest) > 1 else 256
    assert plan(M, N, K, batch, block_n) == want


def test_c_not_storable_by_tma_uses_direct_stores_and_never_splits():
    assert plan(8192, 8192, 8192, tma=False) == {"pair": True, "tile": (256, 256), "stages": 7, "ksplit": 1}
    assert plan(128, 8192, 8192, tma=False)["ksplit"] == 1


def test_bad_arguments():
    with pytest.raises(ValueError):
        plan(256, 256, 256, block_n=64)


def test_autotune_space_maps_to_eight_distinct_kernels():
    """C4's autotune space BLOCK_M x BLOCK_N x BLOCK_K = {128, 256} x {128, 256} x {64, 128}
    (examples/matmul_dot_f16.py CONFIGS) names eight different launches at 8192^3."""
    seen = {}
    for bm in (128, 256):
        for bn in (128, 256):
            for bk in (64, 128):
                p = plan(8192, 8192, 8192, block_n=bn, tile_m=bm, block_k=bk, with_bk=True)
                assert p["pair"] == (bm == 256)
                assert p["block_k"] == bk
                assert p["tile"] == ((128, bn) if bm == 128 else (256, 2 * bn))
                seen[(bm, bn, bk)] = (p["pair"], p["tile"], p["stages"], p["block_k"])
    assert len(set(seen.values())) == 8


def test_explicit_stage_depth_halves_the_ring():
    assert plan(8192, 8192, 8192, tile_m=256, block_n=128, block_k=64)["stages"] == 6
    assert plan(8192, 8192, 8192, tile_m=256, block_n=128, block_k=128)["stages"] == 3
    assert plan(8192, 8192, 8192, tile_m=128, block_n=256, block_k=128)["stages"] == 2
    # a C that TMA cannot store keeps the pair tile at 256 x 256 (no wide kernel without TMA stores)
    assert plan(8192, 8192, 8192, tile_m=256, block_n=256, tma=False)["tile"] == (256, 256)


def test_library_choice_is_unchanged_by_zero_hints():
    for shape in ((8192, 8192, 8192), (4096, 8192, 8192), (128, 8192, 8192), (512, 512, 4096)):
        assert plan(*shape, tile_m=0, block_k=0) == plan(*shape)


@pytest.mark.parametrize("tile_m,block_k", [(64, 0), (0, 32), (512, 64), (128, 256)])
def test_bad_tile_requests(tile_m, block_k):
    with pytest.raises(ValueError):
        plan(256, 256, 256, tile_m=tile_m, block_k=block_k)

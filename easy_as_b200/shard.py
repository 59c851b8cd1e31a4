"""Split one kernel launch across GPUs by program id (one process per GPU).

Programs of an easy_as kernel never communicate (the IR has no atomics,
cross-program barriers or reductions), so a grid can be cut into contiguous
program-id ranges and each range run on its own GPU with no collective on the
data path.  The reference has the same idea on one device
(``PID_M_BASE/PID_N_BASE`` strips, easy_as ``examples/matmul_tiled.py:370-402``).

* :func:`program_range` gives rank ``r`` of ``w`` its balanced contiguous range.
* :func:`run_shard` launches the unmodified kernel for that range on the
  current GPU; the programs keep their global ids, and ``buffer_base`` lets a
  rank hold only its slice of a buffer.
* :func:`gather` brings the slices to one rank with ``torch.distributed``
  point-to-point transfers (NCCL over NVLink on GPUs, gloo on CPU); it is the
  only collective, and it is off the compute path.
"""

from __future__ import annotations

from typing import Any, Mapping, Sequence


def program_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous ``[lo, hi)`` share of ``total`` programs for ``rank`` of ``world`` (sizes differ by <= 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank/world: {rank}/{world}")
    return total * rank // world, total * (rank + 1) // world


def element_range(total_elems: int, block: int, rank: int, world: int) -> tuple[int, int]:
    """Elements owned by a rank when each program handles ``block`` consecutive elements."""
    programs = -(-total_elems // block)
    p0, p1 = program_range(programs, rank, world)
    return p0 * block, min(p1 * block, total_elems)


def run_shard(kernel: Any, *args: Any, _rank: int, _world: int, _axis: int = 0,
              _buffer_base: Mapping[str, int] | None = None, _sync: bool = True, **kwargs: Any) -> tuple[int, int]:
    """Run this rank's share of ``kernel(*args, **kwargs)``; returns the program range it ran.

    Launch options (``_grid``, ``_nthreads``, ``_shape``) describe the *whole*
    launch, exactly as for a single-GPU call.  An autotuned kernel is tuned on
    this rank's own range (its buffers may hold only their slice, so the whole
    launch cannot be timed here); the choice is cached per range.
    """
    from .runtime import get_runtime
    from .runtime.cuda import launch_geometry

    rt = get_runtime()
    fast = getattr(kernel, "_fast", None)
    key = None
    if fast is not None:
        key = kernel._fast_key(args, kwargs)
        if key is not None:
            key = ("shard", _rank, _world, _axis, tuple(sorted((_buffer_base or {}).items()))) + key
            hit = fast.get(key)
            if hit is not None:
                fl, r = hit
                if fl.rt is rt and rt.fast_run(fl, args, _sync):
                    return r
    raw = kernel._extract_runtime_options(kwargs)
    meta, runtime_args = kernel._bind_and_split(*args, **kwargs)

    def share(ck: Any, opts: Mapping[str, Any]) -> tuple[int, int] | None:
        geo = launch_geometry(ck, runtime_args, nthreads=opts["nthreads"], grid=opts["grid"], tptg=None,
                              shape=opts["shape"])
        return None if geo is None else program_range(geo[0][_axis], _rank, _world)

    if kernel._autotune_spec is not None:
        spec = kernel._autotune_spec

        def timer(ck: Any, m: Mapping[str, Any], opts: Mapping[str, Any]) -> float:
            r = share(ck, opts)
            if r is None:
                return 0.0
            return rt.benchmark_range(ck, runtime_args, m, axis=_axis, lo=r[0], hi=r[1], grid=opts["grid"],
                                      nthreads=opts["nthreads"], shape=opts["shape"], buffer_base=_buffer_base,
                                      repeat=spec.repeat, warmup=spec.warmup)

        extra = ("range", _axis, _rank, _world, tuple(sorted((_buffer_base or {}).items())))
        meta, opts = kernel._autotune_select(spec, meta, runtime_args, raw, timer=timer, key_extra=extra)
    else:
        opts = kernel._normalize_runtime_options(raw, meta, runtime_args)
    ck = kernel._compile_from_split(meta, runtime_args)
    r = share(ck, opts)
    if r is None:
        return (0, 0)
    lo, hi = r
    rt.run_range(ck, runtime_args, meta, axis=_axis, lo=lo, hi=hi, grid=opts["grid"], nthreads=opts["nthreads"],
                 shape=opts["shape"], buffer_base=_buffer_base, sync=_sync)
    if key is not None and len(fast) < 64:
        prep = getattr(rt, "fast_prepare", None)
        fl = prep(ck, runtime_args, opts, kernel._positions, axis=_axis, lo=lo, hi=hi,
                  buffer_base=_buffer_base) if prep is not None else None
        if fl is not None:
            fast[key] = (fl, r)
    return lo, hi


def gather(local: Any, out: Any | None, counts: Sequence[int], *, dst: int = 0, group: Any = None) -> Any:
    """Concatenate every rank's 1-D ``local`` slice (rank order) into ``out`` on rank ``dst``.

    ``counts[r]`` is the number of elements rank ``r`` holds.  Every rank uses batched
    point-to-point send/recv, which NCCL runs over NVLink/NVSwitch.
    """
    import torch.distributed as dist

    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    if len(counts) != world:
        raise ValueError("counts must have one entry per rank")
    if int(local.numel()) != int(counts[rank]):
        raise ValueError(f"rank {rank} holds {local.numel()} elements, counts says {counts[rank]}")
    if rank != dst:
        if counts[rank]:  # batched like the receives, so NCCL does not serialise it with other ops
            for w in dist.batch_isend_irecv([dist.P2POp(dist.isend, local.contiguous(), dst, group=group)]):
                w.wait()
        return None
    if out is None or int(out.numel()) != int(sum(counts)):
        raise ValueError("out on the destination rank must hold sum(counts) elements")
    ops = []
    off = 0
    for r, n in enumerate(counts):
        view = out.view(-1)[off:off + n]
        if r == dst:
            view.copy_(local.view(-1))
        elif n:
            ops.append(dist.P2POp(dist.irecv, view, r, group=group))
        off += n
    if ops:
        for w in dist.batch_isend_irecv(ops):
            w.wait()
    return out

"""``@eas.kernel``: argument binding, compile cache, autotune and dispatch.

Behaviour follows easy_as ``eas/kernel.py``:

* constexpr parameters are split from runtime ones by annotation (``:14-29``);
* the compile cache key is ``(sorted meta items, runtime_arg_signature)`` so
  scalar *values* never trigger a recompile (``:242-255``);
* launch options ``_sync, _grid, _tptg, _shape, _nthreads`` are popped from
  the keyword arguments and normalised (``:129-240``); ``_grid`` may be a
  callable ``(meta, runtime_args) -> dims``;
* ``_tptg`` must equal ``(block, 1, 1)`` in thread mode and ``(1, 1, 1)`` in
  SPMD mode, else ``ValueError`` (``:306-319``);
* ``@eas.autotune`` times every config once per key with the runtime's
  ``benchmark`` and caches the winner (``:73-127``).
"""

from __future__ import annotations

import inspect
import os as _os
from typing import Any, Callable, Mapping

import numpy as _np

from .autotune import AutotuneSpec, Config
from .compiler import CompiledKernel, compile as _compile, fast_arg_sig, runtime_arg_signature
from .meta import constexpr
from .compiler import _torch
from .runtime import env_bytes, get_runtime
from .tensor import Tensor as _Tensor

_LAUNCH_OPTIONS = ("_sync", "_shape", "_grid", "_tptg", "_nthreads")


def _dims(value: Any, what: str, *, lo: int, hi: int, pad: bool, min_value: int) -> tuple[int, ...]:
    if isinstance(value, int):
        dims = [int(value)]
    elif isinstance(value, (tuple, list)):
        dims = [int(x) for x in value]
    else:
        raise TypeError(f"{what} must be int or tuple/list of ints, got {type(value)!r}")
    if not (lo <= len(dims) <= hi):
        raise ValueError(f"{what} must have {lo}..{hi} dims" if hi < 99 else f"{what} must have >= {lo} dim")
    if pad:
        dims += [1] * (3 - len(dims))
    if any(d < min_value for d in dims):
        raise ValueError(f"{what} dims must be {'>= 0' if min_value == 0 else '> 0'}")
    return tuple(dims)


class Kernel:
    def __init__(self, fn: Callable[..., Any]):
        self.fn = fn
        self.name = fn.__name__
        self.sig = inspect.signature(fn)
        ann = inspect.get_annotations(fn, eval_str=True)
        self.meta_params = {n for n, p in self.sig.parameters.items()
                            if ann.get(n, p.annotation) is constexpr}
        self._cache: dict[tuple[Any, Any], CompiledKernel] = {}
        # fast argument binding when every parameter is a plain positional-or-keyword one
        kinds = {p.kind for p in self.sig.parameters.values()}
        self._simple = kinds <= {inspect.Parameter.POSITIONAL_OR_KEYWORD}
        self._names = tuple(self.sig.parameters)
        self._name_set = frozenset(self._names)
        self._defaults = {n: p.default for n, p in self.sig.parameters.items() if p.default is not p.empty}
        self._autotune_spec: AutotuneSpec | None = None
        self._tuned_cache: dict[tuple[Any, ...], Config] = {}
        self._tuned_times: dict[tuple[Any, ...], list[tuple[dict[str, Any], float]]] = {}
        # prepared launches of repeated calls (runtime fast path); EAS_FAST_LAUNCH=0 turns it off
        self._fast: dict[tuple[Any, ...], Any] | None = (
            None if _os.environ.get("EAS_FAST_LAUNCH", "1") in ("0", "off") else {})
        runtime_names = [n for n in self._names if n not in self.meta_params]
        self._positions = {n: i for i, n in enumerate(runtime_names)}
        self._runtime_first = tuple(self._names[:len(runtime_names)]) == tuple(runtime_names)

    def _set_autotune_spec(self, spec: AutotuneSpec) -> None:
        self._autotune_spec = spec

    # -- launch options ------------------------------------------------------
    def _extract_runtime_options(self, kwargs: dict[str, Any]) -> dict[str, Any]:
        sync = kwargs.pop("_sync", True)
        if not isinstance(sync, bool):
            raise TypeError(f"_sync must be bool, got {type(sync)!r}")
        shape = kwargs.pop("_shape", None)
        grid = kwargs.pop("_grid", None)
        tptg = kwargs.pop("_tptg", None)
        nthreads = kwargs.pop("_nthreads", None)
        if nthreads is not None:
            try:
                nthreads = int(nthreads)
            except Exception as e:
                raise TypeError(f"_nthreads must be an int-like value, got {type(nthreads)!r}") from e
            if nthreads < 0:
                raise ValueError("_nthreads must be >= 0")
        return {"sync": sync, "nthreads": nthreads, "grid": grid, "shape": shape, "tptg": tptg}

    def _normalize_runtime_options(self, raw: dict[str, Any], meta: dict[str, Any],
                                   runtime_args: dict[str, Any]) -> dict[str, Any]:
        shape = raw.get("shape")
        if shape is not None:
            if not isinstance(shape, (int, tuple, list)):
                raise TypeError(f"_shape must be int or tuple/list of ints, got {type(shape)!r}")
            shape = _dims(shape, "_shape", lo=1, hi=99, pad=False, min_value=0)
        grid = raw.get("grid")
        if callable(grid):
            grid = grid(meta, runtime_args)
        if grid is not None:
            if not isinstance(grid, (int, tuple, list)):
                raise TypeError(f"_grid must be int/tuple/list or callable, got {type(grid)!r}")
            grid = _dims(grid, "_grid", lo=1, hi=3, pad=True, min_value=0)
        tptg = raw.get("tptg")
        if tptg is not None:
            tptg = _dims(tptg, "_tptg", lo=1, hi=3, pad=True, min_value=1)
        return {"sync": bool(raw["sync"]), "nthreads": raw["nthreads"], "grid": grid,
                "shape": shape, "tptg": tptg}

    @staticmethod
    def _check_tptg(ck: CompiledKernel, tptg: tuple[int, int, int] | None) -> None:
        if tptg is None:
            raise RuntimeError("internal error: normalized tptg must not be None")
        expected = (int(ck.block_size), 1, 1) if ck.launch_mode == "thread" else (1, 1, 1)
        if tuple(int(x) for x in tptg) != expected:
            raise ValueError(f"_tptg must match kernel launch mode: expected {expected}, "
                             f"got ({tptg[0]}, {tptg[1]}, {tptg[2]})")

    # -- autotune --------------------------------------------------------------
    def _autotune_key(self, spec: AutotuneSpec, meta: Mapping[str, Any],
                      runtime_args: Mapping[str, Any]) -> tuple[Any, ...]:
        def norm(v: Any) -> Any:
            if isinstance(v, (bool, int, float, str, type(None))):
                return v
            if isinstance(v, (tuple, list)):
                return tuple(norm(x) for x in v)
            if isinstance(v, dict):
                return tuple(sorted((str(k), norm(x)) for k, x in v.items()))
            for conv in (int, float):
                try:
                    return conv(v)
                except Exception:
                    pass
            if hasattr(v, "shape"):
                try:
                    return ("shape", tuple(int(x) for x in v.shape))
                except Exception:
                    pass
            raise TypeError(f"autotune key value must be hashable/normalizable, got {type(v)!r}")

        key = []
        for name in spec.key:
            if name in meta:
                key.append(norm(meta[name]))
            elif name in runtime_args:
                key.append(norm(runtime_args[name]))
            else:
                raise KeyError(f"autotune key {name!r} not found in args/meta")
        return tuple(key)

    def _autotune_select(self, spec: AutotuneSpec, meta: dict[str, Any], runtime_args: dict[str, Any],
                         raw_opts: dict[str, Any], timer: Callable[..., float] | None = None,
                         key_extra: tuple[Any, ...] = ()) -> tuple[dict[str, Any], dict[str, Any]]:
        """Fastest config for this key (easy_as ``eas/kernel.py:73-127``): each config is timed
        with the runtime's ``benchmark`` (or ``timer(ck, meta, opts)`` when a caller times a
        different launch, such as one rank's program-id range, whose identity goes in
        ``key_extra``).  The seconds per config of a search are kept in ``_tuned_times``."""
        key = self._autotune_key(spec, meta, runtime_args) + tuple(key_extra)
        best = self._tuned_cache.get(key)
        disk_key = None
        if best is None:
            disk_key = _disk_key(self, spec, key, runtime_args)
            stored = _disk_load(disk_key)
            if stored is not None:
                best = next((c for c in spec.configs if dict(c.meta) == stored), None)
                if best is not None:
                    self._tuned_cache[key] = best
        if best is None:
            if timer is None:
                bench = getattr(get_runtime(), "benchmark", None)
                if not callable(bench):
                    raise RuntimeError("autotune requires a runtime with benchmark(); use the CUDA runtime")

                def timer(ck: CompiledKernel, m: dict[str, Any], opts: dict[str, Any]) -> float:
                    return float(bench(ck, runtime_args, m, repeat=spec.repeat, warmup=spec.warmup,
                                       nthreads=opts["nthreads"], grid=opts["grid"], tptg=opts["tptg"],
                                       shape=opts["shape"]))
            best_t = None
            times = []
            for cfg in spec.configs:
                m = {**meta, **dict(cfg.meta)}
                opts = self._normalize_runtime_options(raw_opts, m, runtime_args)
                ck = self._compile_from_split(m, runtime_args)
                t = float(timer(ck, m, opts))
                times.append((dict(cfg.meta), t))
                if best_t is None or t < best_t:
                    best, best_t = cfg, t
            if best is None:  # pragma: no cover
                raise RuntimeError("autotune failed to select a config")
            self._tuned_cache[key] = best
            self._tuned_times[key] = times
            _disk_store(disk_key, dict(best.meta))
        m = {**meta, **dict(best.meta)}
        return m, self._normalize_runtime_options(raw_opts, m, runtime_args)

    # -- compile / launch -----------------------------------------------------------
    def _compile_from_split(self, meta: dict[str, Any], runtime_args: dict[str, Any]) -> CompiledKernel:
        # kinds/dtypes/devices of the runtime args, never scalar values (same distinctions as
        # runtime_arg_signature, computed without sorting on the launch path)
        key = (tuple(sorted(meta.items())) if len(meta) > 1 else tuple(meta.items()),
               tuple((n, fast_arg_sig(v)) for n, v in runtime_args.items()),
               _os.environ.get("EAS_BOUNDS_CHECK"))   # checked and unchecked lowerings are distinct
        ck = self._cache.get(key)
        if ck is None:
            ck = _compile(self.fn, runtime_args, meta)
            self._cache[key] = ck
        return ck

    def _bind_and_split(self, /, *args: Any, **kwargs: Any) -> tuple[dict[str, Any], dict[str, Any]]:
        if self._simple and len(args) <= len(self._names):
            values = dict(zip(self._names, args))
            ok = True
            for k, v in kwargs.items():
                if k not in self._name_set or k in values:
                    ok = False
                    break
                values[k] = v
            if ok:
                for n in self._names[len(args):]:
                    if n not in values:
                        if n not in self._defaults:
                            ok = False
                            break
                        values[n] = self._defaults[n]
            if ok:
                meta, rt = {}, {}
                for n in self._names:
                    (meta if n in self.meta_params else rt)[n] = values[n]
                return meta, rt
        bound = self.sig.bind(*args, **kwargs)  # slow path: produces the standard error messages
        bound.apply_defaults()
        meta = {k: bound.arguments.pop(k) for k in list(bound.arguments) if k in self.meta_params}
        return meta, dict(bound.arguments)

    def _prepare(self, args: tuple[Any, ...], kwargs: dict[str, Any]):
        raw = self._extract_runtime_options(kwargs)
        meta, runtime_args = self._bind_and_split(*args, **kwargs)
        if self._autotune_spec is not None:
            meta, opts = self._autotune_select(self._autotune_spec, meta, runtime_args, raw)
        else:
            opts = self._normalize_runtime_options(raw, meta, runtime_args)
        ck = self._compile_from_split(meta, runtime_args)
        if raw.get("tptg") is not None:
            self._check_tptg(ck, opts.get("tptg"))
        return ck, meta, runtime_args, opts

    def compile(self, /, *args: Any, **kwargs: Any) -> CompiledKernel:
        return self._prepare(args, dict(kwargs))[0]

    def _fast_key(self, args: tuple[Any, ...], kwargs: dict[str, Any]) -> tuple[Any, ...] | None:
        """Key of a call that a prepared launch can repeat: the scalar values, the kind, dtype,
        device and size of every buffer (and which arguments are the same host array), the
        keyword arguments and the bounds-check switch.  None for calls the fast path does not
        take (autotuned kernels, callable grids, other argument types)."""
        if self._autotune_spec is not None or not self._runtime_first or len(args) != len(self._positions):
            return None
        parts: list[Any] = []
        for i, v in enumerate(args):
            t = type(v)
            if t is int or t is float or t is bool:
                parts.append((t, v))
            elif t is _Tensor:
                if v._device != "cuda":
                    return None
                parts.append((v._dtype, v._cuda_device(), v.nbytes))
            elif t is _np.ndarray:
                alias = next((j for j in range(i) if args[j] is v), i)
                parts.append((v.dtype, v.shape, alias, v.flags.c_contiguous))
            elif t.__name__ == "Tensor" and (tm := _torch()) is not None and t is tm.Tensor:
                parts.append((v.dtype, v.device, v.numel(), v.is_contiguous(), v.requires_grad))
            else:
                return None
        for k, v in kwargs.items():
            if k == "_sync":
                continue
            if callable(v) or isinstance(v, (list, dict)):
                return None
            parts.append((k, v))
        parts.append(env_bytes(b"EAS_BOUNDS_CHECK"))
        if any(type(v) is _np.ndarray for v in args):
            parts.append(env_bytes(b"EAS_ZERO_COPY"))   # host arrays: in place on pinned memory or not
        try:
            return tuple(parts)
        except TypeError:
            return None

    def __call__(self, /, *args: Any, **kwargs: Any) -> None:
        key = self._fast_key(args, kwargs) if self._fast is not None else None
        if key is not None:
            fl = self._fast.get(key)
            if fl is not None:
                rt = get_runtime()
                if fl.rt is rt and rt.fast_run(fl, args, kwargs.get("_sync", True)):
                    return
        ck, meta, runtime_args, opts = self._prepare(args, dict(kwargs))
        rt = get_runtime()
        rt.run(ck, runtime_args, meta, **opts)
        if key is not None and len(self._fast) < 64:
            prep = getattr(rt, "fast_prepare", None)
            fl = prep(ck, runtime_args, opts, self._positions) if prep is not None else None
            if fl is not None:
                try:
                    self._fast[key] = fl
                except TypeError:   # an unhashable keyword value
                    pass

    def to_cuda(self, /, *args: Any, **kwargs: Any) -> str:
        """Generated CUDA C++ source for this specialisation."""
        return self.compile(*args, **kwargs).src

    # the reference's name for the same query; returns the CUDA source here
    to_msl = to_cuda


# ---------------------------------------------------------------------------
# on-disk autotune results (EAS_CACHE_DIR/autotune.json; EAS_AUTOTUNE_CACHE=0 disables)
# ---------------------------------------------------------------------------


def _autotune_file() -> Any:
    import os
    from pathlib import Path

    if os.environ.get("EAS_AUTOTUNE_CACHE", "1") in ("0", "off", "false"):
        return None
    d = os.environ.get("EAS_CACHE_DIR", str(Path.home() / ".cache" / "easy_as_b200"))
    if d in ("", "0", "off", "none"):
        return None
    return Path(d) / "autotune.json"


def _disk_key(k: "Kernel", spec: AutotuneSpec, key: tuple[Any, ...], runtime_args: Mapping[str, Any]) -> str | None:
    import hashlib

    try:
        src = inspect.getsource(k.fn)
    except (OSError, TypeError):
        return None
    sig = runtime_arg_signature(runtime_args)
    blob = repr((k.fn.__module__, k.fn.__qualname__, src, [sorted(dict(c.meta).items()) for c in spec.configs],
                 key, sig, "sm_100a"))
    return hashlib.sha256(blob.encode()).hexdigest()


def _disk_load(dkey: str | None) -> dict[str, Any] | None:
    import json

    f = _autotune_file()
    if dkey is None or f is None or not f.exists():
        return None
    try:
        return json.loads(f.read_text()).get(dkey)
    except (OSError, ValueError):
        return None


def _disk_store(dkey: str | None, meta: dict[str, Any]) -> None:
    import json
    import os

    f = _autotune_file()
    if dkey is None or f is None:
        return
    try:
        f.parent.mkdir(parents=True, exist_ok=True)
        data = json.loads(f.read_text()) if f.exists() else {}
        data[dkey] = meta
        tmp = f.with_name(f"autotune.{os.getpid()}.tmp")
        tmp.write_text(json.dumps(data))
        os.replace(tmp, f)
    except (OSError, ValueError):
        pass


def kernel(fn: Callable[..., Any]) -> Kernel:
    k = Kernel(fn)
    spec = getattr(fn, "__eas_autotune_spec__", None)
    if isinstance(spec, AutotuneSpec):
        k._set_autotune_spec(spec)
    return k

"""Random SPMD kernels written in the DSL, for differential tests of the CUDA lowering against the
CPU oracle.

Each seed gives one kernel over f32 inputs ``x`` and ``y``, an f16 input ``h``, a u32 scalar
``S`` and an f32 scalar ``alpha``, storing an f32 expression to ``out``, an integer
expression (as f32) to ``outi`` and the f32 expression rounded to f16 to ``outh``.  The expressions mix every elementwise op of the DSL with
exactly defined results: f32 add, mul and fma (single rounding), f32 <-> f16 <-> u32 casts,
u32 add, mul, floordiv and mod by non-zero constants (mod 2^32), u32 comparisons, boolean
and/or/not, ``where``, and masked loads (zero fill) at shifted or permuted offsets.  Results
are therefore bit-exact between any two correct implementations."""

from __future__ import annotations

import random

import numpy as np

import eas
from eas import mk  # noqa: F401  (the generated source refers to it)


class _Gen:
    def __init__(self, seed: int):
        self.r = random.Random(seed)
        self.lines: list[str] = []
        self.n = 0

    def fresh(self, expr: str) -> str:
        self.n += 1
        name = f"v{self.n}"
        self.lines.append(f"    {name} = {expr}")
        return name

    # u32 expressions
    def u(self, depth: int) -> str:
        r = self.r
        if depth <= 0 or r.random() < 0.25:
            # leaves are traced values (constants only ever appear on the right of an operator)
            return r.choice(["offs", "pid", "S", "mk.to_u32(a)", f"(pid + {r.randint(0, 1 << 20)})", "(offs % 97)"])
        op = r.choice(["add", "mul", "div", "mod", "where", "cast"])
        x = self.u(depth - 1)
        if op == "add":
            return self.fresh(f"{x} + {self.u(depth - 1)}")
        if op == "mul":
            return self.fresh(f"{x} * {r.choice([3, 7, 255, 65537, 'S'])}")
        if op == "div":
            return self.fresh(f"{x} // {r.randint(1, 1000)}")
        if op == "mod":
            return self.fresh(f"{x} % {r.randint(1, 1 << 16)}")
        if op == "where":
            return self.fresh(f"mk.where({self.cond(depth - 1)}, {x}, {self.u(depth - 1)})")
        return self.fresh(f"mk.to_u32({self.f(depth - 1)})")

    def cond(self, depth: int) -> str:
        r = self.r
        kind = r.choice(["lt", "lt", "and", "or", "not"]) if depth > 0 else "lt"
        if kind == "lt":
            return self.fresh(f"{self.u(depth - 1)} < {self.u(depth - 1)}")
        if kind == "and":
            return self.fresh(f"{self.cond(depth - 1)} & {self.cond(depth - 1)}")
        if kind == "or":
            return self.fresh(f"{self.cond(depth - 1)} | {self.cond(depth - 1)}")
        return self.fresh(f"~{self.cond(depth - 1)}")

    # f32 expressions
    def f(self, depth: int) -> str:
        r = self.r
        if depth <= 0 or r.random() < 0.2:
            return r.choice(["a", "b", "hv", "alpha", "mk.to_f32(offs)", "1.5", "-0.25"])
        op = r.choice(["add", "mul", "fma", "where", "f16", "fromu", "load"])
        if op == "add":
            return self.fresh(f"{self.f(depth - 1)} + {self.f(depth - 1)}")
        if op == "mul":
            return self.fresh(f"{self.f(depth - 1)} * {self.f(depth - 1)}")
        if op == "fma":
            return self.fresh(f"mk.fma({self.f(depth - 1)}, {self.f(depth - 1)}, {self.f(depth - 1)})")
        if op == "where":
            return self.fresh(f"mk.where({self.cond(depth - 1)}, {self.f(depth - 1)}, {self.f(depth - 1)})")
        if op == "f16":
            return self.fresh(f"mk.to_f32(mk.to_f16({self.f(depth - 1)}))")
        if op == "fromu":
            return self.fresh(f"mk.to_f32({self.u(depth - 1)})")
        # a masked load at a shifted or permuted offset (always inside [0, N) when the mask holds)
        idx = r.choice(["(offs + {c}) % N", "(offs * {o}) % N", "offs"]).format(c=r.randint(1, 500),
                                                                              o=r.choice([3, 5, 7, 11]))
        buf = r.choice(["x", "y"])
        return self.fresh(f"mk.load({buf}, {idx}, m & {self.cond(depth - 1)})")


def kernel_source(seed: int) -> str:
    g = _Gen(seed)
    depth = 2 + seed % 3
    fexpr = g.f(depth)
    iexpr = g.u(depth)
    smask = g.cond(1)
    body = "\n".join(g.lines)
    return f'''
@eas.kernel
def fuzz_{seed}(x, y, h, out, outi, outh, N, S, alpha, BLOCK: eas.constexpr):
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    pid = mk.program_id(0)
    m = offs < N
    a = mk.load(x, offs, m)
    b = mk.load(y, offs, m)
    hv = mk.to_f32(mk.load(h, offs, m))
{body}
    mk.store(out, offs, {fexpr}, m)
    mk.store(outi, offs, mk.to_f32({iexpr}), m & {smask})
    mk.store(outh, offs, mk.to_f16({fexpr}), m)
'''


def make(seed: int):
    """(kernel, source) for one seed."""
    src = kernel_source(seed)
    ns: dict = {"eas": eas, "mk": mk}
    exec(compile(src, f"<fuzz_{seed}>", "exec"), ns)
    return ns[f"fuzz_{seed}"], src


def inputs(seed: int, n: int) -> dict:
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(n) * 100).astype(np.float32)
    y = rng.standard_normal(n).astype(np.float32)
    x[: min(n, 4)] = [0.0, -0.0, 3.0e38, -1.0e-40][: min(n, 4)]   # signed zero, large, subnormal
    h = rng.standard_normal(n).astype(np.float16)
    return {"x": x, "y": y, "h": h, "out": np.full(n, -7.0, np.float32), "outi": np.full(n, -7.0, np.float32),
            "outh": np.full(n, -3.0, np.float16),
            "N": n, "S": int(rng.integers(1, 1 << 31)), "alpha": float(np.float32(rng.standard_normal()))}


# ---------------------------------------------------------------------------
# thread-mode kernels: threadgroup memory, barriers, dot
# ---------------------------------------------------------------------------


def thread_kernel_source(seed: int) -> tuple[str, dict]:
    """A kernel of NT threads per group: every thread fills distinct slots of two threadgroup
    arrays (masked global loads and f32 expressions; the second array is f16 in about half the
    seeds), then after a barrier reads other threads'
    slots at permuted positions into an fma chain, optionally adds an ``mk.dot`` over the
    arrays, optionally refills one array in a second phase, and stores one result per thread."""
    r = random.Random(10_000 + seed)
    nt = r.choice([32, 64, 128, 256])
    ts = nt * r.choice([1, 2, 3]) + r.choice([0, 0, 5, 17])
    reps = r.randint(1, 6)
    sb_f16 = r.random() < 0.5          # second threadgroup array in f16 (stores round, loads widen)
    g = _Gen(20_000 + seed)
    lines = []
    fill = []
    for i in range(0, ts, nt):
        src_idx = r.choice(["(pid * {ts} + t + {i}) % N", "(gi * {p} + {i}) % N"]).format(ts=ts, i=i, p=r.choice([3, 5]))
        fill.append(f"    mk.store(sa, t + {i}, mk.load(x, {src_idx}, m2 & (t + {i} < {ts})), t + {i} < {ts})")
        val = r.choice(['a', 'b', 'a * b', 'mk.fma(a, alpha, b)', 'mk.to_f32(t + ' + str(i) + ')'])
        if sb_f16:
            val = f"mk.to_f16({val})"
        fill.append(f"    mk.store(sb, t + {i}, {val}, t + {i} < {ts})")
    chain = []
    acc = g.f(1)
    lines.extend(g.lines)
    g.lines = []
    for j in range(reps):
        p_, q_ = r.choice([1, 3, 5, 7]), r.randint(0, ts - 1)
        sb_val = f"mk.load(sb, (t + {j * 13 + 1}) % {ts})"
        if sb_f16:
            sb_val = f"mk.to_f32({sb_val})"
        chain.append(f"    acc = mk.fma(mk.load(sa, (t * {p_} + {q_}) % {ts}), {sb_val}, acc)")
    if r.random() < 0.6 and not sb_f16:
        k = r.randint(1, min(16, ts))
        sa_stride = r.choice([1, 1, 2]) if ts >= 2 * k else 1
        span_a = (k - 1) * sa_stride + 1
        chain.append(f"    acc = acc + mk.dot(sa, t % {ts - span_a + 1}, {sa_stride}, sb, (t * 3) % {ts - k + 1}, 1, {k})")
    second = []
    if r.random() < 0.5:
        second = ["    mk.barrier()"] + [f"    mk.store(sa, t + {i}, acc * {r.choice(['0.5', 'alpha', 'a'])}, t + {i} < {ts})"
                                          for i in range(0, ts, nt)] + \
                 ["    mk.barrier()", f"    acc = acc + mk.load(sa, (t * 7 + 3) % {ts})"]
    body = "\n".join(lines)
    src = f'''
@eas.kernel
def tfuzz_{seed}(x, y, out, N, S, alpha, NT: eas.constexpr):
    t = mk.tid(0, NT)
    pid = mk.program_id(0)
    gi = pid * NT + t
    m = gi < N
    m2 = gi < N + 0
    a = mk.load(x, gi, m)
    b = mk.load(y, gi, m)
    offs = gi
    hv = a
    sa = mk.alloc_tg({ts})
    sb = mk.alloc_tg{'_f16' if sb_f16 else ''}({ts})
{chr(10).join(fill)}
    mk.barrier()
{body}
    acc = {acc}
{chr(10).join(chain)}
{chr(10).join(second)}
    mk.store(out, gi, acc, m)
'''
    return src, {"NT": nt}


def make_thread(seed: int):
    """(kernel, source, meta) for one seed."""
    src, meta = thread_kernel_source(seed)
    ns: dict = {"eas": eas, "mk": mk}
    exec(compile(src, f"<tfuzz_{seed}>", "exec"), ns)
    return ns[f"tfuzz_{seed}"], src, meta


def thread_inputs(seed: int, n: int) -> dict:
    rng = np.random.default_rng(50_000 + seed)
    return {"x": rng.standard_normal(n).astype(np.float32), "y": rng.standard_normal(n).astype(np.float32),
            "out": np.full(n, -7.0, np.float32), "N": n, "S": int(rng.integers(1, 1 << 20)),
            "alpha": float(np.float32(rng.standard_normal()))}

"""Generate golden vectors from the reference implementation itself.

Run once, in a container where the reference checkout is present:

    python tests/golden/make_golden.py --reference <path-to-Ntilang-checkout>

It imports the reference package (``python/ntilang``) and its ``examples/*.py`` kernels,
evaluates each kernel with the reference's own serial NumPy evaluator
``ntilang.testing.reference`` (python/ntilang/testing.py:34) — and, for a larger
bit-exact scan case, ``ntilang.scan.evaluate`` (scan.py:349-389) — on seeded inputs, and
writes ``tests/golden/<case>.npz`` with the inputs, outputs and parameters.  The tests
and the GPU box only read the committed ``.npz`` files; nothing imports the reference at
test time.
"""

from __future__ import annotations

import argparse
import importlib.util
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def load_example(ref: Path, name: str):
    spec = importlib.util.spec_from_file_location(f"ref_example_{name}", ref / "examples" / f"{name}.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--only", default="", help="comma-separated case-name prefixes to (re)write")
    args = ap.parse_args()
    only = tuple(x for x in args.only.split(",") if x)
    ref = args.reference.resolve()
    # The reference package is also called `ntilang`: make sure it, not this repo's alias, is imported.
    sys.path = [str(ref / "python")] + [p for p in sys.path if Path(p or ".").resolve() != HERE.parents[1]]
    import ntilang  # noqa: F401  (the reference)
    from ntilang import scan as ref_scan
    from ntilang.testing import reference

    assert Path(ntilang.__file__).resolve().is_relative_to(ref), ntilang.__file__

    def wanted(name):
        return not only or name.startswith(only)

    def save(name, **arrays):
        if not wanted(name):
            return
        np.savez_compressed(HERE / f"{name}.npz", **arrays)
        print("wrote", name, {k: getattr(v, "shape", v) for k, v in arrays.items()})

    t0 = time.time()
    # vector add (examples/vector_add.py)
    va = load_example(ref, "vector_add")
    rng = np.random.default_rng(0)
    a = rng.normal(size=1000).astype(np.float32)
    b = rng.normal(size=1000).astype(np.float32)
    c = np.full_like(a, np.nan)
    reference(va.vector_add(n=1000, block=128), a, b, c)
    save("vadd_1000", a=a, b=b, c=c)

    # cumsum (examples/cumsum.py), forward and reverse
    cs = load_example(ref, "cumsum")
    for rows, cols, seed in ((7, 65, 1), (4, 256, 2)):
        rng = np.random.default_rng(seed)
        x = rng.uniform(-1, 1, size=(rows, cols)).astype(np.float32)
        for rev in (False, True):
            y = np.full_like(x, np.nan)
            reference(cs.cumsum(rows, cols, reverse=rev), x, y)
            save(f"cumsum_{rows}x{cols}_{'rev' if rev else 'fwd'}", x=x, y=y, reverse=np.array(rev))
    # special values (signed zeros, infinities, NaN) like the reference's scan tests
    rng = np.random.default_rng(407)
    x = (rng.normal(size=(3, 97)) * 30).astype(np.float32)
    x[0, :6] = [0.0, -0.0, np.inf, -np.inf, np.nan, np.nan]
    x[1, :] = np.nan
    x[2, :5] = [-0.0, -0.0, -0.0, 1e38, 1e38]
    for rev in (False, True):
        y = np.full_like(x, 7.0)
        with np.errstate(over="ignore", invalid="ignore"):
            reference(cs.cumsum(3, 97, reverse=rev), x, y)
        save(f"cumsum_special_{'rev' if rev else 'fwd'}", x=x, y=y, reverse=np.array(rev))
    # a larger scan case through the reference's scan evaluator (the device order)
    rng = np.random.default_rng(3)
    x = rng.uniform(-1, 1, size=(64, 1000)).astype(np.float32)
    for rev in (False, True):
        y = ref_scan.evaluate(x, "sum", 1, rev)
        save(f"cumsum_eval_64x1000_{'rev' if rev else 'fwd'}", x=x, y=y, reverse=np.array(rev))

    # softmax (examples/softmax.py)
    sm = load_example(ref, "softmax")
    for rows, cols, seed, scale in ((9, 113, 491, 100.0), (4, 512, 4, 2.0)):
        rng = np.random.default_rng(seed)
        x = (rng.normal(size=(rows, cols)) * scale).astype(np.float32)
        y = np.full_like(x, np.nan)
        reference(sm.softmax(rows, cols), x, y)
        save(f"softmax_{rows}x{cols}", x=x, y=y)

    # RMSNorm (examples/rmsnorm.py)
    rn = load_example(ref, "rmsnorm")
    for rows, cols, seed in ((6, 1024, 5), (5, 768, 6)):
        rng = np.random.default_rng(seed)
        x = rng.normal(size=(rows, cols)).astype(np.float32)
        w = rng.normal(1.0, 0.1, size=cols).astype(np.float32)
        y = np.full_like(x, np.nan)
        reference(rn.rmsnorm(rows, cols, eps=1e-6), x, w, y)
        save(f"rmsnorm_{rows}x{cols}", x=x, w=w, y=y, eps=np.array(1e-6))

    # LayerNorm (examples/layernorm.py)
    ln = load_example(ref, "layernorm")
    for rows, cols, seed in ((6, 1024, 7), (5, 768, 8), (3, 100, 9)):
        if not wanted(f"layernorm_{rows}x{cols}"):
            continue
        rng = np.random.default_rng(seed)
        x = (rng.normal(size=(rows, cols)) * 2.0 + 0.5).astype(np.float32)
        w = rng.normal(1.0, 0.1, size=cols).astype(np.float32)
        bb = rng.normal(0.0, 0.1, size=cols).astype(np.float32)
        y = np.full_like(x, np.nan)
        reference(ln.layernorm(rows, cols, eps=1e-5), x, w, bb, y)
        save(f"layernorm_{rows}x{cols}", x=x, w=w, b=bb, y=y, eps=np.array(1e-5))

    # Shared-memory transpose (examples/transpose.py)
    tr = load_example(ref, "transpose")
    for m, n, seed in ((65, 71, 10), (33, 130, 11)):
        if not wanted(f"transpose_{m}x{n}"):
            continue
        rng = np.random.default_rng(seed)
        a = rng.normal(size=(m, n)).astype(np.float32)
        bt = np.full((n, m), np.nan, np.float32)
        reference(tr.transpose(m, n), a, bt)
        save(f"transpose_{m}x{n}", a=a, b=bt)

    # GEMM (examples/matmul.py) and GEMM + bias + ReLU (examples/matmul_relu.py)
    mm = load_example(ref, "matmul")
    rng = np.random.default_rng(11)
    a = rng.normal(size=(65, 37)).astype(np.float16)
    b = rng.normal(size=(37, 71)).astype(np.float16)
    c = np.full((65, 71), np.nan, np.float32)
    reference(mm.matmul(), a, b, c)
    save("gemm_65x71x37", a=a, b=b, c=c)
    mr = load_example(ref, "matmul_relu")
    rng = np.random.default_rng(61)
    a = rng.normal(size=(65, 37)).astype(np.float16)
    b = rng.normal(size=(37, 71)).astype(np.float16)
    bias = rng.normal(size=(65, 71)).astype(np.float32)
    c = np.full((65, 71), np.nan, np.float32)
    reference(mr.matmul_relu(), a, b, bias, c)
    save("gemm_relu_65x71x37", a=a, b=b, bias=bias, c=c, alpha=np.array(0.5))

    # FlashAttention-2 forward (examples/flash_attention.py), non-causal and causal
    fa = load_example(ref, "flash_attention")
    for causal in (False, True):
        rng = np.random.default_rng(21 + int(causal))
        shape = (1, 2, 128, 64)
        q, k, v = ((rng.normal(size=shape) * 0.5).astype(np.float16) for _ in range(3))
        o = np.full(shape, np.nan, np.float16)
        kern = fa.flash_attention(1, 2, 128, 64, is_causal=causal)
        reference(kern, q, k, v, o)
        scale = (1.0 / np.sqrt(64)) * 1.44269504
        save(f"fa2_1x2x128x64_{'causal' if causal else 'full'}", q=q, k=k, v=v, o=o, scale_log2=np.array(scale),
             causal=np.array(causal))

    # Row sum and maximum scans of one tile (examples/scan.py), forward and reverse, with
    # signed zeros, infinities and NaN in some rows.
    sc_ex = load_example(ref, "scan")
    rng = np.random.default_rng(51)
    x = rng.normal(size=(9, 113)).astype(np.float32)
    x[2, 10:20] = 0.0
    x[2, 12] = -0.0
    x[3, :] = -0.0
    x[4, 5] = np.nan
    x[5, 40] = np.inf
    x[6, 7] = -np.inf
    for rev in (False, True):
        prefix = np.full_like(x, np.nan)
        maximum = np.full_like(x, np.nan)
        reference(sc_ex.scan(9, 113, reverse=rev), x, prefix, maximum)
        save(f"scan_9x113_{'rev' if rev else 'fwd'}", x=x, prefix=prefix, maximum=maximum, reverse=np.array(rev))

    # Generic elementwise programs (the NVRTC path): the reference's own examples, then the
    # shared programs of pw_programs.py built under the reference package.
    fa_ex = load_example(ref, "fragment_affine")
    rng = np.random.default_rng(31)
    a = np.concatenate([np.linspace(-2, 2, 129, dtype=np.float32), rng.normal(size=128).astype(np.float32)])
    b = np.full_like(a, np.nan)
    reference(fa_ex.fragment_affine(), a, b)
    save("pw_fragment_affine_257", a=a, b=b)
    pw_ex = load_example(ref, "piecewise")
    a = np.concatenate([np.linspace(-2, 2, 61, dtype=np.float32), np.array([-0.0, 0.0, 1.0, -1.0], np.float32),
                        np.random.default_rng(32).normal(size=28).astype(np.float32) * 3])
    b = np.full_like(a, np.nan)
    reference(pw_ex.piecewise(), a, b)
    save("pw_piecewise_93", a=a, b=b)
    ws_ex = load_example(ref, "window_sum")
    a = np.random.default_rng(33).normal(size=(7, 3, 5)).astype(np.float32)
    windows = ((-1, 5), (0, 0), (2, 4), (10, 10), (3, 2))
    outs = []
    for rows, columns in windows:
        b = np.full(7, np.nan, np.float32)
        reference(ws_ex.window_sum(), a, b, rows, columns)
        outs.append(b)
    save("pw_window_sum_7x3x5", a=a, b=np.stack(outs), windows=np.array(windows, np.int32))
    sys.path.insert(0, str(HERE))
    import pw_programs
    import ntilang.language as T_ref

    for name, (factory, build, outs_idx, scalars) in pw_programs.PROGRAMS.items():
        if not wanted(f"pw_{name}"):
            continue
        arrays = build(np.random.default_rng(40 + sorted(pw_programs.PROGRAMS).index(name)))
        inputs = [x.copy() for x in arrays]
        reference(factory(T_ref, ntilang.compile), *arrays, *scalars)
        save(f"pw_{name}", **{f"in{i}": x for i, x in enumerate(inputs)}, **{f"out{i}": arrays[i] for i in outs_idx},
             scalars=np.array(scalars, np.float64))
    print(f"done in {time.time() - t0:.1f} s")


if __name__ == "__main__":
    main()

"""Launchers: an ``OpSpec`` plus argument tensors -> one C-ABI call on the current stream.

This replaces the reference's ``executable(*ffi_arguments)`` (python/ntilang/compiler.py:197):
tensors cross as data pointers, sizes come from the recognised op (symbolic dimensions
are bound from the actual tensor shapes), and the stream is
``torch.cuda.current_stream(device)`` — the stream TVM-FFI's environment stream follows in
the reference.
"""

from __future__ import annotations

from . import _lib
from .recognize import OpSpec

_BINARY_OPS = {"+": 0, "-": 1, "*": 2}


def _ptr(t):
    return t.data_ptr()


_workspaces: dict = {}


def gemm_workspace(device, nbytes: int):
    """A zero-initialised workspace of at least ``nbytes`` on ``device``, cached per device.

    The split-K GEMM keeps its flag words in the first 4 KB of every workspace and leaves
    them zero after every successful call, so the buffer is reused as is for any shape that
    fits.  Calls that share it run in stream order on the caller's stream.
    """
    import torch

    key = torch.device(device).index
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf


def abi_call(spec: OpSpec):
    """(C-ABI entry point, argument recipe) of a recognised op.

    A recipe item is ``("ptr", i)`` (argument i's data pointer), ``("null",)``, ``("i32", v)``,
    ``("i64", v)``, ``("f32", v)``, ``("dim", i, d)`` (argument i's size along d, int64),
    ``("rows", i)`` (product of argument i's sizes but the last) or ``("stream",)``.  The same
    recipe drives ``launch`` and the standalone module ``CompiledKernel.save()`` writes.
    """
    f, p, a = spec.family, spec.params, spec.args
    if f == "elementwise":
        count = ("dim", a["c"], 0) if isinstance(p["count"], str) else ("i64", int(p["count"]))
        return "ntl_binary_f32", [("i32", _BINARY_OPS[p["op"]]), ("ptr", a["a"]), ("ptr", a["b"]), ("ptr", a["c"]),
                                  count, ("stream",)]
    if f in ("cumsum", "cummax"):
        return f"ntl_{f}_f32", [("ptr", a["x"]), ("ptr", a["y"]), ("rows", a["x"]), ("dim", a["x"], -1),
                                ("i32", int(p["reverse"])), ("stream",)]
    if f == "softmax":
        return "ntl_softmax_f32", [("ptr", a["x"]), ("ptr", a["y"]), ("dim", a["x"], 0), ("dim", a["x"], 1),
                                   ("stream",)]
    if f == "rmsnorm":
        return "ntl_rmsnorm_f32", [("ptr", a["x"]), ("ptr", a["w"]), ("ptr", a["y"]), ("dim", a["x"], 0),
                                   ("dim", a["x"], 1), ("f32", float(p["eps"])), ("f32", float(p["inv_n"])),
                                   ("stream",)]
    if f == "layernorm":
        return "ntl_layernorm_f32", [("ptr", a["x"]), ("ptr", a["w"]), ("ptr", a["b"]), ("ptr", a["y"]),
                                     ("dim", a["x"], 0), ("dim", a["x"], 1), ("f32", float(p["eps"])),
                                     ("f32", float(p["inv_n"])), ("stream",)]
    if f == "transpose":
        return "ntl_transpose_f32", [("ptr", a["a"]), ("ptr", a["b"]), ("dim", a["a"], 0), ("dim", a["a"], 1),
                                     ("stream",)]
    if f == "gemm":
        # Data-parallel tiles: on B200 splitting the last wave along K (ntl_gemm_f16_f32_ws)
        # measured no faster at any shape tried; the partial-sum fixup costs about what the
        # idle part of the wave does.
        tb = int(p["transpose_b"])
        return "ntl_gemm_f16_f32", [("ptr", a["a"]), ("ptr", a["b"]), ("ptr", a["c"]),
                                    ("ptr", a["bias"]) if "bias" in a else ("null",), ("i32", int(p["bias_mode"])),
                                    ("f32", float(p["alpha"])), ("i32", int(p["relu"])), ("dim", a["a"], 0),
                                    ("dim", a["b"], 0 if tb else 1), ("dim", a["a"], 1), ("i32", tb), ("stream",)]
    if f == "fa2":
        return "ntl_fa2_fwd_f16", [("ptr", a["q"]), ("ptr", a["k"]), ("ptr", a["v"]), ("ptr", a["o"]),
                                   ("dim", a["q"], 0), ("dim", a["q"], 1), ("dim", a["q"], 2), ("dim", a["q"], 3),
                                   ("f32", float(p["scale_log2"])), ("i32", int(p["causal"])), ("stream",)]
    raise RuntimeError(f"no C-ABI call for op family {f!r}")  # pragma: no cover


def abi_calls(spec: OpSpec):
    """Every C-ABI call of a recognised op, in launch order: one per family, one per scan for a
    kernel with several row scans of one tile (examples/scan.py)."""
    if spec.family == "scans":
        a = spec.args
        return [(f"ntl_{'cumsum' if kind == 'sum' else 'cummax'}_f32",
                 [("ptr", a["x"]), ("ptr", a[f"y{i}"]), ("rows", a["x"]), ("dim", a["x"], -1), ("i32", int(rev)),
                  ("stream",)])
                for i, (kind, rev) in enumerate(spec.params["scans"])]
    return [abi_call(spec)]


def _recipe_args(recipe, tensors, stream):
    out = []
    for item in recipe:
        kind = item[0]
        if kind == "ptr":
            out.append(_ptr(tensors[item[1]]))
        elif kind == "null":
            out.append(None)
        elif kind in ("i32", "i64", "f32"):
            out.append(item[1])
        elif kind == "dim":
            out.append(int(tensors[item[1]].shape[item[2]]))
        elif kind == "rows":
            t = tensors[item[1]]
            out.append(t.numel() // t.shape[-1] if t.dim() > 1 else 1)
        elif kind == "stream":
            out.append(stream)
        else:  # pragma: no cover - recipes come from abi_call
            raise RuntimeError(f"bad recipe item {item!r}")
    return out


def launch(spec: OpSpec, tensors, stream: int, bindings=None) -> None:
    if spec.family == "pointwise":
        spec.params["kernel"].launch(tensors, bindings or {}, stream)
        return
    for entry, recipe in abi_calls(spec):
        _lib.call(entry, *_recipe_args(recipe, tensors, stream))


def _getter(item):
    kind = item[0]
    if kind == "ptr":
        i = item[1]
        return lambda t, s: t[i].data_ptr()
    if kind == "null":
        return lambda t, s: None
    if kind in ("i32", "i64", "f32"):
        v = item[1]
        return lambda t, s: v
    if kind == "dim":
        i, d = item[1], item[2]
        return lambda t, s: t[i].shape[d]
    if kind == "rows":
        i = item[1]
        return lambda t, s: (t[i].numel() // t[i].shape[-1]) if t[i].dim() > 1 else 1
    return lambda t, s: s


def make_launcher(spec: OpSpec):
    """launch(spec, ...) with the per-op work done once: the C entry points bound and each
    argument recipe turned into getters.  Returns ``run(tensors, stream, bindings)``."""
    if spec.family == "pointwise":
        kernel = spec.params["kernel"]
        return lambda tensors, stream, bindings: kernel.launch(tensors, bindings, stream)
    handle = _lib.lib()
    calls = [(entry, getattr(handle, entry), tuple(_getter(it) for it in recipe)) for entry, recipe in abi_calls(spec)]

    def run(tensors, stream, bindings):
        for entry, fn, getters in calls:
            rc = fn(*[g(tensors, stream) for g in getters])
            if rc:
                msg = handle.ntl_last_error()
                raise _lib.KernelError(entry, rc, msg.decode() if msg else "")

    return run


ABI_CALL = {
    "elementwise": "ntl_binary_f32(op, A, B, C, n, stream)",
    "cumsum": "ntl_cumsum_f32(X, Y, rows, cols, reverse, stream)",
    "cummax": "ntl_cummax_f32(X, Y, rows, cols, reverse, stream)",
    "scans": "ntl_cumsum_f32 / ntl_cummax_f32(X, Y_i, rows, cols, reverse_i, stream), one per output",
    "softmax": "ntl_softmax_f32(X, Y, rows, cols, stream)",
    "rmsnorm": "ntl_rmsnorm_f32(X, W, Y, rows, cols, eps, inv_n, stream)",
    "layernorm": "ntl_layernorm_f32(X, W, B, Y, rows, cols, eps, inv_n, stream)",
    "transpose": "ntl_transpose_f32(A, B, m, n, stream)",
    "gemm": "ntl_gemm_f16_f32(A, B, C, bias, bias_mode, alpha, relu, M, N, K, b_trans, stream)",
    "fa2": "ntl_fa2_fwd_f16(Q, K, V, O, batch, heads, seq, dim, scale_log2, causal, stream)",
    "pointwise": "ntl_rtc_build(cuda_source, name, &handle) once, then ntl_rtc_launch(handle, grid, 256, args, stream)",
}


def describe(spec: OpSpec, name: str, target: str) -> str:
    """The launch plan: what will be launched and how (comment lines)."""
    params = {k: v for k, v in spec.params.items() if k != "kernel"}
    lines = [
        f"# ntilang_b200 launch plan for kernel `{name}` (target {target})",
        f"# op family : {spec.family}",
        f"# parameters: {', '.join(f'{k}={v}' for k, v in params.items())}",
        f"# arguments : {', '.join(f'{k}=arg{v}' for k, v in spec.args.items())}",
        f"# C ABI     : {ABI_CALL[spec.family]}  (libntl_kernels.so, include/ntl_kernels.h)",
    ]
    return "\n".join(lines) + "\n"

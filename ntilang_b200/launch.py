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


def _size(value, tensor, dim):
    """Static size from the spec, or the bound value of a symbolic dimension."""
    return int(tensor.shape[dim]) if isinstance(value, str) else int(value)


def launch(spec: OpSpec, tensors, stream: int) -> None:
    f = spec.family
    p = spec.params
    a = spec.args
    if f == "elementwise":
        x, y, out = tensors[a["a"]], tensors[a["b"]], tensors[a["c"]]
        n = _size(p["count"], out, 0)
        _lib.call("ntl_binary_f32", _BINARY_OPS[p["op"]], _ptr(x), _ptr(y), _ptr(out), n, stream)
    elif f == "cumsum":
        x, y = tensors[a["x"]], tensors[a["y"]]
        rows = x.numel() // x.shape[-1] if x.dim() > 1 else 1
        cols = int(x.shape[-1])
        _lib.call("ntl_cumsum_f32", _ptr(x), _ptr(y), rows, cols, int(p["reverse"]), stream)
    elif f == "softmax":
        x, y = tensors[a["x"]], tensors[a["y"]]
        _lib.call("ntl_softmax_f32", _ptr(x), _ptr(y), int(x.shape[0]), int(x.shape[1]), stream)
    elif f == "rmsnorm":
        x, w, y = tensors[a["x"]], tensors[a["w"]], tensors[a["y"]]
        _lib.call("ntl_rmsnorm_f32", _ptr(x), _ptr(w), _ptr(y), int(x.shape[0]), int(x.shape[1]),
                  float(p["eps"]), float(p["inv_n"]), stream)
    elif f == "layernorm":
        x, w, b, y = tensors[a["x"]], tensors[a["w"]], tensors[a["b"]], tensors[a["y"]]
        _lib.call("ntl_layernorm_f32", _ptr(x), _ptr(w), _ptr(b), _ptr(y), int(x.shape[0]), int(x.shape[1]),
                  float(p["eps"]), float(p["inv_n"]), stream)
    elif f == "transpose":
        src, dst = tensors[a["a"]], tensors[a["b"]]
        _lib.call("ntl_transpose_f32", _ptr(src), _ptr(dst), int(src.shape[0]), int(src.shape[1]), stream)
    elif f == "gemm":
        A, B, C = tensors[a["a"]], tensors[a["b"]], tensors[a["c"]]
        bias = tensors[a["bias"]] if "bias" in a else None
        M, K = int(A.shape[0]), int(A.shape[1])
        N = int(B.shape[0]) if p["transpose_b"] else int(B.shape[1])
        # Data-parallel tiles: on B200 splitting the last wave along K (ntl_gemm_f16_f32_ws)
        # measured no faster at any shape tried; the partial-sum fixup costs about what the
        # idle part of the wave does.
        _lib.call("ntl_gemm_f16_f32", _ptr(A), _ptr(B), _ptr(C), _ptr(bias) if bias is not None else None,
                  int(p["bias_mode"]), float(p["alpha"]), int(p["relu"]), M, N, K, int(p["transpose_b"]), stream)
    elif f == "fa2":
        q, k, v, o = tensors[a["q"]], tensors[a["k"]], tensors[a["v"]], tensors[a["o"]]
        b, h, s, d = (int(x) for x in q.shape)
        _lib.call("ntl_fa2_fwd_f16", _ptr(q), _ptr(k), _ptr(v), _ptr(o), b, h, s, d, float(p["scale_log2"]),
                  int(p["causal"]), stream)
    else:  # pragma: no cover - recognize() only produces the families above
        raise RuntimeError(f"no launcher for op family {f!r}")


ABI_CALL = {
    "elementwise": "ntl_binary_f32(op, A, B, C, n, stream)",
    "cumsum": "ntl_cumsum_f32(X, Y, rows, cols, reverse, stream)",
    "softmax": "ntl_softmax_f32(X, Y, rows, cols, stream)",
    "rmsnorm": "ntl_rmsnorm_f32(X, W, Y, rows, cols, eps, inv_n, stream)",
    "layernorm": "ntl_layernorm_f32(X, W, B, Y, rows, cols, eps, inv_n, stream)",
    "transpose": "ntl_transpose_f32(A, B, m, n, stream)",
    "gemm": "ntl_gemm_f16_f32(A, B, C, bias, bias_mode, alpha, relu, M, N, K, b_trans, stream)",
    "fa2": "ntl_fa2_fwd_f16(Q, K, V, O, batch, heads, seq, dim, scale_log2, causal, stream)",
}


def describe(spec: OpSpec, name: str, target: str) -> str:
    """The text ``CompiledKernel.source`` returns: what will be launched and how."""
    lines = [
        f"# ntilang_b200 launch plan for kernel `{name}` (target {target})",
        f"# op family : {spec.family}",
        f"# parameters: {', '.join(f'{k}={v}' for k, v in spec.params.items())}",
        f"# arguments : {', '.join(f'{k}=arg{v}' for k, v in spec.args.items())}",
        f"# C ABI     : {ABI_CALL[spec.family]}  (libntl_kernels.so, include/ntl_kernels.h)",
    ]
    return "\n".join(lines) + "\n"

"""CPU oracle for the ntilang_b200 hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py``
may import this module, and only as the checker / the timed CPU baseline.  The product
path (``ntilang_b200``) never calls it: a missing CUDA library is an error there.

Each function restates, in NumPy, the arithmetic the reference's generated kernel
performs, in the reference's operation order where the order changes the result:

* ``vadd``            examples/vector_add.py:5-10 (one fp32 add per element)
* ``cumsum_rows``     python/ntilang/scan.py:349-389 (``evaluate``: 32-column Hillis-Steele
                      segments, sequential carry from +0) == the device order of scan.py:132-240
* ``cummax_rows``     the same DAG with fmax and identity -inf (scan.py:26-29, :366-374)
* ``softmax_rows``    examples/softmax.py:9-25 with the reduction tree of codegen.py:1094-1151
* ``rmsnorm_rows``    examples/rmsnorm.py:13-37 with the same tree
* ``gemm``            python/ntilang/testing.py:356-360 (fp32 product of upcast fp16), with the
                      epilogue of examples/matmul_relu.py:35-38
* ``fa2_blockwise``   examples/flash_attention.py:26-79, block by block (online base-2 softmax,
                      P rounded to fp16 before P V)

Parity pins: ``tests/golden/`` holds outputs of the reference's own NumPy evaluator
(``ntilang.testing.reference`` / ``scan.evaluate``) on seeded inputs, generated in a container
where the reference is importable by ``tests/golden/make_golden.py``;
``tests/test_oracle_golden.py`` checks these functions against them.
"""

from __future__ import annotations

import numpy as np

# ------------------------------------------------------------------------- elementwise


def vadd(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    return (a.astype(np.float32) + b.astype(np.float32)).astype(np.float32)


def binary(op: str, a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = a.astype(np.float32)
    b = b.astype(np.float32)
    return {"+": np.add, "-": np.subtract, "*": np.multiply}[op](a, b).astype(np.float32)


# ------------------------------------------------------------------------------ cumsum


def cumsum_rows(x: np.ndarray, reverse: bool = False) -> np.ndarray:
    """Inclusive scan along the last axis in the reference's segment order (scan.py:349-389)."""
    x = np.asarray(x, dtype=np.float32)
    shape = x.shape
    rows = x.reshape(-1, shape[-1]) if x.ndim > 1 else x.reshape(1, -1)
    n = rows.shape[1]
    padded = (n + 31) // 32 * 32
    work = np.zeros((rows.shape[0], padded), dtype=np.float32)
    work[:, :n] = rows
    seg = work.reshape(rows.shape[0], padded // 32, 32)
    with np.errstate(over="ignore", invalid="ignore"):
        for o in (1, 2, 4, 8, 16):
            old = seg.copy()
            if reverse:
                seg[..., :-o] = old[..., :-o] + old[..., o:]
            else:
                seg[..., o:] = old[..., o:] + old[..., :-o]
        carry = np.zeros(rows.shape[0], dtype=np.float32)
        order = range(seg.shape[1] - 1, -1, -1) if reverse else range(seg.shape[1])
        for s in order:
            seg[:, s, :] = seg[:, s, :] + carry[:, None]
            carry = seg[:, s, 0 if reverse else 31].copy()
    return work[:, :n].reshape(shape).copy()


def _fmax_pos_zero(left, right):
    """np.fmax with +0 above -0 (scan.py:366-374: fmaxf ignores NaN and prefers +0)."""
    out = np.fmax(left, right)
    zero = np.where(np.signbit(left) & np.signbit(right), np.float32(-0.0), np.float32(0.0))
    return np.where((left == 0) & (right == 0), zero, out).astype(np.float32)


def cummax_rows(x: np.ndarray, reverse: bool = False) -> np.ndarray:
    """Inclusive prefix maximum along the last axis in the reference's segment order
    (scan.py:349-389 with kind "max": identity -inf, combine fmax)."""
    x = np.asarray(x, dtype=np.float32)
    shape = x.shape
    rows = x.reshape(-1, shape[-1]) if x.ndim > 1 else x.reshape(1, -1)
    n = rows.shape[1]
    padded = (n + 31) // 32 * 32
    work = np.full((rows.shape[0], padded), -np.inf, dtype=np.float32)
    work[:, :n] = rows
    seg = work.reshape(rows.shape[0], padded // 32, 32)
    with np.errstate(invalid="ignore"):
        for o in (1, 2, 4, 8, 16):
            old = seg.copy()
            if reverse:
                seg[..., :-o] = _fmax_pos_zero(old[..., :-o], old[..., o:])
            else:
                seg[..., o:] = _fmax_pos_zero(old[..., o:], old[..., :-o])
        carry = np.full(rows.shape[0], -np.inf, dtype=np.float32)
        order = range(seg.shape[1] - 1, -1, -1) if reverse else range(seg.shape[1])
        for s in order:
            seg[:, s, :] = _fmax_pos_zero(seg[:, s, :], carry[:, None])
            carry = seg[:, s, 0 if reverse else 31].copy()
    return work[:, :n].reshape(shape).copy()


# ---------------------------------------------------------------------- row reductions


def _next_pow2(n: int) -> int:
    return 1 if n <= 1 else 1 << (n - 1).bit_length()


def tree_sum_rows(v: np.ndarray, pad_to: int | None = None) -> np.ndarray:
    """Perfect binary tree sum over the last axis (codegen.py:1094-1151), padded with +0."""
    v = np.asarray(v, dtype=np.float32)
    p = _next_pow2(v.shape[-1]) if pad_to is None else pad_to
    work = np.zeros(v.shape[:-1] + (p,), dtype=np.float32)
    work[..., : v.shape[-1]] = v
    with np.errstate(over="ignore", invalid="ignore"):
        while work.shape[-1] > 1:
            work = work[..., 0::2] + work[..., 1::2]
    return work[..., 0]


def softmax_rows(x: np.ndarray) -> np.ndarray:
    """exp(x - max) / sum over the last axis; sum in the reference's tree order."""
    x = np.asarray(x, dtype=np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        m = np.fmax.reduce(x, axis=-1, initial=-np.inf).astype(np.float32)
        e = np.exp((x - m[..., None]).astype(np.float32)).astype(np.float32)
        s = tree_sum_rows(e)
        return (e / s[..., None]).astype(np.float32)


def rmsnorm_rows(x: np.ndarray, w: np.ndarray, eps: float, inv_n: float | None = None) -> np.ndarray:
    """(x * rsqrt(sum(x^2) * inv_n + eps)) * w with the sum in the reference's tree order."""
    x = np.asarray(x, dtype=np.float32)
    w = np.asarray(w, dtype=np.float32)
    n = x.shape[-1]
    inv_n = np.float32(1.0 / n if inv_n is None else inv_n)
    ss = tree_sum_rows((x * x).astype(np.float32))
    t = (ss * inv_n).astype(np.float32) + np.float32(eps)
    inv = (np.float32(1.0) / np.sqrt(t.astype(np.float64))).astype(np.float32)
    return ((x * inv[..., None]).astype(np.float32) * w).astype(np.float32)


def layernorm_rows(x: np.ndarray, w: np.ndarray, b: np.ndarray, eps: float,
                   inv_n: float | None = None) -> np.ndarray:
    """examples/layernorm.py:18-43 in the reference's order, every step rounded to float32:
    mean = tree_sum(x) * inv_n; d = x - mean; rstd = 1 / sqrt(tree_sum(d * d) * inv_n + eps)
    (the evaluator's rsqrt, testing.py:98); y = ((d * rstd) * w) + b."""
    x = np.asarray(x, dtype=np.float32)
    w = np.asarray(w, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    n = x.shape[-1]
    inv_n = np.float32(1.0 / n if inv_n is None else inv_n)
    mean = (tree_sum_rows(x) * inv_n).astype(np.float32)
    d = (x - mean[..., None]).astype(np.float32)
    var = (tree_sum_rows((d * d).astype(np.float32)) * inv_n).astype(np.float32)
    rstd = (np.float32(1.0) / np.sqrt((var + np.float32(eps)).astype(np.float32))).astype(np.float32)
    return ((((d * rstd[..., None]).astype(np.float32)) * w).astype(np.float32) + b).astype(np.float32)


def transpose(a: np.ndarray) -> np.ndarray:
    """examples/transpose.py:5-15: B = A^T (an exact copy)."""
    return np.ascontiguousarray(np.asarray(a).T)


# -------------------------------------------------------------------------------- GEMM

BIAS_NONE, BIAS_N, BIAS_MN, BIAS_M = 0, 1, 2, 3


def gemm(a, b, bias=None, bias_mode=BIAS_NONE, alpha=1.0, relu=False, b_trans=False, accumulate=np.float64):
    """C = [relu](alpha * (A @ B) [+ bias]) from fp16 operands; accumulation in ``accumulate``."""
    a = np.asarray(a).astype(accumulate)
    b = np.asarray(b).astype(accumulate)
    c = a @ (b.T if b_trans else b)
    c = c.astype(np.float32)
    if alpha != 1.0:
        c = (c * np.float32(alpha)).astype(np.float32)
    if bias_mode == BIAS_N:
        c = c + np.asarray(bias, np.float32)[None, :]
    elif bias_mode == BIAS_MN:
        c = c + np.asarray(bias, np.float32)
    elif bias_mode == BIAS_M:
        c = c + np.asarray(bias, np.float32)[:, None]
    if relu:
        c = np.maximum(c, np.float32(0))
    return c.astype(np.float32)


# --------------------------------------------------------------------------------- FA2


def fa2_blockwise(q, k, v, scale_log2, causal=False, block_m=64, block_n=64):
    """FlashAttention-2 forward as examples/flash_attention.py:26-79 computes it.

    Per query block: running max m (starts -inf), running sum l, accumulator o.  For each key
    block: s = q k^T (fp32); causal keys beyond the query get -1e30; m_new = max(m, rowmax(s));
    r = exp2(m*c - m_new*c); o *= r; p = exp2(s*c - m_new*c); l = l*r + rowsum(p);
    o += fp16(p) @ v.  Finally o / l, rounded to fp16.
    """
    q = np.asarray(q, np.float16)
    k = np.asarray(k, np.float16)
    v = np.asarray(v, np.float16)
    B, H, S, D = q.shape
    out = np.empty_like(q)
    c = np.float32(scale_log2)
    for b in range(B):
        for h in range(H):
            qf = q[b, h].astype(np.float32)
            kf = k[b, h].astype(np.float32)
            vf = v[b, h].astype(np.float32)
            for q0 in range(0, S, block_m):
                qb = qf[q0 : q0 + block_m]
                rows = qb.shape[0]
                m = np.full(rows, -np.inf, np.float32)
                l = np.zeros(rows, np.float32)
                o = np.zeros((rows, D), np.float32)
                kv_end = min(S, q0 + block_m) if causal else S
                for k0 in range(0, kv_end, block_n):
                    s = (qb @ kf[k0 : k0 + block_n].T).astype(np.float32)
                    if causal:
                        qi = np.arange(q0, q0 + rows)[:, None]
                        kj = np.arange(k0, k0 + s.shape[1])[None, :]
                        s = np.where(qi >= kj, s, np.float32(-1e30))
                    m_new = np.maximum(m, s.max(axis=1))
                    r = np.exp2(m * c - m_new * c).astype(np.float32)
                    o *= r[:, None]
                    p = np.exp2(s * c - m_new[:, None] * c).astype(np.float32)
                    l = l * r + p.sum(axis=1, dtype=np.float32)
                    o += p.astype(np.float16).astype(np.float32) @ vf[k0 : k0 + block_n]
                    m = m_new
                out[b, h, q0 : q0 + rows] = (o / l[:, None]).astype(np.float16)
    return out


def attention_reference(q, k, v, causal=False, scale=None):
    """Plain softmax(QK^T * scale) V in float64 (the SDPA definition), rounded to fp16."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    D = q.shape[-1]
    scale = 1.0 / np.sqrt(D) if scale is None else scale
    s = np.einsum("bhqd,bhkd->bhqk", q, k) * scale
    if causal:
        S = q.shape[2]
        mask = np.tril(np.ones((S, k.shape[2]), dtype=bool))
        s = np.where(mask, s, -np.inf)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("bhqk,bhkd->bhqd", p, v).astype(np.float16)


__all__ = [
    "BIAS_M", "BIAS_MN", "BIAS_N", "BIAS_NONE", "attention_reference", "binary", "cumsum_rows",
    "fa2_blockwise", "gemm", "rmsnorm_rows", "softmax_rows", "tree_sum_rows", "vadd",
]

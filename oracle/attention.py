"""Flash-attention oracle — TEST INFRASTRUCTURE (see ``oracle/__init__.py``; parity
unpinned: the reference tree holds no attention kernel, only the vocabulary its flash
kernel is written in).

The definition: O = softmax(scale·Q·Kᵀ + mask)·V per (batch, query head), from inputs
already rounded to fp16/bf16; query head h reads KV head h // (Hq // Hkv); causal mask
keeps key j for query i when j <= i + (Skv - Sq) (bottom-right aligned, which is the
top-left mask when Sq == Skv). Rows with no visible key produce 0 (and lse = -inf).

``attention_ref`` evaluates the definition in float64 per (b, h) — small cases.
``attention_blockwise`` is the online-softmax form the flash kernel uses (row max and row
sum carried across key blocks: coopmat_reduce(max, Row) / coopmat_perelement(exp) /
coopmat_reduce(+, Row) in src/device/coopmat_intrinsics.jl:551-593,702-730), in float32
with BLAS — fast enough for the benchmark shapes on a sample of (b, h) units and the CPU
baseline.
"""
from __future__ import annotations

import numpy as np


def _mask(sq: int, skv: int) -> np.ndarray:
    i = np.arange(sq)[:, None]
    j = np.arange(skv)[None, :]
    return j <= i + (skv - sq)


def attention_ref(Q, K, V, causal: bool, scale: float, return_lse: bool = False):
    """float64 definition. Q [B,Hq,Sq,D], K/V [B,Hkv,Skv,D] (float arrays of values)."""
    Bq, Hq, Sq, D = Q.shape
    _, Hkv, Skv, _ = K.shape
    g = Hq // Hkv
    O = np.zeros((Bq, Hq, Sq, D), dtype=np.float64)
    L = np.full((Bq, Hq, Sq), -np.inf)
    m = _mask(Sq, Skv) if causal else np.ones((Sq, Skv), dtype=bool)
    for b in range(Bq):
        for h in range(Hq):
            q = Q[b, h].astype(np.float64)
            k = K[b, h // g].astype(np.float64)
            v = V[b, h // g].astype(np.float64)
            s = scale * (q @ k.T)
            s = np.where(m, s, -np.inf)
            mx = s.max(axis=1, keepdims=True)
            ok = np.isfinite(mx[:, 0])
            mx = np.where(np.isfinite(mx), mx, 0.0)
            p = np.exp(s - mx)
            l = p.sum(axis=1, keepdims=True)
            O[b, h] = np.where(ok[:, None], (p @ v) / np.where(l > 0, l, 1.0), 0.0)
            L[b, h] = np.where(ok, mx[:, 0] + np.log(np.where(l[:, 0] > 0, l[:, 0], 1.0)), -np.inf)
    return (O, L) if return_lse else O


def attention_rows(q, k, v, rows, causal: bool, scale: float, sq: int | None = None):
    """The float64 definition for the query rows ``rows`` of one (b, h) unit only:
    q [Sq,D] (or just the selected rows with ``sq`` the unit's full Sq), k/v [Skv,D].
    Returns (O [len(rows),D], lse [len(rows)]). Each row reads only the keys it may see, so
    checking a few hundred rows of a 16k-key head costs a few hundred key rows' products."""
    rows = np.asarray(rows)
    Skv = k.shape[0]
    Sq = q.shape[0] if sq is None else sq
    qs = (q if sq is not None else q[rows]).astype(np.float64)
    last = int(rows.max()) + (Skv - Sq) if causal else Skv - 1
    kk = k[:max(0, min(Skv, last + 1))].astype(np.float64)
    vv = v[:kk.shape[0]].astype(np.float64)
    s = scale * (qs @ kk.T)
    if causal:
        j = np.arange(kk.shape[0])[None, :]
        s = np.where(j <= rows[:, None] + (Skv - Sq), s, -np.inf)
    mx = s.max(axis=1, keepdims=True) if s.shape[1] else np.full((len(rows), 1), -np.inf)
    ok = np.isfinite(mx[:, 0])
    mx = np.where(np.isfinite(mx), mx, 0.0)
    p = np.exp(s - mx)
    l = p.sum(axis=1)
    O = np.where(ok[:, None], (p @ vv) / np.where(l > 0, l, 1.0)[:, None], 0.0)
    lse = np.where(ok, mx[:, 0] + np.log(np.where(l > 0, l, 1.0)), -np.inf)
    return O, lse


def attention_blockwise(q, k, v, causal: bool, scale: float, block: int = 128):
    """One (b, h) unit in float32, online softmax over key blocks. q [Sq,D], k/v [Skv,D].
    Returns (O [Sq,D] float32, lse [Sq] float32)."""
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    Sq, D = q.shape
    Skv = k.shape[0]
    off = Skv - Sq
    m = np.full((Sq,), -np.inf, dtype=np.float32)
    l = np.zeros((Sq,), dtype=np.float32)
    acc = np.zeros((Sq, D), dtype=np.float32)
    rows = np.arange(Sq)[:, None]
    for j0 in range(0, Skv, block):
        j1 = min(Skv, j0 + block)
        if causal and j0 > (Sq - 1) + off:
            break
        s = (q @ k[j0:j1].T) * np.float32(scale)
        if causal:
            cols = np.arange(j0, j1)[None, :]
            s = np.where(cols <= rows + off, s, -np.inf).astype(np.float32)
        m_new = np.maximum(m, s.max(axis=1))
        safe = np.where(np.isfinite(m_new), m_new, 0.0).astype(np.float32)
        p = np.exp(s - safe[:, None])
        corr = np.exp(np.where(np.isfinite(m), m - safe, -np.inf)).astype(np.float32)
        l = l * corr + p.sum(axis=1)
        acc = acc * corr[:, None] + p @ v[j0:j1]
        m = m_new
    ok = l > 0
    O = np.where(ok[:, None], acc / np.where(ok, l, 1.0)[:, None], 0.0).astype(np.float32)
    lse = np.where(ok, m + np.log(np.where(ok, l, 1.0)), -np.inf).astype(np.float32)
    return O, lse


def attention_flops(B: int, Hq: int, Sq: int, Skv: int, D: int, causal: bool) -> float:
    """Algorithmic FLOPs: 4·B·Hq·Sq·Skv·D, halved for causal (FlashAttention convention)."""
    f = 4.0 * B * Hq * Sq * Skv * D
    return f / 2 if causal else f

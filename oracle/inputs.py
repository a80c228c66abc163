"""Seeded synthetic inputs of the benchmark configurations — TEST INFRASTRUCTURE.

Generator: ``numpy.random.Generator(PCG64(seed))`` (Julia's RNG stream cannot be
reproduced without Julia; parity is always checked on identical input bytes). Draw order is
fixed: A first, then B, each in its STORAGE order — A (M,K) row-major, B (K,N) column-major
drawn as its (N,K) storage array — so the same seed gives the same bytes everywhere.

Configs (the reference's benchmark list):
  C1  fp16 GEMM 512³, fp32 C, U[-1,1) seed 0
  C2  fp16 GEMM 8192³, fp16 C, U[-1,1) seed 1
  C3  int8 GEMM 8192³, int32 C, U{-128..127} seed 2
  C4  attention fp16 B4 H32 S4096 D128 causal, N(0,1) seed 3
  C5  attention bf16 B8 Hq64 Hkv8 S16384 D128 causal, N(0,1) seed 4;
      bf16 GEMM M65536 N=K=8192, U[-1,1) seed 5
"""
from __future__ import annotations

import numpy as np

from .vocab import round_bf16

GEMM_CONFIGS = {
    "C1": dict(M=512, N=512, K=512, ab="Float16", out="Float32", seed=0),
    "C2": dict(M=8192, N=8192, K=8192, ab="Float16", out="Float16", seed=1),
    "C3": dict(M=8192, N=8192, K=8192, ab="Int8", out="Int32", seed=2),
    "C5g": dict(M=65536, N=8192, K=8192, ab="BFloat16", out="BFloat16", seed=5),
}
ATTN_CONFIGS = {
    "C4": dict(B=4, Hq=32, Hkv=32, S=4096, D=128, dtype="Float16", causal=True, seed=3),
    "C5": dict(B=8, Hq=64, Hkv=8, S=16384, D=128, dtype="BFloat16", causal=True, seed=4),
}


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def cast(x: np.ndarray, T: str) -> np.ndarray:
    """Round float values to T: float16 array for Float16, float32 array holding bf16
    values for BFloat16 (RNE)."""
    if T == "Float16":
        return x.astype(np.float32).astype(np.float16)
    if T == "BFloat16":
        return round_bf16(x.astype(np.float32))
    if T == "Float32":
        return x.astype(np.float32)
    raise ValueError(T)


def gemm_inputs(M: int, N: int, K: int, ab: str, seed: int):
    """(A (M,K), Bt (N,K)) storage arrays; B = Bt.T is the column-major K×N operand."""
    g = rng(seed)
    if ab in ("Int8", "UInt8"):
        lo, hi, dt = (-128, 128, np.int8) if ab == "Int8" else (0, 256, np.uint8)
        A = g.integers(lo, hi, size=(M, K), dtype=np.int16).astype(dt)
        Bt = g.integers(lo, hi, size=(N, K), dtype=np.int16).astype(dt)
        return A, Bt
    A = cast(g.uniform(-1.0, 1.0, size=(M, K)), ab)
    Bt = cast(g.uniform(-1.0, 1.0, size=(N, K)), ab)
    return A, Bt


def attention_inputs(B: int, Hq: int, Hkv: int, S: int, D: int, dtype: str, seed: int,
                     Skv: int | None = None):
    """Q [B,Hq,S,D], K and V [B,Hkv,Skv,D], i.i.d. N(0,1) rounded to dtype."""
    g = rng(seed)
    Skv = S if Skv is None else Skv
    Q = cast(g.standard_normal(size=(B, Hq, S, D), dtype=np.float32), dtype)
    K = cast(g.standard_normal(size=(B, Hkv, Skv, D), dtype=np.float32), dtype)
    V = cast(g.standard_normal(size=(B, Hkv, Skv, D), dtype=np.float32), dtype)
    return Q, K, V

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

from .vocab import round_bf16, f32_to_bf16_bits

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


def _operand_stored(g: np.random.Generator, rows: int, K: int, ab: str, chunk: int):
    """One operand's storage array, drawn ``chunk`` rows at a time from ``g``. A uniform
    draw takes one 64-bit output per element in order, so the chunks continue the same stream
    and the bytes equal one draw of the whole array. 16-bit floats come back as their stored
    bits: float16, or uint16 bf16 bits (half the memory of float32 values)."""
    if ab in ("Int8", "UInt8"):
        lo, hi, dt = (-128, 128, np.int8) if ab == "Int8" else (0, 256, np.uint8)
        out = np.empty((rows, K), dtype=dt)
        if (chunk * K) % 2:
            chunk = rows   # 16-bit integer draws share 32-bit outputs: keep chunks even
        for r in range(0, rows, chunk):
            n = min(chunk, rows - r)
            out[r:r + n] = g.integers(lo, hi, size=(n, K), dtype=np.int16).astype(dt)
        return out
    out = np.empty((rows, K), dtype=np.float16 if ab == "Float16" else np.uint16)
    for r in range(0, rows, chunk):
        n = min(chunk, rows - r)
        x = g.uniform(-1.0, 1.0, size=(n, K)).astype(np.float32)
        out[r:r + n] = x.astype(np.float16) if ab == "Float16" else f32_to_bf16_bits(x)
    return out


def gemm_inputs_stored(M: int, N: int, K: int, ab: str, seed: int, chunk: int = 2048):
    """``gemm_inputs`` for the large configurations: the same bytes, generated in row chunks
    so the float64 draw never holds more than ``chunk`` rows; BFloat16 operands are returned
    as uint16 bit arrays (see ``vocab.bf16_bits_to_f32``)."""
    g = rng(seed)
    A = _operand_stored(g, M, K, ab, chunk)
    Bt = _operand_stored(g, N, K, ab, chunk)
    return A, Bt


def attention_inputs_stored(B: int, Hq: int, Hkv: int, S: int, D: int, dtype: str, seed: int,
                            Skv: int | None = None):
    """``attention_inputs`` for the large configurations: the same values, drawn one batch
    index at a time (sequential normal draws continue the same stream), returned as the
    stored 16-bit patterns (float16, or uint16 bf16 bits)."""
    g = rng(seed)
    Skv = S if Skv is None else Skv

    def draw(H, L):
        out = np.empty((B, H, L, D), dtype=np.float16 if dtype == "Float16" else np.uint16)
        for b in range(B):
            x = g.standard_normal(size=(H, L, D), dtype=np.float32)
            out[b] = x.astype(np.float16) if dtype == "Float16" else f32_to_bf16_bits(x)
        return out
    Q = draw(Hq, S)
    K = draw(Hkv, Skv)
    V = draw(Hkv, Skv)
    return Q, K, V

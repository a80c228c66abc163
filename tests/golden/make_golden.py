"""Generate the small golden fixtures in tests/golden/ from the oracle.

    python tests/golden/make_golden.py

Each fixture stores its seeded inputs and the oracle's output (float64 accumulation rounded
once to the output type; int64 accumulation for integers). The GPU tests compare the
kernels against these bytes, and the CPU tests check the oracle still reproduces them, so a
change to either side shows up as a fixture mismatch. The reference (Lava.jl) cannot run
here and ships no numeric goldens for this path; these fixtures pin regressions, not the
reference itself.
"""
from pathlib import Path
import sys

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle import vocab  # noqa: E402
from oracle.gemm import gemm_ref  # noqa: E402
from oracle.attention import attention_ref  # noqa: E402
from oracle.inputs import gemm_inputs, attention_inputs  # noqa: E402

GEMMS = [
    # name, M, N, K, ab, out, seed
    ("gemm_f16_f32_ragged", 37, 29, 70, "Float16", "Float32", 101),
    ("gemm_f16_f16_ragged", 130, 66, 136, "Float16", "Float16", 102),
    ("gemm_bf16_bf16", 64, 48, 128, "BFloat16", "BFloat16", 103),
    ("gemm_bf16_f32_kodd", 17, 40, 200, "BFloat16", "Float32", 104),
    ("gemm_i8_i32", 70, 33, 160, "Int8", "Int32", 105),
    ("gemm_u8_u32", 20, 130, 96, "UInt8", "UInt32", 106),
    # matrix-vector products (N = 1 / M = 1): the streaming kernel, dot4x8 for 8-bit
    ("gemm_gemv_i8_i32", 300, 1, 1000, "Int8", "Int32", 108),
    ("gemm_vecmat_f16_f32", 1, 200, 300, "Float16", "Float32", 109),
]


def main():
    for name, M, N, K, ab, out, seed in GEMMS:
        A, Bt = gemm_inputs(M, N, K, ab, seed)
        B = np.ascontiguousarray(Bt.T)
        C = gemm_ref(A, B, out)
        if ab == "BFloat16":
            A, B = vocab.f32_to_bf16_bits(A), vocab.f32_to_bf16_bits(B)
        if out == "BFloat16":
            C = vocab.f32_to_bf16_bits(C)
        np.savez_compressed(HERE / f"{name}.npz", kind="gemm", ab=ab, out=out, A=A, B=B, C=C)
    Q, K, V = attention_inputs(1, 4, 2, 64, 64, "Float16", seed=107, Skv=112)
    O64 = attention_ref(Q.astype(np.float32), K.astype(np.float32), V.astype(np.float32),
                        True, 0.125)
    np.savez_compressed(HERE / "attn_f16_gqa_causal.npz", kind="attention", Q=Q, K=K, V=V,
                        causal=True, scale=0.125, O=O64.astype(np.float32))
    # decoding: one query per sequence, a GQA group of 8 against a 700-key cache
    Q, K, V = attention_inputs(2, 8, 1, 1, 128, "BFloat16", seed=110, Skv=700)
    O64 = attention_ref(Q, K, V, True, 128 ** -0.5)
    np.savez_compressed(HERE / "attn_bf16_decode_gqa.npz", kind="attention",
                        Q=vocab.f32_to_bf16_bits(Q), K=vocab.f32_to_bf16_bits(K),
                        V=vocab.f32_to_bf16_bits(V), causal=True, scale=128 ** -0.5,
                        O=O64.astype(np.float32), dtype="BFloat16")
    print("wrote", len(GEMMS) + 2, "fixtures")


if __name__ == "__main__":
    main()

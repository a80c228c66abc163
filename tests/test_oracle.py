"""CPU tier: pin the oracle against the reference's executable definitions (worked by hand)
and against exact arithmetic; check the committed golden fixtures."""
from fractions import Fraction
from pathlib import Path

import numpy as np
import pytest

from oracle import vocab
from oracle.gemm import gemm_ref, gemm_tiled, rel_frobenius, ulp_distance_f16
from oracle.attention import attention_ref, attention_blockwise
from oracle.inputs import gemm_inputs, attention_inputs, cast

GOLDEN = Path(__file__).parent / "golden"


# ---- known answers from the reference's own definitions ---------------------------------
def test_dot4x8_known_answers():
    # src/vocabulary/vocabulary.jl:31-35 — bytes are Int8, byte i pairs with byte i.
    assert vocab.dot4x8(0x04030201, 0x08070605) == 1 * 5 + 2 * 6 + 3 * 7 + 4 * 8  # 70
    assert vocab.dot4x8(0x000000FF, 0x00000001) == -1            # 0xFF is -1, not 255
    assert vocab.dot4x8(0x80808080, 0x80808080) == 4 * 128 * 128  # (-128)^2 * 4 = 65536
    assert vocab.dot4x8(0x7F7F7F7F, 0x80808080) == 4 * 127 * -128
    assert vocab.dot4x8(0, 0xFFFFFFFF) == 0


def test_int8_matvec_is_dot4x8():
    """An int8 matrix-vector product as Lava's dot4x8 computes it — bytes packed four to a
    word, row by row, each word pair summed exactly into Int32 (src/vocabulary/vocabulary.jl:
    18-35) — equals the exact int64 GEMM oracle the GPU tests compare the kernel with."""
    from oracle.inputs import gemm_inputs
    A, Bt = gemm_inputs(37, 1, 96, "Int8", seed=5)
    x = Bt[0]
    words = lambda v: [int.from_bytes(v[i:i + 4].tobytes(), "little") for i in range(0, len(v), 4)]
    xw = words(x)
    y = [sum(vocab.dot4x8(a, b) for a, b in zip(words(row), xw)) for row in A]
    assert np.array_equal(np.array(y, dtype=np.int64), gemm_ref(A, Bt.T, "Int32")[:, 0])


def test_clamp_modes_and_reduce_masks():
    # src/vocabulary/tensor.jl:46-51, src/vocabulary/coopmat.jl:292-297
    assert (vocab.TENSOR_CLAMP_UNDEFINED, vocab.TENSOR_CLAMP_CONSTANT,
            vocab.TENSOR_CLAMP_TO_EDGE) == (0, 1, 2)
    assert (vocab.REDUCE_ROW, vocab.REDUCE_COLUMN, vocab.REDUCE_ROW_AND_COLUMN) == (1, 2, 3)


def test_tensor_clampbits():
    # src/vocabulary/tensor.jl:83-85: 1.0 in Float16 is 0x3C00, in Float32 0x3F800000.
    assert vocab.tensor_clampbits(1.0, "Float16") == 0x3C00
    assert vocab.tensor_clampbits(1.0, "Float32") == 0x3F800000
    assert vocab.tensor_clampbits(-2.0, "Float16") == 0xC000
    assert vocab.tensor_clampbits(7, "Int32") == 7


def test_coopmat_load_store_addressing():
    mem = np.arange(1, 101, dtype=np.float32)     # mem[i] = i+1
    # column-major 3x2 tile at offset 5 (1-based), stride 10: (r,c) -> mem[4 + c*10 + r]
    t = vocab.coopmat_load(mem, 5, 10, 3, 2)
    assert t.tolist() == [[5, 15], [6, 16], [7, 17]]
    # row-major: (r,c) -> mem[4 + r*10 + c]
    t = vocab.coopmat_load(mem, 5, 10, 3, 2, rowmajor=True)
    assert t.tolist() == [[5, 6], [15, 16], [25, 26]]
    out = np.zeros(100, dtype=np.float32)
    vocab.coopmat_store(out, 5, 10, t, rowmajor=True)
    assert vocab.coopmat_load(out, 5, 10, 3, 2, rowmajor=True).tolist() == t.tolist()


def test_reduce_smears_and_perelement_is_zero_based():
    m = np.array([[1.0, 5.0, 2.0], [-1.0, -3.0, 0.5]], dtype=np.float32)
    r = vocab.coopmat_reduce(max, m, vocab.REDUCE_ROW)
    assert r.tolist() == [[5, 5, 5], [0.5, 0.5, 0.5]]         # smeared, not a vector
    c = vocab.coopmat_reduce(lambda a, b: a + b, m, vocab.REDUCE_COLUMN)
    assert c.tolist() == [[0, 2, 2.5], [0, 2, 2.5]]
    idx = vocab.coopmat_perelement(lambda r, c, e: np.float32(10 * int(r) + int(c)), m)
    assert idx.tolist() == [[0, 1, 2], [10, 11, 12]]


def test_int8_signedness():
    # Int8 operands are signed, UInt8 unsigned (test/spirv/test_coopmat_int8.jl:56-68,94-97)
    a = np.array([[0xFF]], dtype=np.uint8)
    assert gemm_ref(a.view(np.int8), a.view(np.int8), "Int32")[0, 0] == 1      # (-1)(-1)
    assert gemm_ref(a, a, "UInt32")[0, 0] == 255 * 255


def test_bf16_rne():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, 1.0 + 2 ** -9, -3.14159],
                 dtype=np.float32)
    # ties go to even: 1+2^-8 is halfway between 1 and 1+2^-7 -> 1 ; 1+3·2^-8 -> 1+2^-6
    assert vocab.round_bf16(x).tolist()[:4] == [1.0, 1.0, 1.0 + 2 ** -6, 1.0]
    assert vocab.f32_to_bf16_bits(np.array([1.0], np.float32))[0] == 0x3F80


# ---- exactness of the float64 restatement ----------------------------------------------
def _exact_product(A, Bm):
    M, K = A.shape
    N = Bm.shape[1]
    out = np.empty((M, N), dtype=object)
    for i in range(M):
        for j in range(N):
            out[i, j] = sum(Fraction(float(A[i, k])) * Fraction(float(Bm[k, j])) for k in range(K))
    return out


@pytest.mark.parametrize("ab", ["Float16", "BFloat16"])
def test_gemm_ref_matches_exact_rationals(ab):
    A, Bt = gemm_inputs(7, 5, 33, ab, seed=11)
    B = Bt.T
    exact = _exact_product(A.astype(np.float64), B.astype(np.float64))
    got = gemm_ref(A, B, "Float32")
    ref = np.array([[np.float32(float(v)) for v in row] for row in exact], dtype=np.float32)
    assert np.array_equal(got, ref)  # one rounding of the exact sum


def test_gemm_ref_int8_exact():
    A, Bt = gemm_inputs(9, 6, 200, "Int8", seed=12)
    B = Bt.T
    ex = np.array([[sum(int(A[i, k]) * int(B[k, j]) for k in range(200)) for j in range(6)]
                   for i in range(9)], dtype=np.int64)
    assert np.array_equal(gemm_ref(A, B, "Int32").astype(np.int64), ex)


def test_gemm_tiled_algorithm_agrees_with_ref():
    # Quarter-integer inputs make every fp32 partial sum exact, so the workgroup-tile
    # algorithm (coopmat2_gemm_regs.comp) and the one-shot product agree bit for bit,
    # including ragged tiles filled by the constant clamp.
    g = np.random.default_rng(3)
    A = (g.integers(-4, 5, size=(150, 70)) / 4).astype(np.float16)
    B = (g.integers(-4, 5, size=(70, 130)) / 4).astype(np.float16)
    for out in ("Float32", "Float16"):
        assert np.array_equal(gemm_tiled(A, B, out), gemm_ref(A, B, out))
    Ai = g.integers(-128, 128, size=(140, 90)).astype(np.int8)
    Bi = g.integers(-128, 128, size=(90, 131)).astype(np.int8)
    assert np.array_equal(gemm_tiled(Ai, Bi, "Int32"), gemm_ref(Ai, Bi, "Int32"))


def test_attention_blockwise_matches_definition():
    Q, K, V = attention_inputs(1, 4, 2, 200, 64, "Float16", seed=5, Skv=333)
    O, L = attention_ref(Q, K, V, causal=True, scale=0.125, return_lse=True)
    for h in range(4):
        ob, lb = attention_blockwise(Q[0, h], K[0, h // 2], V[0, h // 2], True, 0.125, block=64)
        assert np.abs(ob - O[0, h]).max() < 2e-5
        assert np.abs(lb - L[0, h]).max() < 2e-5
    # non-causal too
    O2 = attention_ref(Q, K, V, causal=False, scale=0.125)
    ob, _ = attention_blockwise(Q[0, 1], K[0, 0], V[0, 0], False, 0.125, block=100)
    assert np.abs(ob - O2[0, 1]).max() < 2e-5


def test_causal_mask_alignment_and_empty_rows():
    # Sq > Skv: the first Sq-Skv query rows see no key (bottom-right alignment) -> O = 0.
    Q, K, V = attention_inputs(1, 1, 1, 8, 64, "Float16", seed=1, Skv=5)
    O, L = attention_ref(Q, K, V, causal=True, scale=0.1, return_lse=True)
    assert np.all(O[0, 0, :3] == 0) and np.all(np.isneginf(L[0, 0, :3]))
    # query row 3 sees exactly key 0 -> O = V[0]
    assert np.allclose(O[0, 0, 3], V[0, 0, 0])


def test_inputs_are_deterministic():
    a1, b1 = gemm_inputs(64, 32, 16, "Float16", seed=1)
    a2, b2 = gemm_inputs(64, 32, 16, "Float16", seed=1)
    assert a1.tobytes() == a2.tobytes() and b1.tobytes() == b2.tobytes()
    assert a1.dtype == np.float16 and np.all(np.abs(a1) <= 1)


# ---- golden fixtures ---------------------------------------------------------------------
def test_golden_fixtures_reproduce():
    files = sorted(GOLDEN.glob("*.npz"))
    assert files, "tests/golden has no fixtures; run tests/golden/make_golden.py"
    for f in files:
        z = np.load(f)
        kind = str(z["kind"])
        if kind == "gemm":
            out = str(z["out"])
            A, B = z["A"], z["B"]
            if str(z["ab"]) == "BFloat16":
                A, B = vocab.bf16_bits_to_f32(A), vocab.bf16_bits_to_f32(B)
            got = gemm_ref(A, B, out)
            C = z["C"]
            if out == "BFloat16":
                got = vocab.f32_to_bf16_bits(got)
            assert np.array_equal(got, C), f.name
        elif kind == "attention":
            Q, K, V = z["Q"], z["K"], z["V"]
            if "dtype" in z.files and str(z["dtype"]) == "BFloat16":
                Q, K, V = (vocab.bf16_bits_to_f32(x) for x in (Q, K, V))
            O = attention_ref(Q.astype(np.float32), K.astype(np.float32),
                              V.astype(np.float32), bool(z["causal"]), float(z["scale"]))
            assert np.abs(O - z["O"]).max() < 1e-6, f.name


def test_epilogue_init_is_stride0_bias_plus_residual():
    """The fused GEMM's initial accumulator: bias read at stride 0 (per row = column-major
    load, per column = row-major load) coopmat_add-ed to the residual, in Float32."""
    from oracle.gemm import epilogue_init
    b_row = np.array([1, 2, 3], dtype=np.float32)
    b_col = np.array([10, 20], dtype=np.float32)
    res = np.arange(6, dtype=np.float32).reshape(3, 2)
    assert np.array_equal(epilogue_init(3, 2, b_row, "row"), [[1, 1], [2, 2], [3, 3]])
    assert np.array_equal(epilogue_init(3, 2, b_col, "col"), [[10, 20]] * 3)
    got = epilogue_init(3, 2, b_col, "col", res)
    assert got.dtype == np.float32 and np.array_equal(got, res + b_col)
    # Float32 addition: 2^24 + 1 rounds to 2^24, as the accumulator type does
    big = epilogue_init(1, 1, np.array([2.0 ** 24], np.float32), "col", np.ones((1, 1), np.float32))
    assert big[0, 0] == 2.0 ** 24


def test_activation_known_values():
    from oracle.gemm import ACTIVATIONS
    x = np.array([-3.0, -1.0, 0.0, 1.0, 2.0])
    assert np.array_equal(ACTIVATIONS["relu"](x), [0, 0, 0, 1, 2])
    assert np.isnan(ACTIVATIONS["relu"](np.array([np.nan])))[0]       # NaN passes
    # gelu(1) = Phi(1) = 0.841344746...; tanh form 0.841191990...
    assert abs(ACTIVATIONS["gelu_erf"](np.array([1.0]))[0] - 0.8413447460685429) < 1e-15
    assert abs(ACTIVATIONS["gelu"](np.array([1.0]))[0] - 0.8411919906082768) < 1e-15
    assert abs(ACTIVATIONS["silu"](np.array([1.0]))[0] - 1.0 / (1.0 + np.exp(-1.0))) < 1e-15
    assert ACTIVATIONS["silu"](np.array([-1000.0]))[0] == 0.0            # no overflow error


def test_epilogue_ref_is_perelement_over_the_accumulator():
    """gemm_epilogue_ref equals the vocabulary spelled out: accumulator init, muladd,
    perelement(act), convert."""
    from oracle.gemm import ACTIVATIONS, epilogue_init, gemm_epilogue_ref
    rng = np.random.default_rng(0)
    A = rng.uniform(-1, 1, (16, 32)).astype(np.float16)
    B = rng.uniform(-1, 1, (32, 8)).astype(np.float16)
    bias = rng.uniform(-1, 1, 8).astype(np.float32)
    res = rng.uniform(-1, 1, (16, 8)).astype(np.float32)
    acc = epilogue_init(16, 8, bias, "col", res).astype(np.float64)
    acc = vocab.coopmat_muladd(A, B, acc)
    f = lambda r, c, e: ACTIVATIONS["gelu"](np.array([e]))[0]
    want = vocab.coopmat_convert(vocab.coopmat_perelement(f, acc), "Float16")
    got = gemm_epilogue_ref(A, B, "Float16", bias, "col", res, "gelu")
    assert np.array_equal(got, want)


def test_chunked_generators_match_the_one_shot_draw():
    """The full-size parity tests draw their inputs in chunks (``gemm_inputs_stored``,
    ``attention_inputs_stored``); the bytes must equal one draw of the whole arrays."""
    from oracle.inputs import (gemm_inputs, gemm_inputs_stored, attention_inputs,
                               attention_inputs_stored)
    from oracle.vocab import bf16_bits_to_f32
    for ab in ("Float16", "BFloat16", "Int8", "UInt8"):
        A, Bt = gemm_inputs(301, 77, 96, ab, seed=11)
        A2, B2 = gemm_inputs_stored(301, 77, 96, ab, seed=11, chunk=13)
        if ab == "BFloat16":
            A2, B2 = bf16_bits_to_f32(A2), bf16_bits_to_f32(B2)
        assert np.array_equal(A, A2) and np.array_equal(Bt, B2), ab
    for T in ("Float16", "BFloat16"):
        ref = attention_inputs(3, 4, 2, 40, 32, T, seed=4, Skv=56)
        got = attention_inputs_stored(3, 4, 2, 40, 32, T, seed=4, Skv=56)
        if T == "BFloat16":
            got = [bf16_bits_to_f32(x) for x in got]
        assert all(np.array_equal(a, b) for a, b in zip(ref, got)), T


def test_attention_rows_matches_the_full_definition():
    from oracle.attention import attention_ref, attention_rows
    from oracle.inputs import attention_inputs
    for Sq, Skv in ((300, 300), (200, 333), (400, 100)):
        Q, K, V = attention_inputs(1, 1, 1, Sq, 64, "Float16", seed=Sq, Skv=Skv)
        O, L = attention_ref(Q, K, V, True, 0.125, return_lse=True)
        rows = np.array([0, 1, Sq // 2, Sq - 1])
        o, l = attention_rows(Q[0, 0], K[0, 0], V[0, 0], rows, True, 0.125)
        assert np.allclose(o, O[0, 0][rows], atol=1e-12, rtol=0)
        fin = np.isfinite(L[0, 0][rows])
        assert np.array_equal(np.isfinite(l), fin)
        assert np.allclose(l[fin], L[0, 0][rows][fin], atol=1e-12, rtol=0)

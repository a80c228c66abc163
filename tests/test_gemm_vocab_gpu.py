"""GPU tier: the rest of the vocabulary on the GEMM's fused epilogue, through the C ABI
(lvb_gemm_ex) against the oracle (oracle/gemm.py ``gemm_vocab_ref``):

  * coopmat_mul — the accumulator multiplied element-wise by a matrix S
    (src/device/coopmat_intrinsics.jl:402-464), with and without bias/residual/activation;
  * coopmat_perelement with a caller-supplied function — a per-element program with 0-based
    row/col and the matrix-operand form (coopmat_intrinsics.jl:520-678), traced from Python
    functions (lava.jl_b200/lvb/perelement.py);
  * TENSOR_CLAMP_CONSTANT with a non-zero value and TENSOR_CLAMP_TO_EDGE on the k tail of a
    padded k extent (src/vocabulary/tensor.jl:46-51; src/device/tensor_intrinsics.jl:139-148).

Tolerances: integer pairs bit-exact. Float outputs per element: one unit in the last place of
the output type at the oracle's value, plus the fp32 accumulation bound 4·√K·2^-24·(|A||B| +
|init|) times the steps' Lipschitz bound L (stated per case), plus 2^-20 of the value for the
fp32 roundings of the epilogue steps; infinities exactly; relative Frobenius <= 1e-3 over the
finite elements. Programs with transcendental functions add an absolute 2^-18 (their fp32
functions are within a few ulp of values of order one, whose sum may cancel).
"""
import numpy as np
import pytest

from oracle import vocab
from oracle.gemm import gemm_vocab_ref, clamp_pad
from oracle.inputs import gemm_inputs

pytestmark = pytest.mark.gpu
TDT = {"Float16": "float16", "BFloat16": "bfloat16", "Float32": "float32", "Int8": "int8",
       "Int32": "int32"}


def _t(torch, T):
    return getattr(torch, TDT[T])


def dev(torch, x, T):
    t = torch.from_numpy(np.ascontiguousarray(x))
    return (t.to(torch.bfloat16) if T == "BFloat16" else t).cuda()


def out_ulp(x, out):
    ax = np.abs(np.asarray(x, dtype=np.float64))
    if out == "Float16":
        return np.spacing(np.minimum(ax, 65504).astype(np.float16)).astype(np.float64)
    if out == "BFloat16":
        return 2.0 ** (np.floor(np.log2(np.maximum(ax, 2.0 ** -126))) - 7)
    return np.spacing(ax.astype(np.float32)).astype(np.float64)


def cmat(torch, x, T, rowmajor):
    """An M×N matrix in the given layout on the device."""
    if rowmajor:
        return dev(torch, x, T)
    return dev(torch, np.ascontiguousarray(x.T), T).t()


def compare(got, ref, A64, B64, init_abs, out, L=1.0, floor=0.0):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    inf = np.isinf(ref)
    assert np.array_equal(np.isinf(got), inf) and np.array_equal(got[inf], ref[inf])
    K = A64.shape[1]
    acc = 4.0 * np.sqrt(max(K, 1)) * 2.0 ** -24 * (np.abs(A64) @ np.abs(B64) + init_abs)
    bound = out_ulp(ref, out) + L * acc + 2.0 ** -20 * np.abs(ref) + floor + 1e-30
    err = np.where(inf, 0.0, np.abs(got - ref))
    bad = err > bound
    assert not bad.any(), (f"{int(bad.sum())} elements off; worst excess "
                           f"{float((err - bound)[bad].max()):.3e}")
    fin = ~inf
    den = np.linalg.norm(ref[fin])
    if den > 0:
        assert np.linalg.norm(got[fin] - ref[fin]) / den <= 1e-3


def run(lvb, torch, A, Bt, ab, out, c_rowmajor, **kw):
    M, N = A.shape[0], Bt.shape[0]
    dA, dB = dev(torch, A, ab), dev(torch, Bt, ab).t()
    odt = _t(torch, out)
    dC = (torch.full((M, N), 7, dtype=odt, device="cuda") if c_rowmajor
          else torch.full((N, M), 7, dtype=odt, device="cuda").t())
    lvb.gemm(dC, dA, dB, **kw)
    torch.cuda.synchronize()
    assert lvb.device_status() == (0, 0, 0)
    r = dC.cpu()
    return r.float().numpy() if out == "BFloat16" else r.numpy()


# ---- coopmat_mul ----------------------------------------------------------------------------
@pytest.mark.parametrize("M,N,K", [(200, 136, 120), (300, 520, 1000), (1, 64, 256), (512, 1, 300)])
@pytest.mark.parametrize("ab,out", [("Float16", "Float32"), ("BFloat16", "BFloat16"),
                                    ("Float16", "Float16")])
@pytest.mark.parametrize("c_rowmajor", [False, True])
def test_coopmat_mul(lvb, torch_cuda, M, N, K, ab, out, c_rowmajor):
    """C = (A·B + bias + R) ⊙ S, then gelu; a matrix-vector shape (N or M = 1) runs it on
    the tensor-core kernel too."""
    torch = torch_cuda
    A, Bt = gemm_inputs(M, N, K, ab, seed=M + N + K)
    g = np.random.default_rng(M * N)
    S = vocab.round_bf16(g.uniform(-2, 2, (M, N)).astype(np.float32))
    R = g.uniform(-1, 1, (M, N)).astype(np.float16)
    bias = g.uniform(-1, 1, N).astype(np.float32)
    for act in (None, "gelu"):
        got = run(lvb, torch, A, Bt, ab, out, c_rowmajor, mul=cmat(torch, S, "BFloat16", c_rowmajor),
                  residual=cmat(torch, R, "Float16", c_rowmajor), bias=dev(torch, bias, "Float32"),
                  activation=act)
        ref = gemm_vocab_ref(A, Bt.T, out, ab, bias=bias, residual=R, mul=S, act=act)
        A64, B64 = A.astype(np.float64), Bt.T.astype(np.float64)
        compare(got, ref, A64 * 1, B64, np.abs(R) + np.abs(bias), out, L=2.0 * 1.13)


# ---- per-element programs ---------------------------------------------------------------
def _programs():
    from lvb.perelement import where, tanh, exp, maximum, minimum, fma, erf, sqrt, log
    return {
        # a causal mask with an ALiBi-style slope on the scaled product (L = 0.125)
        "causal_alibi": (lambda x, r, c, e: where(c > r, float("-inf"), 0.125 * x - 0.5 * (r - c)),
                         0.125, False),
        # the matrix-operand form: the other matrix's element and the row index
        "extra_fma": (lambda x, r, c, e: fma(x, e, r * 0.25), 1.0, True),
        # clamps and transcendental functions
        "clip_tanh_exp": (lambda x, r, c, e: maximum(minimum(x, 1.5), -1.0) + tanh(e) * exp(0.05 * x),
                          1.0, True),
        # integer arithmetic on the indices, erf and sqrt
        "index_math": (lambda x, r, c, e: where((r - c) * (r - c) < 100, erf(0.1 * x), sqrt(abs(x) + 1.0)
                                                + log(1.0 + c)), 0.5, False),
    }


@pytest.mark.parametrize("name", ["causal_alibi", "extra_fma", "clip_tanh_exp", "index_math"])
@pytest.mark.parametrize("ab,out", [("Float16", "Float32"), ("BFloat16", "BFloat16"),
                                    ("Float16", "Float16")])
@pytest.mark.parametrize("c_rowmajor", [False, True])
@pytest.mark.parametrize("M,N,K", [(300, 200, 136), (640, 768, 512)])
def test_perelement_program(lvb, torch_cuda, name, ab, out, c_rowmajor, M, N, K):
    """The traced program against the oracle's interpretation of the same instructions, with
    row/col 0-based in C's own orientation whichever way the kernel runs the product."""
    from lvb.perelement import program
    torch = torch_cuda
    fn, L, uses_extra = _programs()[name]
    prog = program(fn)
    A, Bt = gemm_inputs(M, N, K, ab, seed=K + len(name))
    E = np.random.default_rng(M).uniform(-1, 1, (M, N)).astype(np.float32)
    kw = dict(program=prog)
    if uses_extra:
        kw["extra"] = cmat(torch, E, "Float32", c_rowmajor)
    got = run(lvb, torch, A, Bt, ab, out, c_rowmajor, **kw)
    ref = gemm_vocab_ref(A, Bt.T, out, ab, program=prog.code, extra=E if uses_extra else None)
    A64, B64 = A.astype(np.float64), Bt.T.astype(np.float64)
    compare(got, ref, A64, B64, 0.0, out, L=L, floor=2.0 ** -18)


def test_program_with_full_epilogue_and_k0(lvb, torch_cuda):
    """bias + residual + mul + activation + program together; K = 0 gives
    program(act((bias + R) ⊙ S)) through the epilogue-only kernel."""
    from lvb.perelement import program, where
    torch = torch_cuda
    prog = program(lambda x, r, c, e: where(c < r, x, 2.0 * x + e))
    g = np.random.default_rng(5)
    for K in (96, 0):
        M, N = 130, 70
        A, Bt = gemm_inputs(M, N, K, "Float16", seed=3)
        S = g.uniform(-1, 1, (M, N)).astype(np.float32)
        R = g.uniform(-1, 1, (M, N)).astype(np.float32)
        E = g.uniform(-1, 1, (M, N)).astype(np.float32)
        bias = g.uniform(-1, 1, M).astype(np.float32)
        for crm in (False, True):
            got = run(lvb, torch, A, Bt, "Float16", "Float32", crm, bias=dev(torch, bias, "Float32"),
                      bias_axis="row", residual=cmat(torch, R, "Float32", crm),
                      mul=cmat(torch, S, "Float32", crm), activation="silu", program=prog,
                      extra=cmat(torch, E, "Float32", crm))
            ref = gemm_vocab_ref(A, Bt.T, "Float32", "Float16", bias=bias, bias_axis="row",
                                 residual=R, mul=S, act="silu", program=prog.code, extra=E)
            compare(got, ref, A.astype(np.float64), Bt.T.astype(np.float64),
                    np.abs(R) + np.abs(bias)[:, None], "Float32", L=2.2)


# ---- clamp modes on the k tail ------------------------------------------------------------
@pytest.mark.parametrize("ab,out", [("Float16", "Float32"), ("BFloat16", "BFloat16"),
                                    ("Int8", "Int32")])
@pytest.mark.parametrize("a_clamp,b_clamp", [(("constant", 1.0), ("constant", -0.5)),
                                             (("edge", 0), ("constant", 3)),
                                             (("edge", 0), ("edge", 0)),
                                             (("constant", 2), ("undefined", 0))])
@pytest.mark.parametrize("M,N,K,k_pad", [(300, 200, 100, 128), (129, 257, 1000, 1024),
                                         (64, 96, 8, 200)])
@pytest.mark.parametrize("c_rowmajor", [False, True])
def test_clamp_modes_k_tail(lvb, torch_cuda, ab, out, a_clamp, b_clamp, M, N, K, k_pad,
                            c_rowmajor):
    torch = torch_cuda
    A, Bt = gemm_inputs(M, N, K, ab, seed=M + K + k_pad)
    if ab == "Int8":   # an 8-bit operand's clamp value is an integer in its range
        a_clamp = (a_clamp[0], int(np.floor(a_clamp[1])))
        b_clamp = (b_clamp[0], int(np.floor(b_clamp[1])))
    spec = {"constant": lambda v: v, "edge": lambda v: "edge", "undefined": lambda v: None}
    got = run(lvb, torch, A, Bt, ab, out, c_rowmajor, k_pad=k_pad,
              a_clamp=spec[a_clamp[0]](a_clamp[1]), b_clamp=spec[b_clamp[0]](b_clamp[1]))
    ref = gemm_vocab_ref(A, Bt.T, out, ab, k_pad=k_pad, a_clamp=a_clamp, b_clamp=b_clamp)
    if out == "Int32":
        assert np.array_equal(got, ref)
        return
    Ap = clamp_pad(A, k_pad, 1, *a_clamp, ab).astype(np.float64)
    Bp = clamp_pad(Bt.T, k_pad, 0, *b_clamp, ab).astype(np.float64)
    compare(got, ref, Ap, Bp, 0.0, out)


def test_clamp_operands_mn_major_and_repacked(lvb, torch_cuda):
    """TO_EDGE reads the edge element of an operand stored MN-contiguous (A column-major, B
    row-major: read in place), and of operands copied to the aligned workspace first."""
    torch = torch_cuda
    M, N, K, k_pad = 200, 136, 70, 128
    A, Bt = gemm_inputs(M, N, K, "Float16", seed=17)
    dA = dev(torch, np.ascontiguousarray(A.T), "Float16").t()          # column-major A
    dB = dev(torch, np.ascontiguousarray(Bt.T), "Float16")             # row-major B (K×N)
    dC = torch.empty((N, M), dtype=torch.float32, device="cuda").t()
    lvb.gemm(dC, dA, dB, k_pad=k_pad, a_clamp="edge", b_clamp="edge")
    torch.cuda.synchronize()
    ref = gemm_vocab_ref(A, Bt.T, "Float32", "Float16", k_pad=k_pad, a_clamp=("edge", 0),
                         b_clamp=("edge", 0))
    Ap = clamp_pad(A, k_pad, 1, "edge", 0, "Float16").astype(np.float64)
    Bp = clamp_pad(Bt.T, k_pad, 0, "edge", 0, "Float16").astype(np.float64)
    compare(dC.cpu().numpy(), ref, Ap, Bp, 0.0, "Float32")
    # K = 70 fp16 rows are 140 bytes (not a 16-byte multiple): both operands repacked
    dA2 = dev(torch, A, "Float16")
    dB2 = dev(torch, Bt, "Float16").t()
    dC2 = torch.empty((N, M), dtype=torch.float32, device="cuda").t()
    lvb.gemm(dC2, dA2, dB2, k_pad=k_pad, a_clamp="edge", b_clamp=0.75)
    torch.cuda.synchronize()
    ref2 = gemm_vocab_ref(A, Bt.T, "Float32", "Float16", k_pad=k_pad, a_clamp=("edge", 0),
                          b_clamp=("constant", 0.75))
    Bp2 = clamp_pad(Bt.T, k_pad, 0, "constant", 0.75, "Float16").astype(np.float64)
    compare(dC2.cpu().numpy(), ref2, Ap, Bp2, 0.0, "Float32")


def test_clamp_k0_constant_and_checks(lvb, torch_cuda):
    """K = 0 with constant clamps: every element is k_pad·a·b (+ the epilogue); TO_EDGE with
    K = 0 and out-of-range 8-bit constants are argument errors."""
    torch = torch_cuda
    dA = torch.empty(5, 0, dtype=torch.float16, device="cuda")
    dB = torch.empty(0, 7, dtype=torch.float16, device="cuda")
    dC = torch.full((5, 7), 3.0, device="cuda")
    lvb.gemm(dC, dA, dB, k_pad=64, a_clamp=1.5, b_clamp=-2.0)
    torch.cuda.synchronize()
    assert torch.all(dC == 64 * 1.5 * -2.0)
    with pytest.raises(lvb.LavaError) as e:
        lvb.gemm(dC, dA, dB, k_pad=64, a_clamp="edge", b_clamp=1.0)
    assert e.value.status == lvb.LVB_ERR_INVALID_ARG
    A8 = torch.zeros(8, 16, dtype=torch.int8, device="cuda")
    B8 = torch.zeros(16, 8, dtype=torch.int8, device="cuda")
    C8 = torch.zeros(8, 8, dtype=torch.int32, device="cuda")
    with pytest.raises(lvb.LavaError) as e:
        lvb.gemm(C8, A8, B8, k_pad=32, a_clamp=200, b_clamp=1)
    assert e.value.status == lvb.LVB_ERR_INVALID_ARG


def test_vocab_epilogue_on_pair_tile_224(lvb, torch_cuda):
    """The fused epilogue (bias, residual, mul, activation, program, clamp) on the 256×224
    CTA-pair tile, whose accumulator drains in seven 32-column chunks."""
    from lvb.perelement import program, where
    torch = torch_cuda
    M, N, K, k_pad = 1024, 8192, 200, 256
    plan = lvb.gemm_plan(M, N, K, lvb.F16, lvb.F32, c_rowmajor=True)
    assert plan.cta_pair == 1 and plan.tile_n == 224
    A, Bt = gemm_inputs(M, N, K, "Float16", seed=224)
    g = np.random.default_rng(224)
    S = g.uniform(-1, 1, (M, N)).astype(np.float32)
    R = g.uniform(-1, 1, (M, N)).astype(np.float16)
    bias = g.uniform(-1, 1, N).astype(np.float32)
    prog = program(lambda x, r, c, e: where(c > r + 4000, 0.0, x))
    got = run(lvb, torch, A, Bt, "Float16", "Float32", True, bias=dev(torch, bias, "Float32"),
              residual=dev(torch, R, "Float16"), mul=dev(torch, S, "Float32"), activation="silu",
              program=prog, k_pad=k_pad, a_clamp="edge", b_clamp=0.5)
    ref = gemm_vocab_ref(A, Bt.T, "Float32", "Float16", bias=bias, residual=R, mul=S, act="silu",
                         program=prog.code, k_pad=k_pad, a_clamp=("edge", 0),
                         b_clamp=("constant", 0.5))
    Ap = clamp_pad(A, k_pad, 1, "edge", 0, "Float16").astype(np.float64)
    Bp = clamp_pad(Bt.T, k_pad, 0, "constant", 0.5, "Float16").astype(np.float64)
    compare(got, ref, Ap, Bp, np.abs(R) + np.abs(bias), "Float32", L=1.1)

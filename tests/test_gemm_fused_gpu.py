"""GPU tier: the fused GEMM epilogue (lvb_gemm_ex) and transposed (MN-contiguous) operands,
through the C ABI, against the oracle.

Tolerances (written here):
  * relative Frobenius <= 1e-3 against the oracle rounded once to the output type;
  * per element |Δ| <= one output ulp + slope·(fp32 accumulation bound + two fp32 roundings
    of the pre-activation) + 2^-19·(|pre-activation| + |result|): the last term covers the
    fp32 activation itself (the kernel's exp is the hardware approximation, a few ulp plus
    an error growing with |argument|);
  * integer products with transposed operands: bit-exact.
"""
import numpy as np
import pytest

from oracle.gemm import (ACTIVATION_SLOPE, epilogue_init, gemm_epilogue_ref, gemm_ref,
                         rel_frobenius)
from oracle.inputs import gemm_inputs

pytestmark = pytest.mark.gpu
TORCH_DT = {"Float16": "float16", "BFloat16": "bfloat16", "Float32": "float32",
            "Int8": "int8", "UInt8": "uint8", "Int32": "int32"}


def _dev(torch, x, T):
    t = torch.from_numpy(np.ascontiguousarray(x))
    if T == "BFloat16":
        t = t.to(torch.bfloat16)
    return t.cuda()


def _operand(torch, X, T, contiguous_dim):
    """A device view of matrix X (rows, cols) whose `contiguous_dim` (0 or 1) is unit-stride."""
    if contiguous_dim == 1:
        return _dev(torch, X, T)
    return _dev(torch, np.ascontiguousarray(X.T), T).t()


def _out_ulp(x, out):
    ax = np.abs(np.asarray(x, dtype=np.float64))
    if out == "Float16":
        return np.spacing(np.minimum(ax, 65504).astype(np.float16)).astype(np.float64)
    if out == "BFloat16":
        e = np.floor(np.log2(np.maximum(ax, 2.0 ** -126)))
        return 2.0 ** (e - 7)
    return np.spacing(ax.astype(np.float32)).astype(np.float64)


def _to_np(torch, t):
    if t.dtype == torch.bfloat16:
        return t.float().cpu().numpy()
    return t.cpu().numpy()


def check_fused(Cg, A, B, out, bias=None, bias_axis="col", residual=None, act=None):
    ref = gemm_epilogue_ref(A, B, out, bias, bias_axis, residual, act)
    exact = gemm_epilogue_ref(A, B, out, bias, bias_axis, residual, act, rounded=False)
    C64 = np.asarray(Cg, dtype=np.float64)
    assert np.isfinite(C64).all()
    assert rel_frobenius(C64, np.asarray(ref, dtype=np.float64)) <= 1e-3
    K = A.shape[1]
    A64, B64 = A.astype(np.float64), B.astype(np.float64)
    init = np.abs(epilogue_init(A.shape[0], B.shape[1], bias, bias_axis, residual)).astype(np.float64)
    pre = A64 @ B64 + init
    acc = 4.0 * np.sqrt(max(K, 1)) * 2.0 ** -24 * (np.abs(A64) @ np.abs(B64))
    round2 = 2.0 ** -23 * (np.abs(pre) + init)
    bound = (_out_ulp(exact, out) + ACTIVATION_SLOPE[act] * (acc + round2)
             + 2.0 ** -19 * (np.abs(pre) + np.abs(exact)) + 1e-30)
    err = np.abs(C64 - exact)
    bad = err > bound
    assert not bad.any(), (f"{int(bad.sum())} elements out of bound; worst excess "
                           f"{float((err - bound).max()):.3e}")


SHAPES = [(127, 129, 72), (300, 520, 200), (640, 64, 1024), (2048, 2048, 256)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("act", [None, "relu", "gelu", "gelu_erf", "silu"])
def test_bias_residual_activation(lvb, torch_cuda, M, N, K, act):
    torch = torch_cuda
    rng = np.random.default_rng(M + N + K)
    A, Bt = gemm_inputs(M, N, K, "Float16", seed=M * 3 + K)
    B = Bt.T
    bias = rng.uniform(-2, 2, N).astype(np.float16)
    res = rng.uniform(-4, 4, (M, N)).astype(np.float32)
    for c_rowmajor in (True, False):
        dA = _operand(torch, A, "Float16", 1)
        dB = _operand(torch, B, "Float16", 0)
        dbias = _dev(torch, bias, "Float16")
        dres = _operand(torch, res, "Float32", 1 if c_rowmajor else 0)
        dC = _operand(torch, np.full((M, N), 7, np.float32), "Float32", 1 if c_rowmajor else 0)
        lvb.gemm(dC, dA, dB, bias=dbias, residual=dres, activation=act)
        torch.cuda.synchronize()
        assert lvb.device_status() == (0, 0, 0)
        check_fused(_to_np(torch, dC), A, B, "Float32", bias, "col", res, act)


@pytest.mark.parametrize("ab,out,btype,rtype", [
    ("Float16", "Float16", "Float32", "Float16"),
    ("BFloat16", "BFloat16", "BFloat16", "BFloat16"),
    ("Float16", "BFloat16", "Float16", "Float32"),
])
@pytest.mark.parametrize("axis", ["row", "col"])
def test_types_and_bias_axis(lvb, torch_cuda, ab, out, btype, rtype, axis):
    torch = torch_cuda
    M, N, K = 384, 264, 520
    rng = np.random.default_rng(5)
    A, Bt = gemm_inputs(M, N, K, ab, seed=11)
    B = Bt.T
    bias = rng.uniform(-1, 1, M if axis == "row" else N).astype(np.float32)
    res = rng.uniform(-1, 1, (M, N)).astype(np.float32)
    if btype == "Float16":
        bias = bias.astype(np.float16)
    if rtype == "Float16":
        res = res.astype(np.float16)
    from oracle.vocab import round_bf16
    if btype == "BFloat16":
        bias = round_bf16(bias)
    if rtype == "BFloat16":
        res = round_bf16(res)
    cdt = getattr(torch, TORCH_DT[out])
    for c_rowmajor in (True, False):
        cd = 1 if c_rowmajor else 0
        dC = (torch.zeros(M, N, dtype=cdt, device="cuda") if c_rowmajor
              else torch.zeros(N, M, dtype=cdt, device="cuda").t())
        lvb.gemm(dC, _operand(torch, A, ab, 1), _operand(torch, B, ab, 0),
                 bias=_dev(torch, bias, btype), bias_axis=axis,
                 residual=_operand(torch, res, rtype, cd), activation="gelu")
        torch.cuda.synchronize()
        check_fused(_to_np(torch, dC), A, B, out, bias, axis, res, "gelu")


def test_residual_in_place(lvb, torch_cuda):
    """C = A·B + C: the residual is the output itself (read before write per element)."""
    torch = torch_cuda
    M, N, K = 1000, 776, 384
    A, Bt = gemm_inputs(M, N, K, "BFloat16", seed=3)
    B = Bt.T
    rng = np.random.default_rng(8)
    from oracle.vocab import round_bf16
    c0 = round_bf16(rng.uniform(-8, 8, (M, N)).astype(np.float32))
    dC = _dev(torch, c0, "BFloat16")
    lvb.gemm(dC, _operand(torch, A, "BFloat16", 1), _operand(torch, B, "BFloat16", 0), residual=dC)
    torch.cuda.synchronize()
    check_fused(_to_np(torch, dC), A, B, "BFloat16", residual=c0)


def test_k_zero_epilogue(lvb, torch_cuda):
    """K = 0: the empty sum, so C = act(bias + residual)."""
    torch = torch_cuda
    M, N = 70, 45
    rng = np.random.default_rng(2)
    bias = rng.uniform(-1, 1, M).astype(np.float32)
    res = rng.uniform(-1, 1, (M, N)).astype(np.float32)
    dC = torch.full((M, N), 9.0, device="cuda")
    lvb.gemm(dC, torch.empty(M, 0, dtype=torch.float16, device="cuda"),
             torch.empty(0, N, dtype=torch.float16, device="cuda"),
             bias=_dev(torch, bias, "Float32"), bias_axis="row",
             residual=_dev(torch, res, "Float32"), activation="silu")
    torch.cuda.synchronize()
    A = np.zeros((M, 0), np.float16)
    B = np.zeros((0, N), np.float16)
    check_fused(dC.cpu().numpy(), A, B, "Float32", bias, "row", res, "silu")


def test_epilogue_matches_plain_gemm_when_empty(lvb, torch_cuda):
    """An epilogue with nothing in it is the plain GEMM, bit for bit."""
    torch = torch_cuda
    A, Bt = gemm_inputs(256, 512, 1024, "Float16", seed=4)
    dA, dB = _operand(torch, A, "Float16", 1), _operand(torch, Bt.T, "Float16", 0)
    c1 = torch.empty(256, 512, dtype=torch.float16, device="cuda")
    c2 = torch.empty_like(c1)
    lvb.gemm(c1, dA, dB)
    lvb.gemm(c2, dA, dB, activation="none", bias=torch.zeros(512, dtype=torch.float32, device="cuda"))
    torch.cuda.synchronize()
    assert torch.equal(c1, c2)


# ---- transposed operands ----------------------------------------------------------------
# (1536, 1024, 256) plans 128-wide tiles, (4736, 2048, 128) 256-wide 1-CTA tiles, (2048,
# 2048, 512) CTA pairs, the small ones 64-wide tiles.
@pytest.mark.parametrize("M,N,K", [(1, 1, 8), (129, 200, 72), (300, 520, 1000), (2048, 2048, 512),
                                   (1536, 1024, 256), (4736, 2048, 128)])
@pytest.mark.parametrize("ab,out", [("Float16", "Float32"), ("BFloat16", "BFloat16"),
                                    ("Float16", "Float16")])
@pytest.mark.parametrize("a_rm,b_rm", [(0, 0), (1, 1), (0, 1)])
def test_transposed_float(lvb, torch_cuda, M, N, K, ab, out, a_rm, b_rm):
    """A column-major and/or B row-major (Lava's transposing tensor view): read MN-major by
    the tensor core in place (16-bit), or copied K-major when TMA cannot address them."""
    torch = torch_cuda
    A, Bt = gemm_inputs(M, N, K, ab, seed=M + 2 * N + 3 * K)
    B = Bt.T
    for c_rowmajor in (True, False):
        dA = _operand(torch, A, ab, 1 if a_rm else 0)
        dB = _operand(torch, B, ab, 1 if b_rm else 0)
        cdt = getattr(torch, TORCH_DT[out])
        dC = (torch.empty(M, N, dtype=cdt, device="cuda") if c_rowmajor
              else torch.empty(N, M, dtype=cdt, device="cuda").t())
        lvb.gemm(dC, dA, dB)
        torch.cuda.synchronize()
        assert lvb.device_status() == (0, 0, 0)
        check_fused(_to_np(torch, dC), A, B, out)


@pytest.mark.parametrize("M,N,K", [(130, 300, 272), (512, 512, 4096)])
@pytest.mark.parametrize("ab,out", [("Int8", "Int32"), ("UInt8", "UInt32")])
@pytest.mark.parametrize("a_rm,b_rm", [(0, 0), (1, 1), (0, 1)])
def test_transposed_integer_exact(lvb, torch_cuda, M, N, K, ab, out, a_rm, b_rm):
    torch = torch_cuda
    A, Bt = gemm_inputs(M, N, K, ab, seed=M + N + K)
    B = Bt.T
    dA = _operand(torch, A, ab, 1 if a_rm else 0)
    dB = _operand(torch, B, ab, 1 if b_rm else 0)
    dC = torch.empty(M, N, dtype=torch.int32, device="cuda")
    lvb.gemm(dC, dA, dB, c_type=lvb.U32 if out == "UInt32" else None)
    torch.cuda.synchronize()
    got = dC.cpu().numpy()
    if out == "UInt32":
        got = got.view(np.uint32)
    assert np.array_equal(got, gemm_ref(A, B, out))


def test_transposed_unaligned_leading_dimension(lvb, torch_cuda):
    """An MN-contiguous operand whose leading dimension is not a 16-byte multiple (M = 100
    fp16 = 200 bytes) goes through the transposing device copy."""
    torch = torch_cuda
    M, N, K = 100, 72, 136
    A, Bt = gemm_inputs(M, N, K, "Float16", seed=13)
    dA = _operand(torch, A, "Float16", 0)           # column-major, lda = 100
    dB = _operand(torch, Bt.T, "Float16", 1)        # row-major, ldb = 72 (144 bytes)
    dC = torch.empty(M, N, device="cuda")
    lvb.gemm(dC, dA, dB, activation="relu")
    torch.cuda.synchronize()
    check_fused(dC.cpu().numpy(), A, Bt.T, "Float32", act="relu")

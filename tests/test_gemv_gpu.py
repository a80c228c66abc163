"""GPU tier: matrix-vector products — lvb_gemm / lvb_gemm_ex with N == 1 or M == 1 — through
the C ABI against the oracle. These run on the HBM-bound kernel (dot4x8 for 8-bit operands,
Lava's src/vocabulary/vocabulary.jl:18-35), not on the tensor core.

Tolerances (written here, the same as the GEMM's):
  * integer pairs: bit-exact (int64 oracle, Int8 signed / UInt8 unsigned);
  * Float32 output: relative Frobenius <= 1e-3 and per-element |Δ| <= 1e-2 against the float64
    product; Float16 / BFloat16 output: one output ulp plus the fp32 accumulation bound
    against the float64 product (and rel-Frobenius <= 1e-3 against it rounded once);
  * fused epilogue: the bound of the fused-GEMM tests.
"""
import numpy as np
import pytest

from oracle.gemm import gemm_ref
from oracle.inputs import gemm_inputs
from test_gemm_fused_gpu import check_fused
from test_gemm_gpu import check

pytestmark = pytest.mark.gpu
TORCH_DT = {"Float16": "float16", "BFloat16": "bfloat16", "Float32": "float32",
            "Int8": "int8", "UInt8": "uint8", "Int32": "int32", "UInt32": "int32"}


def _dev(torch, x, T):
    t = torch.from_numpy(np.ascontiguousarray(x))
    if T == "BFloat16":
        t = t.to(torch.bfloat16)
    return t.cuda()


def _matrix(torch, X, T, rowmajor, pad=0, offset=0):
    """Device view of X (rows, cols): row-major or column-major, leading dimension padded by
    `pad` elements, starting `offset` elements into its buffer."""
    r, c = X.shape
    if rowmajor:
        ld = c + pad
        buf = torch.zeros(offset + r * ld, dtype=getattr(torch, TORCH_DT[T]), device="cuda")
        v = buf[offset:].view(r, ld)[:, :c]
        v.copy_(_dev(torch, X, T))
        return v
    ld = r + pad
    buf = torch.zeros(offset + c * ld, dtype=getattr(torch, TORCH_DT[T]), device="cuda")
    v = buf[offset:].view(c, ld)[:, :r].t()
    v.copy_(_dev(torch, X, T))
    return v


def _out(torch, M, N, T, rowmajor, pad=0):
    dt = getattr(torch, TORCH_DT[T])
    if rowmajor:
        return torch.full((M, N + pad), 7, dtype=dt, device="cuda")[:, :N]
    return torch.full((N, M + pad), 7, dtype=dt, device="cuda")[:, :M].t()


def _np(torch, t, T):
    t = t.cpu()
    if T == "BFloat16":
        return t.float().numpy()
    if T == "UInt32":
        return t.numpy().view(np.uint32)
    return t.numpy()


def _run(lvb, torch, A, B, ab, out, a_rm=True, b_rm=False, c_rm=False, pads=(0, 0, 0),
         offsets=(0, 0)):
    M, K = A.shape
    N = B.shape[1]
    dA = _matrix(torch, A, ab, a_rm, pads[0], offsets[0])
    dB = _matrix(torch, B, ab, b_rm, pads[1], offsets[1])
    dC = _out(torch, M, N, out, c_rm, pads[2])
    lvb.gemm(dC, dA, dB, c_type=lvb.U32 if out == "UInt32" else None)
    torch.cuda.synchronize()
    assert lvb.device_status() == (0, 0, 0)
    return _np(torch, dC, out)


def _check(C, A, B, out):
    if out in ("Int32", "UInt32"):
        assert np.array_equal(C, gemm_ref(A, B, out))
    else:
        check(C, A, B, out)


@pytest.mark.parametrize("ab,out", [("Int8", "Int32"), ("UInt8", "UInt32")])
@pytest.mark.parametrize("M,K", [(4096, 4096), (1000, 1234), (3, 100003), (70001, 40), (1, 1),
                                 (257, 16)])
@pytest.mark.parametrize("a_rm", [True, False])
def test_int8_matvec_exact(lvb, torch_cuda, ab, out, M, K, a_rm):
    A, Bt = gemm_inputs(M, 1, K, ab, seed=11)
    C = _run(lvb, torch_cuda, A, Bt.T, ab, out, a_rm=a_rm)
    _check(C, A, Bt.T, out)


@pytest.mark.parametrize("ab", ["Float16", "BFloat16"])
@pytest.mark.parametrize("out", ["Float32", "Float16", "BFloat16"])
@pytest.mark.parametrize("M,K", [(4096, 4096), (777, 1001), (64, 65536), (50000, 24)])
@pytest.mark.parametrize("a_rm", [True, False])
def test_float_matvec(lvb, torch_cuda, ab, out, M, K, a_rm):
    A, Bt = gemm_inputs(M, 1, K, ab, seed=12)
    C = _run(lvb, torch_cuda, A, Bt.T, ab, out, a_rm=a_rm)
    _check(C, A, Bt.T, out)


@pytest.mark.parametrize("ab,out", [("Float16", "Float32"), ("BFloat16", "BFloat16"),
                                    ("Int8", "Int32")])
@pytest.mark.parametrize("N,K", [(4096, 3000), (100000, 64), (129, 40000)])
@pytest.mark.parametrize("b_rm", [True, False])
@pytest.mark.parametrize("c_rm", [True, False])
def test_vector_matrix_m1(lvb, torch_cuda, ab, out, N, K, b_rm, c_rm):
    A, Bt = gemm_inputs(1, N, K, ab, seed=13)
    C = _run(lvb, torch_cuda, A, Bt.T, ab, out, b_rm=b_rm, c_rm=c_rm)
    _check(C, A, Bt.T, out)


@pytest.mark.parametrize("ab,out", [("Float16", "Float16"), ("Int8", "Int32")])
@pytest.mark.parametrize("a_rm", [True, False])
def test_strided_and_unaligned(lvb, torch_cuda, ab, out, a_rm):
    """Leading dimensions that are not 16-byte multiples, operands one element off a 16-byte
    boundary, x with a stride (a column of a row-major B), y with a stride (a column of a
    row-major C): the element-wise paths."""
    M, K = 1031, 777
    A, Bt = gemm_inputs(M, 1, K, ab, seed=14)
    for pads, offs, b_rm, c_rm in [((3, 0, 0), (1, 0), False, False),
                                   ((0, 2, 4), (0, 1), True, True),
                                   ((5, 3, 2), (3, 3), True, False)]:
        C = _run(lvb, torch_cuda, A, Bt.T, ab, out, a_rm=a_rm, b_rm=b_rm, c_rm=c_rm, pads=pads,
                 offsets=offs)
        _check(C, A, Bt.T, out)


@pytest.mark.parametrize("shape", [(3000, 1, 2048), (1, 3000, 2048), (48, 1, 70000)])
@pytest.mark.parametrize("act", [None, "relu", "gelu", "silu"])
@pytest.mark.parametrize("axis", ["row", "col"])
def test_matvec_fused_epilogue(lvb, torch_cuda, shape, act, axis):
    torch = torch_cuda
    M, N, K = shape
    A, Bt = gemm_inputs(M, N, K, "Float16", seed=15)
    B = Bt.T
    rng = np.random.default_rng(16)
    bias = rng.uniform(-1, 1, M if axis == "row" else N).astype(np.float32)
    res = rng.uniform(-1, 1, (M, N)).astype(np.float32).astype(np.float16)
    for c_rm in (False, True):
        dC = _out(torch, M, N, "Float16", c_rm)
        dR = _matrix(torch, res, "Float16", c_rm)
        lvb.gemm(dC, _matrix(torch, A, "Float16", True), _matrix(torch, B, "Float16", False),
                 bias=torch.from_numpy(bias).cuda(), bias_axis=axis, residual=dR, activation=act)
        torch.cuda.synchronize()
        assert lvb.device_status() == (0, 0, 0)
        check_fused(_np(torch, dC, "Float16"), A, B, "Float16", bias, axis,
                    res.astype(np.float32), act)


def test_matvec_deterministic(lvb, torch_cuda):
    """The k splits are added in a fixed order: two runs give identical bits."""
    torch = torch_cuda
    A, Bt = gemm_inputs(96, 1, 300000, "BFloat16", seed=17)
    r1 = _run(lvb, torch, A, Bt.T, "BFloat16", "Float32")
    r2 = _run(lvb, torch, A, Bt.T, "BFloat16", "Float32")
    assert np.array_equal(r1, r2)
    check(r1, A, Bt.T, "Float32")

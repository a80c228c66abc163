"""GPU tier: lvb_gemm_noalloc, the GEMM entry point for callers that must not allocate
device memory while they run it (a runtime that owns all device memory through its own
pool, a serving loop that forbids allocation after warm-up). Its scratch is one static
device array shared by every call.

Each case calls it through the C ABI twice in a row and compares the result with what
lvb_gemm gives for the same operands, within the GEMM tests' tolerance (the two share the
kernels; a matrix-vector product that lvb_gemm splits over k, with partial sums in a
workspace, runs unsplit here, so fp32 sums may differ in the last bits), and with the
oracle. Collected last (file name) so a failure here does not hide any other test.
"""
import ctypes as C

import numpy as np
import pytest

from oracle.gemm import gemm_ref, rel_frobenius, max_abs
from oracle.inputs import gemm_inputs

pytestmark = pytest.mark.gpu


def _call(lvb, fn, dC, dA, dB):
    d = lvb.gemm_desc(dC, dA, dB)
    st = fn(C.byref(d), dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), None)
    lvb.check(st)


def _operands(torch, M, N, K, ab, seed, misaligned):
    A, Bt = gemm_inputs(M, N, K, ab, seed)
    tdt = {"Float16": torch.float16, "Int8": torch.int8}[ab]
    if misaligned:
        # base off a 16-byte boundary and a leading dimension that is not a 16-byte multiple:
        # the workspace path
        ld = K + 3
        buf = torch.zeros(M * ld + 1, dtype=tdt, device="cuda")
        dA = buf[1:].view(M, ld)[:, :K]
        dA.copy_(torch.from_numpy(A))
    else:
        dA = torch.from_numpy(A).cuda()
    dB = torch.from_numpy(Bt).cuda()
    return A, Bt, dA, dB.t()


@pytest.mark.parametrize("misaligned", [False, True])
@pytest.mark.parametrize("ab,out,M,N,K", [("Float16", "Float32", 384, 520, 328),
                                          ("Int8", "Int32", 260, 300, 520),
                                          ("Int8", "Int32", 4096, 1, 8192),
                                          ("Float16", "Float32", 64, 1, 100000)])
def test_noalloc_matches_lvb_gemm_twice(lvb, torch_cuda, misaligned, ab, out, M, N, K):
    torch = torch_cuda
    A, Bt, dA, dB = _operands(torch, M, N, K, ab, seed=M + K, misaligned=misaligned)
    odt = torch.float32 if out == "Float32" else torch.int32
    ref_dev = torch.empty(N, M, dtype=odt, device="cuda").t()
    _call(lvb, lvb.lib.lvb_gemm, ref_dev, dA, dB)
    torch.cuda.synchronize()
    expect = ref_dev.cpu().numpy()
    oracle = gemm_ref(A, Bt.T, out)
    for _ in range(2):
        dC = torch.full((N, M), 9, dtype=odt, device="cuda").t()
        _call(lvb, lvb.lib.lvb_gemm_noalloc, dC, dA, dB)
        torch.cuda.synchronize()
        got = dC.cpu().numpy()
        if out == "Int32":
            assert np.array_equal(got, expect)
            assert np.array_equal(got, oracle)
        else:
            assert max_abs(got, expect) <= 1e-2 and rel_frobenius(got, expect) <= 1e-3
            exact = A.astype(np.float64) @ Bt.T.astype(np.float64)
            assert max_abs(got, exact) <= 1e-2 and rel_frobenius(got, exact) <= 1e-3


def test_noalloc_refuses_workspace_beyond_limit(lvb, torch_cuda):
    torch = torch_cuda
    # 4096 x 4099 fp16 rows need repacking: 4096*4112*2 bytes = 32.9 MB > 16 MiB
    M, N, K = 4096, 64, 4099
    dA = torch.zeros(M, K, dtype=torch.float16, device="cuda")
    dB = torch.zeros(N, K + 5, dtype=torch.float16, device="cuda")[:, :K].t()
    dC = torch.zeros(N, M, device="cuda").t()
    d = lvb.gemm_desc(dC, dA, dB)
    st = lvb.lib.lvb_gemm_noalloc(C.byref(d), dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), None)
    assert st == lvb.LVB_ERR_UNSUPPORTED
    msg = lvb.lib.lvb_last_error().decode()
    assert msg.startswith("lvb_gemm_noalloc: ") and "static workspace" in msg

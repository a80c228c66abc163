"""GPU tier: lvb_gemm_noalloc, the GEMM entry point for callers that must not allocate
device memory while they run it (a runtime that owns all device memory through its own
pool, a serving loop that forbids allocation after warm-up). Its scratch is one static
device array shared by every call.

Each case calls it through the C ABI twice in a row and compares the result with what
lvb_gemm gives for the same operands, within the GEMM tests' tolerance (the two share the
kernels; a matrix-vector product that lvb_gemm splits over k, with partial sums in a
workspace, runs unsplit here, so fp32 sums may differ in the last bits), and with the
oracle. Further cases: the CTA-pair kernel's shapes, 8-bit operands stored MN-contiguous
(always copied, so the workspace limit applies at any alignment), the status word's own
reader after a bounded wait ran out, and a fresh process whose first library call is
lvb_gemm_noalloc, in which device memory stays the same across repeated calls. Collected
last (file name) so a failure here does not hide any other test.
"""
import ctypes as C
import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest

from oracle.gemm import gemm_ref, rel_frobenius, max_abs
from oracle.inputs import gemm_inputs

pytestmark = pytest.mark.gpu


def _call(lvb, fn, dC, dA, dB):
    d = lvb.gemm_desc(dC, dA, dB)
    st = fn(C.byref(d), dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), None)
    lvb.check(st)


def _operands(torch, M, N, K, ab, seed, misaligned, a_colmajor=False):
    A, Bt = gemm_inputs(M, N, K, ab, seed)
    tdt = {"Float16": torch.float16, "Int8": torch.int8}[ab]
    if a_colmajor:
        # A stored column-major (MN-contiguous): the (K, M) storage array viewed transposed
        dA = torch.from_numpy(np.ascontiguousarray(A.T)).cuda().t()
    elif misaligned:
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
                                          ("Float16", "Float32", 64, 1, 100000),
                                          # 64 tiles of 256 x 256 on CTA pairs
                                          ("Float16", "Float32", 2048, 2048, 512),
                                          ("Int8", "Int32", 2048, 2048, 512)])
def test_noalloc_matches_lvb_gemm_twice(lvb, torch_cuda, misaligned, ab, out, M, N, K):
    torch = torch_cuda
    if M == 2048:
        plan = lvb.gemm_plan(M, N, K, lvb.F16 if ab == "Float16" else lvb.I8,
                             lvb.F32 if out == "Float32" else lvb.I32)
        assert plan.cta_pair == 1
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


@pytest.mark.parametrize("M,K,fits", [(1024, 1024, True), (4096, 8192, False)])
def test_noalloc_int8_mn_contiguous(lvb, torch_cuda, M, K, fits):
    """An Int8 A stored column-major is copied K-major at any alignment: 1 MB of copy runs and
    matches the oracle exactly; 32 MB is refused, with a message that names the case."""
    torch = torch_cuda
    N = 64
    A, Bt, dA, dB = _operands(torch, M, N, K, "Int8", seed=M + 1, misaligned=False,
                              a_colmajor=True)
    assert dA.stride() == (1, M) and dA.data_ptr() % 16 == 0
    dC = torch.full((N, M), 9, dtype=torch.int32, device="cuda").t()
    d = lvb.gemm_desc(dC, dA, dB)
    st = lvb.lib.lvb_gemm_noalloc(C.byref(d), dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), None)
    if not fits:
        assert st == lvb.LVB_ERR_UNSUPPORTED
        msg = lvb.lib.lvb_last_error().decode()
        assert "static workspace" in msg and "8-bit operand stored MN-contiguous" in msg
        return
    lvb.check(st)
    torch.cuda.synchronize()
    assert np.array_equal(dC.cpu().numpy(), gemm_ref(A, Bt.T, "Int32"))


def test_noalloc_status_word_reader(lvb, torch_cuda):
    """A bounded wait that runs out against lvb_gemm_noalloc's status word (the self-test
    kernel, 50 ms) is reported by lvb_gemm_noalloc_status, not by lvb_device_status; the word
    is cleared once read and the next noalloc GEMM is correct."""
    torch = torch_cuda
    assert lvb.gemm_noalloc_status() == (0, 0, 0)
    lvb.check(lvb.lib.lvb_gemm_noalloc_selftest_wait_timeout(50, None))
    code, where, block = lvb.gemm_noalloc_status()
    assert code == lvb.LVB_ERR_TIMEOUT and where == 99 and block == 0
    assert lvb.gemm_noalloc_status() == (0, 0, 0)
    assert lvb.device_status() == (0, 0, 0)
    A, Bt, dA, dB = _operands(torch, 300, 200, 256, "Int8", seed=3, misaligned=True)
    dC = torch.empty(200, 300, dtype=torch.int32, device="cuda").t()
    _call(lvb, lvb.lib.lvb_gemm_noalloc, dC, dA, dB)
    assert lvb.gemm_noalloc_status() == (0, 0, 0)
    assert np.array_equal(dC.cpu().numpy(), gemm_ref(A, Bt.T, "Int32"))


_FRESH = textwrap.dedent("""
    import ctypes as C, sys
    import numpy as np, torch
    sys.path[:0] = [{repo!r}, {pkg!r}]
    import lvb
    from oracle.gemm import gemm_ref
    from oracle.inputs import gemm_inputs
    torch.cuda.set_device(0)
    cases = []
    for (ab, M, N, K, mis) in [("Float16", 384, 520, 328, False), ("Float16", 384, 520, 328, True),
                               ("Int8", 2048, 2048, 512, False), ("Int8", 4096, 1, 8192, True)]:
        A, Bt = gemm_inputs(M, N, K, ab, 7)
        tdt = torch.float16 if ab == "Float16" else torch.int8
        if mis:
            buf = torch.zeros(M * (K + 3) + 1, dtype=tdt, device="cuda")
            dA = buf[1:].view(M, K + 3)[:, :K]
            dA.copy_(torch.from_numpy(A))
        else:
            dA = torch.from_numpy(A).cuda()
        dB = torch.from_numpy(Bt).cuda().t()
        odt = torch.float32 if ab == "Float16" else torch.int32
        dC = torch.empty(N, M, dtype=odt, device="cuda").t()
        cases.append((A, Bt, dA, dB, dC, "Float32" if ab == "Float16" else "Int32"))
    torch.cuda.synchronize()

    def call_all():
        for (A, Bt, dA, dB, dC, out) in cases:
            d = lvb.gemm_desc(dC, dA, dB)
            lvb.check(lvb.lib.lvb_gemm_noalloc(C.byref(d), dA.data_ptr(), dB.data_ptr(),
                                               dC.data_ptr(), None))
        torch.cuda.synchronize()

    call_all()        # the first call of this process: loads the library's kernels
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        call_all()
    free1 = torch.cuda.mem_get_info()[0]
    for (A, Bt, dA, dB, dC, out) in cases:
        got = dC.cpu().numpy()
        ref = gemm_ref(A, Bt.T, out)
        if out == "Int32":
            assert np.array_equal(got, ref)
        else:
            assert np.abs(got.astype(np.float64) - ref).max() <= 1e-2
    assert lvb.gemm_noalloc_status() == (0, 0, 0)
    print("free", free0, free1)
    assert free0 == free1, (free0, free1)
""")


def test_noalloc_first_call_in_fresh_process_allocates_nothing_after(lvb, torch_cuda):
    """A process whose first library call is lvb_gemm_noalloc (aligned, misaligned, CTA-pair
    and matrix-vector shapes): after the first round of calls, which loads the kernels onto the
    device, three more rounds leave the device's free memory exactly where it was."""
    repo = Path(__file__).resolve().parents[1]
    code = _FRESH.format(repo=str(repo), pkg=str(repo / "lava.jl_b200"))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "free" in r.stdout

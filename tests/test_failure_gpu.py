"""GPU tier: failure detection without a GPU fault. Every in-kernel wait of the library is
bounded; a wait that nothing satisfies records LVB_ERR_TIMEOUT in the device status word,
the kernel returns, and the context stays usable — the counterpart of Lava's exception flag
read after a sync (src/compiler/entry_wrapper.jl:199-216). The wait here runs out after
50 ms: no fault, no hang."""
import time

import numpy as np
import pytest

from oracle.inputs import gemm_inputs

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(lvb, torch_cuda):
    torch = torch_cuda
    assert lvb.device_status() == (0, 0, 0)
    t0 = time.perf_counter()
    lvb.selftest_wait_timeout(50)
    code, where, block = lvb.device_status()          # synchronises
    elapsed = time.perf_counter() - t0
    assert code == lvb.LVB_ERR_TIMEOUT and where == 99 and block == 0
    assert 0.04 <= elapsed < 5.0
    # the status word is cleared once read
    assert lvb.device_status() == (0, 0, 0)
    # the context is still usable: a GEMM right after is correct
    A, Bt = gemm_inputs(128, 96, 64, "Int8", seed=1)
    dC = torch.empty(96, 128, dtype=torch.int32, device="cuda").t()
    lvb.gemm(dC, torch.from_numpy(A).cuda(), torch.from_numpy(Bt).cuda().t())
    torch.cuda.synchronize()
    ref = A.astype(np.int64) @ Bt.T.astype(np.int64)
    assert np.array_equal(dC.cpu().numpy(), ref)
    assert lvb.device_status() == (0, 0, 0)


def test_selftest_argument_checks(lvb, torch_cuda):
    with pytest.raises(lvb.LavaError) as e:
        lvb.selftest_wait_timeout(0)
    assert e.value.status == lvb.LVB_ERR_INVALID_ARG

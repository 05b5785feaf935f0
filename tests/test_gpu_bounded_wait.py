"""A device-side wait that runs out of time ends with an error status the host
reads, and the device stays usable.

Every wait in the library's kernels (TMA, MMA and softmax hand-offs of the
tensor-core attention, the GEMMs' rings) is bounded: past its limit it raises
the block's abort flag, which stops the block's other roles, and records a code
in the device status flag. awa_selftest_bounded_wait runs that same wait on
mbarriers nothing ever completes -- no copy, MMA or arrival is issued, so
nothing is in flight -- with a short limit. No fault, trap or hang is involved.
"""

import ctypes

import numpy as np
import pytest

from awa_testlib import BF16_REL_L2, make_inputs, plan_for, rel_l2, to_device, to_host
from oracle.oracle import LayerConfig

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import awa_b200  # noqa: E402


def test_wait_that_runs_out_reports_and_device_recovers(oracle):
    lib = awa_b200.library()
    awa_b200.device_status()  # start from a clear flag
    observed = ctypes.c_int(0)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.awa_selftest_bounded_wait(2000, ctypes.byref(observed), stream) == awa_b200.AWA_OK
    # bit 0: the 2 ms wait gave up; bit 1: the second waiter stopped on the abort flag
    assert observed.value == 3
    rc = lib.awa_device_status()
    assert rc == awa_b200.AWA_ERR_DEVICE
    assert "code 51" in lib.awa_last_error().decode()
    assert lib.awa_device_status() == awa_b200.AWA_OK  # read and cleared

    # the same GPU then runs a normal forward correctly
    cfg = LayerConfig(1, 16, 16, 1, 8, 8, shifted=1, heads=4)
    v, t = make_inputs(cfg, 5, True, oracle)
    ref = oracle.chain(cfg, v, t)
    video, text = plan_for(cfg).forward(to_device(v, torch.bfloat16), to_device(t, torch.bfloat16),
                                        awa_b200.AWA_PREC_BF16, out_dtype=torch.float32)
    torch.cuda.synchronize()
    awa_b200.device_status()
    assert rel_l2(to_host(video), ref["video"]) < BF16_REL_L2
    assert rel_l2(to_host(text), ref["text"]) < BF16_REL_L2


def test_selftest_rejects_unbounded_limits():
    lib = awa_b200.library()
    observed = ctypes.c_int(0)
    assert lib.awa_selftest_bounded_wait(0, ctypes.byref(observed), None) == awa_b200.AWA_ERR_INVALID
    assert lib.awa_selftest_bounded_wait(2_000_000, ctypes.byref(observed), None) == awa_b200.AWA_ERR_INVALID

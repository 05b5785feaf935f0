"""GPU parity of the AWA output's consumer (awa_out_project: proj_out, the Ada
"out" gate and the residual add) through the C ABI, against the oracle
restatement (oracle.out_project, bit-exact with FixedDitBlock's modules in
test_oracle.py) and against the reference fixture.

Tolerance: the kernel accumulates x W^T in another order than the CPU, so a
few of the Linear's bf16 outputs round the other way; relative L2 within 5e-3."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from awa_testlib import rel_l2

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import awa_b200  # noqa: E402
from oracle.oracle import out_project, round_bf16_rne  # noqa: E402

TOL = 5e-3


def _run(x, w, bias, gate, residual, res_dtype, out_dtype):
    dev = torch.device("cuda")
    got = awa_b200.out_project(torch.from_numpy(x).to(dev, torch.bfloat16), torch.from_numpy(w).to(dev, torch.bfloat16),
                               torch.from_numpy(bias).to(dev), torch.from_numpy(gate).to(dev),
                               torch.from_numpy(residual).to(dev, res_dtype), out_dtype=out_dtype)
    awa_b200.device_status()
    return got.float().cpu().numpy()


def test_reference_fixture():
    f = np.load(os.path.join(os.path.dirname(__file__), "golden", "out_project.npz"))
    got = _run(f["x"], f["w"], f["bias"], f["gate"], f["residual"], torch.float32, torch.float32)
    assert rel_l2(got, f["out"]) < TOL


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
@pytest.mark.parametrize("tokens,in_dim,out_dim", [(300, 2560, 2560), (1, 128, 128), (129, 384, 640)],
                         ids=["300x2560", "1x128", "129x384-640"])
def test_matches_oracle(tokens, in_dim, out_dim, dtype):
    """Residual and output in `dtype`."""
    rng = np.random.default_rng(tokens + in_dim + out_dim)
    x = round_bf16_rne(rng.standard_normal((tokens, in_dim), dtype=np.float32))
    w = round_bf16_rne((rng.standard_normal((out_dim, in_dim)) / np.sqrt(in_dim)).astype(np.float32))
    bias = (0.1 * rng.standard_normal(out_dim)).astype(np.float32)
    gate = (0.2 * rng.standard_normal(out_dim)).astype(np.float32)
    residual = rng.standard_normal((tokens, out_dim), dtype=np.float32)
    if dtype == torch.bfloat16:
        residual = round_bf16_rne(residual)
    ref = out_project(x, w, bias, gate, residual)
    if dtype == torch.bfloat16:
        ref = round_bf16_rne(ref)
    got = _run(x, w, bias, gate, residual, dtype, dtype)
    assert got.shape == ref.shape
    assert rel_l2(got, ref) < TOL


def test_rejects_bad_arguments():
    dev = torch.device("cuda")
    x = torch.zeros(4, 128, dtype=torch.bfloat16, device=dev)
    w = torch.zeros(192, 128, dtype=torch.bfloat16, device=dev)
    v = torch.zeros(192, device=dev)
    res = torch.zeros(4, 192, device=dev)
    out = torch.empty(4, 192, device=dev)
    lib = awa_b200.library()
    # out_dim not a multiple of 128
    rc = lib.awa_out_project(4, 128, 192, x.data_ptr(), 128, w.data_ptr(), 128, v.data_ptr(), v.data_ptr(),
                             res.data_ptr(), 192, awa_b200.AWA_F32, awa_b200.AWA_F32, out.data_ptr(), 192, None)
    assert rc == awa_b200.AWA_ERR_INVALID and b"multiple of 128" in lib.awa_last_error()
    awa_b200.device_status()

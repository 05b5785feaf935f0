"""GPU parity of the AWA input's producer (awa_qkv_project: the block's QKV
projection with the per-head RMSNorm of Q and K) through the C ABI, against
the oracle restatement (oracle.qkv_project, pinned to FixedMMAttention's
modules in test_oracle.py) and against the reference fixture itself.

Tolerances: the kernel accumulates x W^T in a different order than the CPU,
so a few of the Linear's bf16 outputs round the other way; relative L2 within
5e-3 for both output dtypes (the bf16 block tolerance is 2e-2)."""

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
from oracle.oracle import qkv_project, round_bf16_rne  # noqa: E402

TOL = 5e-3


def _inputs(tokens, model_dim, heads, seed):
    rng = np.random.default_rng(seed)
    x = round_bf16_rne(rng.standard_normal((tokens, model_dim), dtype=np.float32))
    w = round_bf16_rne((rng.standard_normal((3 * heads * 128, model_dim)) * (1.0 / np.sqrt(model_dim)))
                       .astype(np.float32))
    gq = (1.0 + 0.25 * rng.standard_normal(128)).astype(np.float32)
    gk = (1.0 + 0.25 * rng.standard_normal(128)).astype(np.float32)
    return x, w, gq, gk


def _run(x, w, gq, gk, eps, heads, out_dtype):
    dev = torch.device("cuda")
    out = awa_b200.qkv_project(torch.from_numpy(x).to(dev, torch.bfloat16), torch.from_numpy(w).to(dev, torch.bfloat16),
                               torch.from_numpy(gq).to(dev), torch.from_numpy(gk).to(dev), eps, heads,
                               out_dtype=out_dtype)
    awa_b200.device_status()
    return out.float().cpu().numpy()


def test_reference_fixture():
    f = np.load(os.path.join(os.path.dirname(__file__), "golden", "qkv_project.npz"))
    got = _run(f["x"], f["w"], f["gamma_q"], f["gamma_k"], float(f["eps"]), int(f["heads"]), torch.bfloat16)
    assert rel_l2(got, f["out"]) < TOL


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
@pytest.mark.parametrize("tokens,model_dim,heads", [(300, 2560, 20), (128, 192, 3), (1, 64, 1), (58, 2560, 20)],
                         ids=["300x2560-h20", "128x192-h3", "1x64-h1", "text58-h20"])
def test_matches_oracle(tokens, model_dim, heads, out_dtype):
    x, w, gq, gk = _inputs(tokens, model_dim, heads, seed=tokens * 7 + heads)
    ref = qkv_project(x, w, gq, gk, 1e-5, heads)
    if out_dtype == torch.bfloat16:
        ref = round_bf16_rne(ref)
    got = _run(x, w, gq, gk, 1e-5, heads, out_dtype)
    assert got.shape == ref.shape
    assert rel_l2(got, ref) < TOL
    # V heads are the Linear's output, rounded to bf16: all but a few exact
    assert np.mean(got[:, 2] == ref[:, 2]) > 0.99


def test_rejects_bad_arguments():
    dev = torch.device("cuda")
    x = torch.zeros(4, 64, dtype=torch.bfloat16, device=dev)
    w = torch.zeros(384, 64, dtype=torch.bfloat16, device=dev)
    g = torch.ones(128, device=dev)
    out = torch.empty(4, 384, dtype=torch.bfloat16, device=dev)
    lib = awa_b200.library()
    # head_dim other than 128
    rc = lib.awa_qkv_project(4, 64, 1, 64, x.data_ptr(), 64, w.data_ptr(), 64, g.data_ptr(), g.data_ptr(), 1e-5,
                             awa_b200.AWA_BF16, out.data_ptr(), 384, None)
    assert rc == awa_b200.AWA_ERR_INVALID and b"head_dim" in lib.awa_last_error()
    # output rows not 32-byte aligned
    rc = lib.awa_qkv_project(4, 64, 1, 128, x.data_ptr(), 64, w.data_ptr(), 64, g.data_ptr(), g.data_ptr(), 1e-5,
                             awa_b200.AWA_BF16, out.data_ptr() + 2, 384, None)
    assert rc == awa_b200.AWA_ERR_INVALID
    awa_b200.device_status()

"""RoPE in the producer's epilogue: awa_qkv_project_rotated and
awa_forward_prerotated through the C ABI.

The reference rotates Q and K in its MMRoPE layer (awa_layers.cpp:867-953) on
the fp32 output of DitRMSNorm (src/dit/dit_precision.cpp:22-90), with
window-local coordinates that depend on the block's window layout (its
shift). awa_qkv_project_rotated applies that rotation in the QKV projection's
epilogue, in fp32 after the RMSNorm, with each token's coordinates from the
block's AWA plan, and rounds once; awa_forward_prerotated then attends
without rotating. Checks:

* fp32 output: bit-identical to awa_qkv_project's fp32 output rotated by the
  oracle's MMRoPE (the reference's own rotation, pinned bit-exact) with each
  token's table row -- video tokens through the plan's index maps, text tokens
  at (i, i, i);
* bf16 output: the same values rounded once (bit-identical);
* awa_forward_prerotated on those rows against the oracle's whole chain on the
  unrotated fp32 rows (2e-2, bf16 tensor cores; 1e-5 with fp32 rows on the
  fp32 kernel), for an unshifted and a shifted layer.
"""

import numpy as np
import pytest

from awa_testlib import BF16_REL_L2, FP32_REL_L2, rel_l2
from oracle.oracle import LayerConfig

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import awa_b200  # noqa: E402
from awa_b200 import AWA_BRANCH_TEXT, AWA_BRANCH_VIDEO, AWA_PREC_BF16, AWA_PREC_FP32  # noqa: E402

HEADS, DIM, EPS = 20, 2560, 1e-5


def _weights(seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn(3 * DIM, DIM, device="cuda", generator=g) * DIM ** -0.5).bfloat16()
    gq = 1.0 + 0.25 * torch.randn(128, device="cuda", generator=g)
    gk = 1.0 + 0.25 * torch.randn(128, device="cuda", generator=g)
    return g, w, gq, gk


def _table_rows(oracle, cfg, maps):
    """Each source token's MMRoPE table row (video: through its packed
    position; text token i: the row of window 0's text token i)."""
    table = oracle.rope_table(cfg)
    cu = maps["cu_seqlens"]
    video_rows = table[maps["video_positions"]]
    text_rows = table[cu[1] - cfg.text_tokens + np.arange(cfg.text_tokens)]
    return video_rows, text_rows


@pytest.mark.parametrize("shifted", [0, 1], ids=["unshifted", "shifted"])
def test_rotated_projection_is_the_reference_rotation(oracle, shifted):
    cfg = LayerConfig(6, 16, 16, 2, 8, 8, shifted=shifted, heads=HEADS)
    plan = awa_b200.AwaPlan(*cfg.params[:6], text_tokens=cfg.text_tokens, shifted=bool(shifted))
    g, w, gq, gk = _weights(11 + shifted)
    video_rows, text_rows = _table_rows(oracle, cfg, plan.maps())
    for branch, tokens, rows in ((AWA_BRANCH_VIDEO, cfg.source_tokens, video_rows),
                                 (AWA_BRANCH_TEXT, cfg.text_tokens, text_rows)):
        x = torch.randn(tokens, DIM, device="cuda", generator=g).bfloat16()
        plain = awa_b200.qkv_project(x, w, gq, gk, EPS, HEADS, out_dtype=torch.float32)
        rot32 = awa_b200.qkv_project_rotated(x, w, gq, gk, EPS, HEADS, plan, branch, out_dtype=torch.float32)
        rot16 = awa_b200.qkv_project_rotated(x, w, gq, gk, EPS, HEADS, plan, branch, out_dtype=torch.bfloat16)
        torch.cuda.synchronize()
        awa_b200.device_status()
        want = oracle.rope(plain.cpu().numpy(), rows, HEADS, 128, cfg.rope_dim)
        assert np.array_equal(rot32.cpu().numpy(), want), branch
        assert torch.equal(rot16, rot32.bfloat16()), branch


@pytest.mark.parametrize("precision", ["bf16", "fp32"])
@pytest.mark.parametrize("shifted", [0, 1], ids=["unshifted", "shifted"])
def test_prerotated_forward_matches_the_oracle_chain(oracle, shifted, precision):
    bf16 = precision == "bf16"
    cfg = LayerConfig(6, 16, 16, 2, 8, 8, shifted=shifted, heads=HEADS)
    plan = awa_b200.AwaPlan(*cfg.params[:6], text_tokens=cfg.text_tokens, shifted=bool(shifted))
    g, w, gq, gk = _weights(21 + shifted)
    xv = torch.randn(cfg.source_tokens, DIM, device="cuda", generator=g).bfloat16()
    xt = torch.randn(cfg.text_tokens, DIM, device="cuda", generator=g).bfloat16()
    dt = torch.bfloat16 if bf16 else torch.float32
    qv = awa_b200.qkv_project_rotated(xv, w, gq, gk, EPS, HEADS, plan, AWA_BRANCH_VIDEO, out_dtype=dt)
    qt = awa_b200.qkv_project_rotated(xt, w, gq, gk, EPS, HEADS, plan, AWA_BRANCH_TEXT, out_dtype=dt)
    prec = AWA_PREC_BF16 if bf16 else AWA_PREC_FP32
    video, text = plan.forward_prerotated(qv, qt, prec, out_dtype=torch.float32)
    # the oracle rotates the unrotated fp32 rows itself
    pv = awa_b200.qkv_project(xv, w, gq, gk, EPS, HEADS, out_dtype=torch.float32)
    pt = awa_b200.qkv_project(xt, w, gq, gk, EPS, HEADS, out_dtype=torch.float32)
    torch.cuda.synchronize()
    awa_b200.device_status()
    ref = oracle.chain(cfg, pv.cpu().numpy(), pt.cpu().numpy())
    tol = BF16_REL_L2 if bf16 else FP32_REL_L2
    assert rel_l2(video.cpu().numpy(), ref["video"]) < tol
    assert rel_l2(text.cpu().numpy(), ref["text"]) < tol
    if bf16:
        # one rounding fewer than rotating bf16 rows on the fly
        video_fly, text_fly = plan.forward(pv.bfloat16(), pt.bfloat16(), prec, out_dtype=torch.float32)
        torch.cuda.synchronize()
        assert rel_l2(video.cpu().numpy(), ref["video"]) <= rel_l2(video_fly.cpu().numpy(), ref["video"]) * 1.05


def test_rotated_projection_rejects_a_mismatched_branch():
    plan = awa_b200.AwaPlan(6, 16, 16, 2, 8, 8)
    g, w, gq, gk = _weights(5)
    x = torch.randn(100, DIM, device="cuda", generator=g).bfloat16()
    with pytest.raises(awa_b200.AwaError, match="video branch has 1536"):
        awa_b200.qkv_project_rotated(x, w, gq, gk, EPS, HEADS, plan, AWA_BRANCH_VIDEO)

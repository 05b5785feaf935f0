"""Parity at BASELINE's full sizes, where the naive oracle cannot run the whole
layer in seconds:

* index maps of the full configuration are bit-exact (CPU test in
  test_library_host.py);
* Pack and MMRoPE are bit-exact over the full layer (checked here by hashing
  against the oracle's per-window restatement on sampled windows);
* attention of sampled windows (a full one, a short one, edge windows of the
  shifted layer) against the oracle run on exactly those windows;
* the fused chain against the layer-by-layer chain over the whole layer
  (video rows and the text mean over all windows).
"""

import numpy as np
import pytest

from awa_testlib import BF16_REL_L2, FP32_REL_L2, plan_for, rel_l2, to_host
from oracle.oracle import LayerConfig

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import awa_b200  # noqa: E402
from awa_b200 import AWA_PREC_BF16, AWA_PREC_FP32  # noqa: E402

FULL = [
    ("cfg4", LayerConfig(21, 64, 64, 6, 8, 8, shifted=0), AWA_PREC_BF16),
    ("cfg4-shifted", LayerConfig(21, 64, 64, 6, 8, 8, shifted=1), AWA_PREC_BF16),
    ("cfg5-fp32-shifted", LayerConfig(9, 45, 80, 3, 6, 10, shifted=1), AWA_PREC_FP32),
]


def sample_windows(cu: np.ndarray):
    lengths = np.diff(cu)
    count = len(lengths)
    picks = {0, count - 1, int(np.argmax(lengths)), int(np.argmin(lengths)), count // 2}
    return sorted(picks)


@pytest.mark.parametrize("name,cfg,precision", FULL, ids=[f[0] for f in FULL])
def test_full_layer(name, cfg, precision, oracle):
    gen = torch.Generator(device="cuda").manual_seed(0)
    dtype = torch.bfloat16 if precision == AWA_PREC_BF16 else torch.float32
    v = torch.randn(cfg.source_tokens, 3, cfg.heads, cfg.head_dim, device="cuda", generator=gen).to(dtype)
    t = torch.randn(cfg.text_tokens, 3, cfg.heads, cfg.head_dim, device="cuda", generator=gen).to(dtype)
    plan = plan_for(cfg)
    maps = plan.maps()
    cu = maps["cu_seqlens"]

    # Layer chain in fp32 (Pack, MMRoPE bit-exact; fp32 attention).
    packed32, _ = plan.pack(v.float(), t.float())
    roped32 = plan.mmrope(packed32)

    # Sampled windows: oracle Pack + MMRoPE + attention on exactly those windows.
    table = oracle.rope_table(cfg)
    video, _ = plan.forward(v, t, precision, out_dtype=torch.float32)
    tol = BF16_REL_L2 if precision == AWA_PREC_BF16 else FP32_REL_L2
    for w in sample_windows(cu):
        rows = np.arange(cu[w], cu[w + 1])
        seq = maps["sequence_index"][rows]
        seq_t = torch.from_numpy(seq.astype(np.int64)).cuda()
        is_video = seq_t < cfg.source_tokens
        src = torch.empty(len(rows), 3, cfg.heads, cfg.head_dim, device="cuda")
        src[is_video] = v[seq_t[is_video]].float()
        src[~is_video] = t[seq_t[~is_video] - cfg.source_tokens].float()
        packed_w = np.ascontiguousarray(to_host(src))
        assert np.array_equal(to_host(packed32[cu[w]:cu[w + 1]]), packed_w)
        roped_w = oracle.rope(packed_w, table[rows], cfg.heads, cfg.head_dim, cfg.rope_dim)
        assert np.array_equal(to_host(roped32[cu[w]:cu[w + 1]]), roped_w)
        att_w = np.empty((len(rows), cfg.heads, cfg.head_dim), np.float32)
        oracle.attention_range(roped_w, np.array([0, len(rows)], np.int32), 0, 1, cfg.heads, cfg.head_dim, att_w,
                               threads=8)
        vrows = seq[seq < cfg.source_tokens]
        ours = to_host(video[torch.from_numpy(vrows.astype(np.int64)).cuda()])
        assert rel_l2(ours, att_w[: len(vrows)]) < tol, (name, w)

    # Whole layer: fused chain == layer chain (same precision), video and text.
    attended = plan.window_attention(roped32.to(dtype), precision, out_dtype=torch.float32)
    video_l, text_l = plan.unpack(attended)
    video_f, text_f = plan.forward(v, t, precision, out_dtype=torch.float32)
    tol = 1e-2 if precision == AWA_PREC_BF16 else 1e-6
    assert rel_l2(to_host(video_f), to_host(video_l)) < tol
    assert rel_l2(to_host(text_f), to_host(text_l)) < tol
    awa_b200.device_status()


def test_sharded_windows_reassemble_the_layer():
    """awa_forward_windows over a 4-way partition + text finalize == awa_forward."""
    cfg = LayerConfig(6, 16, 16, 2, 8, 8, shifted=1)
    gen = torch.Generator(device="cuda").manual_seed(1)
    v = torch.randn(cfg.source_tokens, 3, cfg.heads, cfg.head_dim, device="cuda", generator=gen).bfloat16()
    t = torch.randn(cfg.text_tokens, 3, cfg.heads, cfg.head_dim, device="cuda", generator=gen).bfloat16()
    plan = plan_for(cfg)
    video_ref, text_ref = plan.forward(v, t, AWA_PREC_BF16, out_dtype=torch.float32)
    bounds = plan.partition(4)
    video = torch.full_like(video_ref, float("nan"))
    total = torch.zeros(cfg.text_tokens, cfg.heads, cfg.head_dim, device="cuda")
    for b0, b1 in zip(bounds, bounds[1:]):
        part = torch.empty_like(total)
        plan.forward_windows(v, t, b0, b1, video, part, AWA_PREC_BF16)
        total += part
        # shard round trip: gather this range's rows into a dense shard and back
        shard = torch.empty(plan.range_video_rows(b0, b1), cfg.heads, cfg.head_dim, device="cuda")
        plan.gather_video_shard(video, b0, b1, shard)
        other = torch.zeros_like(video)
        plan.scatter_video_shard(shard, b0, b1, other)
        rows = torch.from_numpy(np.concatenate([np.zeros(0, np.int64)] + [
            np.array(plan.maps()["sequence_index"][plan.maps()["cu_seqlens"][w]:plan.maps()["cu_seqlens"][w + 1] - cfg.text_tokens], np.int64)
            for w in range(b0, b1)])).cuda()
        assert torch.equal(other[rows], video[rows])
    assert torch.equal(video, video_ref)
    text = plan.text_finalize(total, torch.float32)
    assert rel_l2(to_host(text), to_host(text_ref)) < 1e-6
    awa_b200.device_status()

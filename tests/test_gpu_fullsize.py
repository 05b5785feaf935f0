"""Parity at BASELINE's full sizes, where the naive oracle cannot run the whole
layer in seconds:

* index maps of the full configuration are bit-exact (CPU test in
  test_library_host.py);
* Pack and MMRoPE are bit-exact over the full layer (checked here by hashing
  against the oracle's per-window restatement on sampled windows);
* attention of at least 16 sampled windows -- one of every window shape
  (each clipped edge class of the shifted and non-divisible layers), the
  longest and shortest, and windows spread over the layer -- against the
  oracle run on exactly those windows: video rows and each window's text rows;
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
    # BASELINE's "1344 windows": 1x8x8 windows of the same grid
    ("cfg4b", LayerConfig(21, 64, 64, 21, 8, 8, shifted=0), AWA_PREC_BF16),
    ("cfg4b-shifted", LayerConfig(21, 64, 64, 21, 8, 8, shifted=1), AWA_PREC_BF16),
    # adaptive windows on 9x45x80 (3x8x8, 3x5x8 at the bottom edge)
    ("cfg5", LayerConfig(9, 45, 80, 3, 6, 10, shifted=0), AWA_PREC_BF16),
    ("cfg5-shifted", LayerConfig(9, 45, 80, 3, 6, 10, shifted=1), AWA_PREC_BF16),
    ("cfg5-fp32", LayerConfig(9, 45, 80, 3, 6, 10, shifted=0), AWA_PREC_FP32),
    ("cfg5-fp32-shifted", LayerConfig(9, 45, 80, 3, 6, 10, shifted=1), AWA_PREC_FP32),
]

MIN_SAMPLES = 16


def sample_windows(windows, cu: np.ndarray):
    """At least MIN_SAMPLES windows: one of every window shape (each clipped
    edge class of a shifted or non-divisible layer), the first, last, longest
    and shortest, then windows spread evenly over the list."""
    count = len(windows)
    lengths = np.diff(cu)
    picks = {0, count - 1, int(np.argmax(lengths)), int(np.argmin(lengths))}
    shapes = {}
    for i, (t0, t1, h0, h1, w0, w1) in enumerate(windows):
        shapes.setdefault((t1 - t0, h1 - h0, w1 - w0), i)
    picks.update(shapes.values())
    step = max(1, count // MIN_SAMPLES)
    i = step // 2
    while len(picks) < min(MIN_SAMPLES, count):
        picks.add(i % count)
        i += step
    return sorted(picks), len(shapes)


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

    # Sampled windows: oracle Pack + MMRoPE + attention on exactly those windows,
    # against the fused chain's video rows and its per-window text rows (the
    # text partials it leaves in the workspace, in window order).
    table = oracle.rope_table(cfg)
    workspace = torch.empty(plan.workspace_bytes(cfg.heads, cfg.head_dim), dtype=torch.uint8, device="cuda")
    video, _ = plan.forward(v, t, precision, out_dtype=torch.float32, workspace=workspace)
    torch.cuda.synchronize()
    tc = plan.attention_kernel_kind(precision, cfg.heads, cfg.head_dim, dtype) == 1
    rows_per_window = cfg.text_tokens * cfg.heads * cfg.head_dim
    partials = (workspace.view(torch.bfloat16) if tc else workspace.view(torch.float32))[
        : plan.info.window_count * rows_per_window].view(plan.info.window_count, cfg.text_tokens, cfg.heads,
                                                          cfg.head_dim)
    tol = BF16_REL_L2 if precision == AWA_PREC_BF16 else FP32_REL_L2
    picks, shapes = sample_windows(maps["windows"], cu)
    assert len(picks) >= min(MIN_SAMPLES, len(cu) - 1) and shapes >= 1
    for w in picks:
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
        assert rel_l2(ours, att_w[: len(vrows)]) < tol, (name, w, "video")
        assert rel_l2(to_host(partials[w]), att_w[len(vrows):]) < tol, (name, w, "text")

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

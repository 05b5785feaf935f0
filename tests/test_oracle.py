"""Pin the C oracle (oracle/awa_oracle.c) before it is trusted as the checker.

* against the golden vectors written by the reference's PyTorch mirror
  (tests/golden/make_golden.py), and
* against the reference's own awa_layers.cpp CPU forward compiled unmodified
  (oracle/_ref), bit for bit.
"""

import hashlib
import json
import os

import numpy as np
import pytest

from oracle.oracle import LayerConfig

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _sha(array) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


def _rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


with open(os.path.join(GOLDEN, "windows.json")) as _f:
    WINDOW_CASES = json.load(_f)["cases"]


@pytest.mark.parametrize("case", WINDOW_CASES, ids=lambda c: f"{c['size']}-{c['num_windows']}-s{int(c['shifted'])}")
def test_windows_and_index_maps_match_python_reference(oracle, case):
    size, num, shifted = case["size"], case["num_windows"], case["shifted"]
    windows = oracle.make_windows(size, num, shifted)
    assert [list(w) for w in windows] == case["windows"]
    cfg = LayerConfig(*size, *num, text_tokens=case["text_tokens"], shifted=int(shifted))
    maps = oracle.index_maps(cfg)
    # awa_round_trip's target map = sequence_index without the text entries (int64 bytes).
    source_tokens = cfg.source_tokens
    seq = maps["sequence_index"].astype(np.int64)
    target = seq[seq < source_tokens]
    assert _sha(target) == case["target_index_sha256"]
    assert _sha(np.argsort(target, kind="stable")) == case["reverse_index_sha256"]
    assert _sha(seq) == case["sequence_index_int64_sha256"]
    assert _sha(maps["text_positions"].astype(np.int64)) == case["text_positions_int64_sha256"]
    # The Python mirror's video_positions are packed positions in partition order.
    vpos_partition = maps["video_positions"].astype(np.int64)[target]
    assert _sha(vpos_partition) == case["video_positions_int64_sha256"]
    assert maps["cu_seqlens"].tolist() == case["cu_seqlens"]


CHAIN_FILES = sorted(f for f in os.listdir(GOLDEN) if f.startswith("chain_") and f.endswith(".npz"))


@pytest.mark.parametrize("name", CHAIN_FILES)
def test_chain_matches_python_reference(oracle, name):
    g = np.load(os.path.join(GOLDEN, name))
    size = [int(v) for v in g["size"]]
    num = [int(v) for v in g["num_windows"]]
    cfg = LayerConfig(*size, *num, text_tokens=int(g["text_tokens"]), shifted=int(g["shifted"]),
                      heads=int(g["heads"]), head_dim=int(g["head_dim"]))
    out = oracle.chain(cfg, g["video_qkv"], g["text_qkv"], threads=2)
    # Integer / copy work is bit-exact.
    assert _sha(out["packed"]) == str(g["packed_fp32_sha256"])
    assert np.array_equal(out["cu_seqlens"], g["cu_seqlens"].astype(np.float32))
    # fp32 arithmetic: the Python mirror computes the RoPE angles with torch
    # (not powf/cosf/sinf) and softmax/matmul in another order, so only the
    # reference's fp32 tolerance (dit_block.py:28-29: 2e-4) can hold; the
    # observed differences are ~1e-7.
    rows = g["rope_positions"]
    assert _rel_l2(out["roped"][rows, :2], g["roped_qk"]) < 1e-6
    assert _rel_l2(out["attended"], g["attended"]) < 1e-6
    assert _rel_l2(out["video"], g["video"]) < 1e-6
    assert _rel_l2(out["text"], g["text"]) < 1e-6
    np.testing.assert_allclose(out["video"], g["video"], atol=2e-4, rtol=2e-4)
    np.testing.assert_allclose(out["text"], g["text"], atol=2e-4, rtol=2e-4)


REF_WINDOW_GRID = [(1, 16, 16), (6, 16, 16), (21, 64, 64), (9, 45, 80), (2, 19, 23), (1, 45, 80), (3, 7, 11),
                   (40, 9, 13), (1, 1, 1), (7, 3, 29)]
REF_WINDOW_NUMS = [(1, 8, 8), (2, 8, 8), (6, 8, 8), (3, 6, 10), (4, 3, 3), (21, 8, 8), (1, 1, 1), (5, 3, 7)]


def test_windows_match_compiled_reference(oracle, reference):
    for size in REF_WINDOW_GRID:
        for num in REF_WINDOW_NUMS:
            for shifted in (False, True):
                assert oracle.make_windows(size, num, shifted) == reference.make_windows(size, num, shifted)


def test_random_windows_match_compiled_reference(oracle, reference):
    rng = np.random.default_rng(7)
    for _ in range(300):
        size = tuple(int(v) for v in rng.integers(1, [40, 90, 120]))
        num = tuple(int(v) for v in rng.integers(1, [8, 12, 12]))
        shifted = bool(rng.integers(0, 2))
        assert oracle.make_windows(size, num, shifted) == reference.make_windows(size, num, shifted)


REF_CHAIN_CASES = [
    LayerConfig(2, 5, 7, 2, 2, 3, text_tokens=3, shifted=1, heads=2, head_dim=8, rope_dim=6),
    LayerConfig(2, 19, 23, 4, 3, 3, text_tokens=5, shifted=0, heads=2, head_dim=3, rope_dim=0),
    LayerConfig(1, 16, 16, 1, 8, 8, text_tokens=58, shifted=0, heads=2, head_dim=128),
    LayerConfig(1, 16, 16, 1, 8, 8, text_tokens=58, shifted=1, heads=2, head_dim=128),
    LayerConfig(3, 9, 10, 2, 2, 3, text_tokens=7, shifted=1, heads=3, head_dim=12, rope_dim=12),
]


@pytest.mark.parametrize("cfg", REF_CHAIN_CASES, ids=lambda c: f"{c.source_t}x{c.source_h}x{c.source_w}-s{c.shifted}")
@pytest.mark.parametrize("layout", [0, 1, 2])
def test_chain_bitexact_with_compiled_reference(oracle, reference, cfg, layout):
    if cfg.rope_dim == 0:
        pytest.skip("rope_dim 0 is rejected by the reference MMRoPE (awa_layers.cpp:873)")
    rng = np.random.default_rng(cfg.source_tokens + layout)
    v = rng.standard_normal((cfg.source_tokens, 3, cfg.heads, cfg.head_dim), dtype=np.float32)
    t = rng.standard_normal((cfg.text_tokens, 3, cfg.heads, cfg.head_dim), dtype=np.float32)
    ours = oracle.chain(cfg, v, t, threads=2)
    ref = reference.chain(cfg, v, t, layout=layout, runtime_spec=(layout == 1))
    for key in ("packed", "cu_seqlens", "roped", "attended", "video", "text"):
        assert np.array_equal(ours[key], ref[key]), key


@pytest.mark.parametrize("cfg", [c for c in REF_CHAIN_CASES if c.rope_dim and c.head_dim < 128] + REF_CHAIN_CASES[3:4],
                         ids=lambda c: f"{c.source_t}x{c.source_h}x{c.source_w}-s{c.shifted}")
def test_ncnn_batch_reference_build(oracle, cfg):
    """The reference compiled with NCNN_BATCH=1 (describe_qkv_layout's c=3,
    n=N branch, awa_layers.cpp:142-149; the 4-D batched video output of
    :655-656 and :668-670): on the batched QKV encoding it gives the same values
    as the C restatement, and on the other encodings too."""
    from oracle.oracle import REF_BATCH_SO, Reference

    if not Reference.available(REF_BATCH_SO):
        pytest.skip("oracle/_ref/libawa_ref_batch.so not built")
    ref = Reference(REF_BATCH_SO)
    assert ref.batch_build
    rng = np.random.default_rng(11 + cfg.source_tokens)
    v = rng.standard_normal((cfg.source_tokens, 3, cfg.heads, cfg.head_dim), dtype=np.float32)
    t = rng.standard_normal((cfg.text_tokens, 3, cfg.heads, cfg.head_dim), dtype=np.float32)
    ours = oracle.chain(cfg, v, t, threads=2)
    for layout in (3, 0):
        got = ref.chain(cfg, v, t, layout=layout)
        for key in ("packed", "cu_seqlens", "roped", "attended", "video", "text"):
            assert np.array_equal(ours[key], got[key]), (layout, key)


def test_reference_rejects_bad_rope_dim(reference):
    handle, status = reference.create(LayerConfig(1, 4, 4, 1, 2, 2, text_tokens=2, rope_dim=125, heads=1, head_dim=128))
    assert not handle and status == -1


def test_round_bf16_is_rne(oracle):
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, 1e-40], np.float32)
    r = oracle.round_bf16(x)
    bits = r.view(np.uint32)
    assert np.all(bits & 0xFFFF == 0)
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == np.float32(1.015625)


def test_qkv_project_oracle_matches_reference_fixture():
    """The producer's restatement against FixedMMAttention's own proj_qkv +
    norm_q / norm_k run (tests/golden/qkv_project.npz, tokens 70, model_dim 160,
    2 heads). The PyTorch mirror rounds the RMSNorm output to bf16 (its input
    is bf16); the oracle keeps fp32 as DitRMSNorm does, so it is compared after
    the same rounding: all but a few values equal (the two CPU Linears and the
    RMSNorm sums add in different orders)."""
    from oracle.oracle import qkv_project, round_bf16_rne

    f = np.load(os.path.join(os.path.dirname(__file__), "golden", "qkv_project.npz"))
    out = qkv_project(f["x"], f["w"], f["gamma_q"], f["gamma_k"], float(f["eps"]), int(f["heads"]))
    ref = f["out"]
    assert out.shape == ref.shape
    rounded = round_bf16_rne(out)
    # all but a few values bit-equal; the rest are sums that round the other way
    # (near-cancelling dot products move by more than one ulp of their value)
    assert int((rounded != ref).sum()) <= ref.size // 1000
    assert float(np.linalg.norm(rounded - ref) / np.linalg.norm(ref)) < 1e-5


def test_out_project_oracle_matches_reference_fixture():
    """The consumer's restatement against FixedDitBlock's own proj_out, Ada
    "out" gate and residual run (tests/golden/out_project.npz, tokens 70,
    256 -> 256): bit-exact."""
    from oracle.oracle import out_project

    f = np.load(os.path.join(os.path.dirname(__file__), "golden", "out_project.npz"))
    out = out_project(f["x"], f["w"], f["bias"], f["gate"], f["residual"])
    assert np.array_equal(out, f["out"])

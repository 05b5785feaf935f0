"""Host-side checks of the B200 library that need no GPU.

* the C-ABI libraries load and export every entry point include/*.h declares;
* the window rule and every index map of a plan are bit-identical to the oracle
  (which is itself pinned to the reference);
* load_param's error behaviour (invalid params, -1,-1,-1 grid with/without a
  runtime spec, rope_dim) and the forward calls' rejection of a host-only plan.
"""

import ctypes
import json
import os
import re

import numpy as np
import pytest

import awa_b200
from oracle.oracle import LayerConfig

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", h) for h in ("awa_b200.h", "awa_package.h", "awa_stack.h")]
GOLDEN = os.path.join(ROOT, "tests", "golden")


def declared_functions():
    text = "".join(open(h).read() for h in HEADERS)
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(awa_\w+)\s*\(", text)))


def test_header_and_binding_agree():
    assert sorted(awa_b200.EXPORTED_SYMBOLS) == declared_functions()


def test_library_exports_every_declared_symbol():
    lib = awa_b200.library()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert b"sm_100a" in lib.awa_version()


@pytest.mark.parametrize("batch", [False, True], ids=["plain", "ncnn-batch"])
def test_ncnn_compat_library_loads(batch):
    lib = awa_b200.ncnn_compat(batch)
    assert hasattr(lib, "awa_ncnn_run_chain")
    assert lib.awa_ncnn_batch_build() == int(batch)


with open(os.path.join(GOLDEN, "windows.json")) as _f:
    GOLDEN_CASES = json.load(_f)["cases"]


@pytest.mark.parametrize("case", GOLDEN_CASES, ids=lambda c: f"{c['size']}-{c['num_windows']}-s{int(c['shifted'])}")
def test_make_windows_matches_golden(case):
    windows = awa_b200.make_windows(case["size"], case["num_windows"], case["shifted"])
    assert [list(w) for w in windows] == case["windows"]


def test_random_windows_match_oracle(oracle):
    rng = np.random.default_rng(11)
    for _ in range(500):
        size = [int(v) for v in rng.integers(1, [48, 100, 130])]
        num = [int(v) for v in rng.integers(1, [9, 13, 13])]
        shifted = bool(rng.integers(0, 2))
        assert awa_b200.make_windows(size, num, shifted) == oracle.make_windows(size, num, shifted)


MAP_CASES = [
    LayerConfig(1, 16, 16, 1, 8, 8, shifted=0),
    LayerConfig(1, 16, 16, 1, 8, 8, shifted=1),
    LayerConfig(6, 16, 16, 2, 8, 8, shifted=1),
    LayerConfig(21, 64, 64, 6, 8, 8, shifted=0),
    LayerConfig(21, 64, 64, 6, 8, 8, shifted=1),
    LayerConfig(21, 64, 64, 21, 8, 8, shifted=1),
    LayerConfig(9, 45, 80, 3, 6, 10, shifted=0),
    LayerConfig(9, 45, 80, 3, 6, 10, shifted=1),
    LayerConfig(1, 45, 80, 4, 3, 3, shifted=1),
    LayerConfig(2, 19, 23, 4, 3, 3, text_tokens=5, shifted=1),
    LayerConfig(5, 2, 97, 2, 1, 9, text_tokens=1, shifted=1),
]


@pytest.mark.parametrize("cfg", MAP_CASES, ids=lambda c: f"{c.source_t}x{c.source_h}x{c.source_w}-{c.num_t}{c.num_h}{c.num_w}-s{c.shifted}")
def test_plan_maps_bitexact_with_oracle(oracle, cfg):
    plan = awa_b200.AwaPlan(*cfg.params[:6], text_tokens=cfg.text_tokens, shifted=cfg.shifted, host_only=True)
    ours = plan.maps()
    ref = oracle.index_maps(cfg)
    assert ours["windows"] == ref["windows"]
    for key in ("sequence_index", "cu_seqlens", "video_positions", "text_positions"):
        assert np.array_equal(ours[key], ref[key]), key
    info = plan.info
    assert info.window_count == len(ref["windows"])
    assert info.sequence_tokens == len(ref["sequence_index"])
    assert info.device == -1


def test_runtime_spec_grid():
    a = awa_b200.AwaPlan(-1, -1, -1, 1, 8, 8, runtime_spec=(1, 16, 16), host_only=True)
    b = awa_b200.AwaPlan(1, 16, 16, 1, 8, 8, host_only=True)
    for key in ("sequence_index", "cu_seqlens", "video_positions", "text_positions"):
        assert np.array_equal(a.maps()[key], b.maps()[key])
    with pytest.raises(awa_b200.AwaError) as err:
        awa_b200.AwaPlan(-1, -1, -1, 1, 8, 8, host_only=True)
    assert err.value.code == -1


@pytest.mark.parametrize("bad", [
    dict(source_t=0), dict(windows_h=0), dict(text_tokens=0), dict(rope_dim=125), dict(rope_dim=-6),
])
def test_invalid_params_rejected_like_load_param(bad):
    args = dict(source_t=1, source_h=16, source_w=16, windows_t=1, windows_h=8, windows_w=8, text_tokens=58,
                rope_dim=126)
    args.update(bad)
    with pytest.raises(awa_b200.AwaError) as err:
        awa_b200.AwaPlan(args["source_t"], args["source_h"], args["source_w"], args["windows_t"], args["windows_h"],
                         args["windows_w"], text_tokens=args["text_tokens"], rope_dim=args["rope_dim"], host_only=True)
    assert err.value.code == -1


def test_host_plan_rejects_forward_calls():
    lib = awa_b200.library()
    plan = awa_b200.AwaPlan(1, 16, 16, 1, 8, 8, host_only=True)
    rc = lib.awa_window_attention(plan.handle, 0, 20, 128, 0, 16, 7680, 0, 16, 2560, None)
    assert rc == -1
    assert b"without device tables" in lib.awa_last_error()


def test_partition_windows_covers_all_and_balances():
    plan = awa_b200.AwaPlan(21, 64, 64, 6, 8, 8, shifted=1, host_only=True)
    maps = plan.maps()
    lengths = np.diff(maps["cu_seqlens"]).astype(np.float64)
    for parts in (1, 2, 3, 4, 8):
        bounds = plan.partition(parts)
        assert bounds[0] == 0 and bounds[-1] == plan.info.window_count
        assert all(b0 <= b1 for b0, b1 in zip(bounds, bounds[1:]))
        costs = [float((lengths[b0:b1] ** 2).sum()) for b0, b1 in zip(bounds, bounds[1:])]
        assert max(costs) <= 1.1 * sum(costs) / parts + float((lengths ** 2).max())
    rows = sum(plan.range_video_rows(b0, b1) for b0, b1 in zip(bounds, bounds[1:]))
    assert rows == plan.info.source_tokens


def test_workspace_size():
    plan = awa_b200.AwaPlan(21, 64, 64, 6, 8, 8, host_only=True)
    assert plan.workspace_bytes(20, 128) == 384 * 58 * 20 * 128 * 4

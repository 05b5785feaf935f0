"""Two-rank (gloo, CPU) test of the multi-GPU protocol of awa_forward_sharded.

On GPUs the split comes from awa_shard_split / awa_shard_windows. With enough
windows, rank r computes the windows of its bands (runs of whole grid lines:
its video rows + an unnormalised fp32 text partial sum), the ranks all-reduce
the partial, divide by the window count and exchange the video rows. With fewer than 4
windows per rank, rank r computes every window for heads [bounds[r],
bounds[r+1)) and the ranks all-gather the head slices. Here each rank runs the
same protocol on the CPU with the oracle standing in for the kernels: the
split comes from the library's host-side plan, the exchange is a real gloo
all-reduce / all-gather between two processes, and the result must equal the
single-process reference chain (video rows bit-exact, text within the fp32
tolerance: the cross-rank sum adds in a different order).
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from awa_testlib import FP32_REL_L2, rel_l2

CASES = [
    # grid, window counts, shifted, heads, head_dim, text tokens
    ((2, 45, 80), (1, 3, 4), True, 2, 16, 6),
    ((3, 12, 20), (2, 3, 4), False, 2, 32, 5),
    # 3 windows on 2 ranks: split by heads
    ((1, 12, 20), (1, 1, 3), False, 5, 12, 4),
]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _config(case):
    from oracle.oracle import LayerConfig

    grid, num, shifted, heads, head_dim, text = case
    return LayerConfig(*grid, *num, text_tokens=text, shifted=int(shifted), rope_dim=6 * (head_dim // 6) if
                       head_dim < 126 else 126, heads=heads, head_dim=head_dim)


def _inputs(cfg):
    rng = np.random.default_rng(11)
    v = rng.standard_normal((cfg.source_tokens, 3, cfg.heads, cfg.head_dim), dtype=np.float32)
    t = rng.standard_normal((cfg.text_tokens, 3, cfg.heads, cfg.head_dim), dtype=np.float32)
    return v, t


def _rank_main(rank: int, world: int, port: int, case, result_dir: str):
    import torch
    import torch.distributed as dist

    import awa_b200
    from oracle.oracle import Oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = _config(case)
        oracle = Oracle()
        v, t = _inputs(cfg)
        h, d, text = cfg.heads, cfg.head_dim, cfg.text_tokens
        plan = awa_b200.AwaPlan(*cfg.params[:6], text_tokens=text, shifted=bool(cfg.shifted), rope_dim=cfg.rope_dim,
                                host_only=True)
        by_heads, bounds = plan.shard_split(world, h)
        assert by_heads == (plan.info.window_count < 4 * world)
        begin, end = bounds[rank], bounds[rank + 1]
        W = plan.info.window_count
        maps = oracle.index_maps(cfg)
        seq = maps["sequence_index"]
        cu = maps["cu_seqlens"].astype(np.int32)
        packed = v.reshape(cfg.source_tokens, -1)[np.minimum(seq, cfg.source_tokens - 1)].reshape(-1, 3, h, d).copy()
        is_text = seq >= cfg.source_tokens
        packed[is_text] = t[seq[is_text] - cfg.source_tokens]
        roped = oracle.rope(packed, oracle.rope_table(cfg), h, d, cfg.rope_dim)
        video = np.zeros((cfg.source_tokens, h, d), np.float32)
        owned = np.zeros((cfg.source_tokens, h), np.int32)
        if by_heads:
            # every window, heads [begin, end): the same math on a head slice
            hn = end - begin
            sub = np.ascontiguousarray(roped[:, :, begin:end])
            att = np.zeros((len(seq), hn, d), np.float32)
            if hn:
                oracle.attention_range(sub, cu, 0, W, hn, d, att)
            attended = np.zeros((len(seq), h, d), np.float32)
            attended[:, begin:end] = att
            windows = range(W)
        else:
            # this rank's bands: the windows awa_shard_windows names
            windows = plan.shard_windows(world, h, rank)
            assert len(windows) == end - begin and windows == sorted(windows)
            attended = np.zeros((len(seq), h, d), np.float32)
            for w in windows:
                oracle.attention_range(roped, cu, w, w + 1, h, d, attended)
        heads_owned = slice(begin, end) if by_heads else slice(0, h)
        partial = np.zeros((text, h, d), np.float32)
        for w in windows:
            rows = np.arange(cu[w], cu[w + 1] - text)
            video[seq[rows]] = attended[rows]
            owned[seq[rows], heads_owned] += 1
            partial += attended[cu[w + 1] - text:cu[w + 1]]  # window order, fp32
        if not by_heads:
            assert int(owned[:, 0].sum()) == sum(plan.range_video_rows(w, w + 1) for w in windows)
        # awa_shard_runs: exactly the video rows these windows read and write
        runs = plan.shard_runs(world, h, rank)
        covered = np.zeros(cfg.source_tokens, np.int32)
        for first, count in runs:
            assert count > 0
            covered[first:first + count] += 1
        assert covered.max(initial=0) <= 1
        np.testing.assert_array_equal(covered, (owned[:, 0] > 0) if not by_heads else np.ones_like(covered))
        # the exchange: all-reduce of the partials (a head split's are disjoint),
        # all-gather of the video rows
        total = torch.from_numpy(partial)
        dist.all_reduce(total, op=dist.ReduceOp.SUM)
        text_out = (total / np.float32(W)).numpy()
        gathered = [torch.zeros(cfg.source_tokens, h, d) for _ in range(world)]
        owners = [torch.zeros(cfg.source_tokens, h, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(video))
        dist.all_gather(owners, torch.from_numpy(owned))
        if rank == 0:
            count = sum(o.numpy() for o in owners)
            merged = sum(g.numpy() for g in gathered)
            np.savez(os.path.join(result_dir, "result.npz"), video=merged, text=text_out, count=count,
                     bounds=np.array(bounds), by_heads=by_heads)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", CASES, ids=lambda c: "x".join(map(str, c[0])) + ("s" if c[2] else ""))
def test_window_sharded_protocol_matches_single_process(case, tmp_path, oracle):
    import torch.multiprocessing as mp

    world = 2
    mp.spawn(_rank_main, args=(world, _free_port(), case, str(tmp_path)), nprocs=world, join=True)
    res = np.load(tmp_path / "result.npz")
    cfg = _config(case)
    v, t = _inputs(cfg)
    ref = oracle.chain(cfg, v, t)
    bounds = res["bounds"]
    last = cfg.heads if bool(res["by_heads"]) else len(ref["maps"]["windows"])
    assert bounds[0] == 0 and bounds[-1] == last and np.all(np.diff(bounds) > 0)
    assert np.all(res["count"] == 1), "every video token and head must be computed by exactly one rank"
    assert np.array_equal(res["video"], ref["video"])
    assert rel_l2(res["text"], ref["text"]) <= FP32_REL_L2

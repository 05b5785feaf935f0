"""One rank of the multi-GPU parity test (tests/test_gpu_sharded.py).

Run as `python tests/sharded_worker.py RANK WORLD STORE_FILE OUT_JSON`, one
process per GPU. Each rank builds the same seeded inputs, runs
awa_forward_sharded over an NCCL communicator (awa_comm_create, id handed out
over a gloo process group that meets through STORE_FILE, so no port can be
taken) and the single-GPU awa_forward on its own GPU, and writes what it
observed to OUT_JSON. Every rank takes the same collective steps whatever its
checks find; the test asserts on the JSON files.
"""

import datetime
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for _p in (ROOT, os.path.join(ROOT, "seedvr2-ncnn_b200"), os.path.join(ROOT, "tests")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import awa_b200  # noqa: E402
from awa_testlib import make_inputs, rel_l2  # noqa: E402
from oracle.oracle import LayerConfig, Oracle  # noqa: E402

BF16, FP32 = awa_b200.AWA_PREC_BF16, awa_b200.AWA_PREC_FP32

# name, layer, precision, check against the oracle's whole chain (small layers)
CASES = [
    ("cfg2-windows", LayerConfig(6, 16, 16, 2, 8, 8, shifted=0), BF16, True),
    ("cfg2-shifted-windows", LayerConfig(6, 16, 16, 2, 8, 8, shifted=1), BF16, True),
    ("cfg1-heads-bf16", LayerConfig(1, 16, 16, 1, 8, 8, shifted=0), BF16, True),
    ("cfg1-heads-fp32", LayerConfig(1, 16, 16, 1, 8, 8, shifted=0), FP32, True),
    ("cfg1-shifted-fp32", LayerConfig(1, 16, 16, 1, 8, 8, shifted=1), FP32, True),
    ("cfg5-fp32-shifted", LayerConfig(9, 45, 80, 3, 6, 10, shifted=1), FP32, False),
    ("cfg4", LayerConfig(21, 64, 64, 6, 8, 8, shifted=0), BF16, False),
]


def main(rank: int, world: int, store_file: str, out_path: str) -> None:
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"file://{store_file}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    box = [awa_b200.AwaComm.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    comm = awa_b200.AwaComm(box[0], world, rank)
    oracle = Oracle()
    results = {}
    for name, cfg, prec, check_oracle in CASES:
        bf16 = prec == BF16
        dtype = torch.bfloat16 if bf16 else torch.float32
        if check_oracle:
            v_np, t_np = make_inputs(cfg, 17, bf16, oracle)
            v = torch.from_numpy(v_np).cuda().to(dtype)
            t = torch.from_numpy(t_np).cuda().to(dtype)
        else:
            gen = torch.Generator(device="cuda").manual_seed(23)  # same draws on every rank
            v = torch.randn(cfg.source_tokens, 3, cfg.heads, cfg.head_dim, device="cuda", generator=gen).to(dtype)
            t = torch.randn(cfg.text_tokens, 3, cfg.heads, cfg.head_dim, device="cuda", generator=gen).to(dtype)
        plan = awa_b200.AwaPlan(*cfg.params[:6], text_tokens=cfg.text_tokens, shifted=cfg.shifted)
        by_heads, bounds = plan.shard_split(world, cfg.heads)
        video_s, text_s = plan.forward_sharded(comm, v, t, prec, out_dtype=torch.float32)
        video_b, text_b = plan.forward_sharded(comm, v, t, prec, out_dtype=dtype)  # outputs in the block dtype
        video_1, text_1 = plan.forward(v, t, prec, out_dtype=torch.float32)
        # direct mode: the video output in a buffer shared over the ranks, each
        # rank's rows pushed into every rank's copy -- by the copy engines and by
        # the SM push kernel
        direct_equal, direct_text_rel = True, 0.0
        shared = comm.shared_tensor((cfg.source_tokens, cfg.heads, cfg.head_dim), torch.float32)
        for mode in (awa_b200.AWA_PUSH_COPY_ENGINES, awa_b200.AWA_PUSH_KERNEL):
            comm.set_push(mode)
            shared.fill_(float("nan"))
            torch.cuda.synchronize()
            dist.barrier()
            video_d, text_d = plan.forward_sharded(comm, v, t, prec, out_dtype=torch.float32, video_out=shared)
            torch.cuda.synchronize()
            direct_equal = direct_equal and bool(torch.equal(video_d, video_1))
            direct_text_rel = max(direct_text_rel, rel_l2(text_d.cpu().numpy(), text_1.cpu().numpy()))
            dist.barrier()
        comm.set_push(awa_b200.AWA_PUSH_AUTO)
        comm.free_shared(shared)
        torch.cuda.synchronize()
        status = 0
        try:
            awa_b200.device_status()
        except awa_b200.AwaError as err:
            status = err.code
        res = {
            "by_heads": by_heads, "bounds": bounds, "status": status,
            "video_equal": bool(torch.equal(video_s, video_1)),
            "direct_video_equal": direct_equal, "direct_text_rel": direct_text_rel,
            "text_rel": rel_l2(text_s.cpu().numpy(), text_1.cpu().numpy()),
            "video_block_rel": rel_l2(video_b.float().cpu().numpy(), video_1.cpu().numpy()),
            "text_block_rel": rel_l2(text_b.float().cpu().numpy(), text_1.cpu().numpy()),
        }
        if check_oracle and rank == 0:
            ref = oracle.chain(cfg, v.float().cpu().numpy(), t.float().cpu().numpy())
            res["oracle_video_rel"] = rel_l2(video_s.cpu().numpy(), ref["video"])
            res["oracle_text_rel"] = rel_l2(text_s.cpu().numpy(), ref["text"])
        results[name] = res
    dist.barrier()
    comm.destroy()
    dist.destroy_process_group()
    with open(out_path, "w") as f:
        json.dump(results, f)


if __name__ == "__main__":
    main(int(sys.argv[1]), int(sys.argv[2]), sys.argv[3], sys.argv[4])

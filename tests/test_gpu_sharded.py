"""One AWA layer split over 2 GPUs with NCCL (awa_forward_sharded).

Two processes (AWA_TEST_WORLD of them, up to the GPUs present, when that
variable is set), one per GPU (tests/sharded_worker.py), run each layer sharded
and on their own GPU alone. Windows are independent, so the video rows a rank
receives through the all-gather must equal, bit for bit, the single-GPU
awa_forward's; the text mean sums the same per-window values in another
grouping (per-rank partial sums, then the all-reduce), so it agrees to fp32
rounding. Small layers are also checked against the oracle's whole chain.
Covered: the window split (cfg2, cfg2 shifted, cfg4, cfg5-fp32 shifted) and
the head split of a layer with fewer than 4 windows per rank (cfg1, 4 windows),
bf16 (tensor cores) and fp32 (SIMT), fp32 and block-dtype outputs, and the
direct mode, where the video output lies in a buffer shared over the ranks
(awa_comm_alloc_shared) and each rank's rows are pushed into every rank's copy
over NVLink, by the copy engines and by the SM push kernel.
"""

import json
import os
import subprocess
import sys

import pytest

from awa_testlib import BF16_REL_L2, FP32_REL_L2

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
    pytest.skip("needs 2 CUDA devices", allow_module_level=True)

HERE = os.path.dirname(os.path.abspath(__file__))
WORLD = int(os.environ.get("AWA_TEST_WORLD", "2"))
if WORLD < 2 or torch.cuda.device_count() < WORLD:
    pytest.skip(f"needs {WORLD} CUDA devices", allow_module_level=True)


@pytest.fixture(scope="module")
def rank_results(tmp_path_factory):
    out = tmp_path_factory.mktemp("sharded")
    store = out / "rendezvous"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "sharded_worker.py"), str(r), str(WORLD), str(store),
                               str(out / f"rank{r}.json")], env=env) for r in range(WORLD)]
    codes = []
    for p in procs:
        try:
            codes.append(p.wait(timeout=600))
        except subprocess.TimeoutExpired:
            p.kill()
            codes.append(-9)
    assert codes == [0] * WORLD, f"rank exit codes {codes}"
    return [json.load(open(out / f"rank{r}.json")) for r in range(WORLD)]


CASES = ["cfg2-windows", "cfg2-shifted-windows", "cfg1-heads-bf16", "cfg1-heads-fp32", "cfg1-shifted-fp32",
         "cfg5-fp32-shifted", "cfg4"]


@pytest.mark.parametrize("name", CASES)
def test_sharded_layer_matches_single_gpu(rank_results, name):
    bf16 = "fp32" not in name
    for rank, res in enumerate(rank_results):
        r = res[name]
        assert r["status"] == 0, (rank, r)
        if WORLD == 2:
            assert r["by_heads"] == ("heads" in name), r
        assert r["video_equal"], (rank, name)
        assert r["text_rel"] < 1e-6, (rank, r["text_rel"])
        # the video output in a buffer shared over the ranks, rows pushed by the
        # copy engines and by the SM push kernel
        assert r["direct_video_equal"], (rank, name, "direct")
        assert r["direct_text_rel"] < 1e-6, (rank, r["direct_text_rel"])
        block_tol = 1e-2 if bf16 else 1e-6
        assert r["video_block_rel"] < block_tol and r["text_block_rel"] < block_tol, r
    r0 = rank_results[0][name]
    if "oracle_video_rel" in r0:
        tol = BF16_REL_L2 if bf16 else FP32_REL_L2
        assert r0["oracle_video_rel"] < tol and r0["oracle_text_rel"] < tol, r0

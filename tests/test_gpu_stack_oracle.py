"""BASELINE config 3 through the block-stack driver, pinned to the oracle.

Config 3 is one sampling step of the DiT's attention path at the 21-frame
256x256 shape: 32 blocks of the AWA layer on the 6x16x16 grid (num_windows
2,8,8), the shift alternating by block (tools/reference/dit_stack.py:75-79),
blocks 0-8 fp32 and 9-31 bf16 (the reference's mixed mode, dit_stack.cpp:519,
934-950). Per block the stack driver (awa_stack_run, include/awa_stack.h) runs
the hook's QKV projection with the Q/K RMSNorm (awa_qkv_project), the block's
AWA chain at the block's precision, and the hook's proj_out + gate + residual
(awa_out_project) -- DitStackSession::run (dit_stack.cpp:931-982) restricted to
the attention path.

The oracle is the numpy / C restatement of the same steps: oracle.qkv_project
(pinned to FixedMMAttention's modules), oracle.chain (pinned to the reference's
compiled awa_layers.cpp) and oracle.out_project (pinned to FixedDitBlock's
modules). Checks:

* every block against the oracle fed the GPU's own block input (so errors do
  not compound): QKV rows 5e-3 relative L2 (bf16 GEMM), the AWA output 1e-5 in
  the fp32 blocks and 2e-2 in the bf16 blocks, the block output 5e-3;
* the whole 32-block step against the oracle's own 32-block step, 2e-2.
"""

import numpy as np
import pytest

from awa_testlib import BF16_REL_L2, FP32_REL_L2, rel_l2
from oracle.oracle import LayerConfig, out_project, qkv_project, round_bf16_rne

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import awa_b200  # noqa: E402
from awa_b200 import AWA_BF16, AWA_F32, AWA_PREC_FP32, AWA_STACK_BEFORE  # noqa: E402

HEADS, HEAD_DIM, DIM, EPS = 20, 128, 2560, 1e-5
GRID, WINDOWS, TEXT = (6, 16, 16), (2, 8, 8), 58
BLOCKS, FP32_BLOCKS = 32, 9
N_V = GRID[0] * GRID[1] * GRID[2]
GEMM_REL_L2 = 5e-3


def host(t):
    return t.detach().float().cpu().numpy()


class Step:
    """Weights, buffers and the hook of one 32-block attention step; records
    every block's input, QKV rows, AWA output and output."""

    def __init__(self, seed=3):
        dev = torch.device("cuda", 0)
        g = torch.Generator(device=dev).manual_seed(seed)

        def rnd(*shape, scale=1.0):
            return torch.randn(*shape, device=dev, generator=g) * scale

        self.x0 = rnd(N_V, DIM).bfloat16()
        self.t0 = rnd(TEXT, DIM).bfloat16()
        self.w = [{"wqkv": rnd(3 * DIM, DIM, scale=DIM ** -0.5).bfloat16(),
                   "wout": rnd(DIM, DIM, scale=DIM ** -0.5).bfloat16(),
                   "gq": 1.0 + 0.2 * rnd(HEAD_DIM), "gk": 1.0 + 0.2 * rnd(HEAD_DIM),
                   "bias": 0.02 * rnd(DIM), "gate": 0.1 * rnd(DIM)} for _ in range(BLOCKS)]
        self.xv = [self.x0.clone(), torch.empty_like(self.x0)]
        self.xt = [self.t0.clone(), torch.empty_like(self.t0)]
        self.qkv = {dt: (torch.empty(N_V, 3, HEADS, HEAD_DIM, device=dev, dtype=dt),
                         torch.empty(TEXT, 3, HEADS, HEAD_DIM, device=dev, dtype=dt))
                    for dt in (torch.float32, torch.bfloat16)}
        # AWA outputs: fp32 in the fp32 blocks, bf16 in the others; proj_out reads bf16
        self.attn = {dt: (torch.empty(N_V, DIM, device=dev, dtype=dt), torch.empty(TEXT, DIM, device=dev, dtype=dt))
                     for dt in (torch.float32, torch.bfloat16)}
        self.cur = 0
        self.log = []

    def hook(self, stage, io, stream):
        lib, b, w = awa_b200.library(), io.block, self.w[io.block]
        fp32 = io.precision == AWA_PREC_FP32
        dt = torch.float32 if fp32 else torch.bfloat16
        qv, qt = self.qkv[dt]
        av, at = self.attn[dt]
        if stage == AWA_STACK_BEFORE:
            code = AWA_F32 if fp32 else AWA_BF16
            for x, q, rows in ((self.xv[self.cur], qv, N_V), (self.xt[self.cur], qt, TEXT)):
                if lib.awa_qkv_project(rows, DIM, HEADS, HEAD_DIM, x.data_ptr(), DIM, w["wqkv"].data_ptr(), DIM,
                                       w["gq"].data_ptr(), w["gk"].data_ptr(), EPS, code, q.data_ptr(), 3 * DIM,
                                       stream):
                    return 1
            io.in_dtype = code
            io.video_qkv, io.video_token_stride, io.video_qkv_stride = qv.data_ptr(), 3 * DIM, DIM
            io.text_qkv, io.text_token_stride, io.text_qkv_stride = qt.data_ptr(), 3 * DIM, DIM
            io.out_dtype = code
            io.video_out, io.video_out_stride = av.data_ptr(), DIM
            io.text_out, io.text_out_stride = at.data_ptr(), DIM
            return 0
        bv, bt = self.attn[torch.bfloat16]
        if fp32:  # proj_out takes bf16 rows
            bv.copy_(av)
            bt.copy_(at)
        rec = {"b": b, "x": (self.xv[self.cur].clone(), self.xt[self.cur].clone()), "qkv": (qv.clone(), qt.clone()),
               "attn": (av.clone(), at.clone())}
        nxt = 1 - self.cur
        for a, x, y, rows in ((bv, self.xv[self.cur], self.xv[nxt], N_V), (bt, self.xt[self.cur], self.xt[nxt], TEXT)):
            if lib.awa_out_project(rows, DIM, DIM, a.data_ptr(), DIM, w["wout"].data_ptr(), DIM, w["bias"].data_ptr(),
                                   w["gate"].data_ptr(), x.data_ptr(), DIM, AWA_BF16, AWA_BF16, y.data_ptr(), DIM,
                                   stream):
                return 1
        self.cur = nxt
        rec["y"] = (self.xv[nxt].clone(), self.xt[nxt].clone())
        self.log.append(rec)
        return 0


def oracle_block(oracle, b, w, xv, xt):
    """One block of the attention path in the oracle: (qkv rows, AWA output, block output)."""
    fp32 = b < FP32_BLOCKS
    wn = {k: host(v) for k, v in w.items()}
    q = [qkv_project(x, wn["wqkv"], wn["gq"], wn["gk"], EPS, HEADS) for x in (xv, xt)]
    if not fp32:
        q = [round_bf16_rne(a) for a in q]
    cfg = LayerConfig(*GRID, *WINDOWS, text_tokens=TEXT, shifted=b % 2, heads=HEADS, head_dim=HEAD_DIM)
    chain = oracle.chain(cfg, q[0], q[1])
    attn = [chain["video"].reshape(-1, DIM), chain["text"].reshape(-1, DIM)]
    if not fp32:
        attn = [round_bf16_rne(a) for a in attn]
    a16 = [round_bf16_rne(a) for a in attn]
    y = [round_bf16_rne(out_project(a, wn["wout"], wn["bias"], wn["gate"], x)) for a, x in zip(a16, (xv, xt))]
    return q, attn, y


@pytest.fixture(scope="module")
def gpu_step():
    torch.cuda.set_device(0)
    params = [{"source_t": -1, "source_h": -1, "source_w": -1, "windows_t": WINDOWS[0], "windows_h": WINDOWS[1],
               "windows_w": WINDOWS[2], "text_tokens": TEXT, "shifted": b % 2, "rope_dim": 126} for b in range(BLOCKS)]
    stack = awa_b200.AwaStack(params, runtime_spec=GRID, fp32_blocks=FP32_BLOCKS, heads=HEADS, head_dim=HEAD_DIM)
    step = Step()
    torch.cuda.synchronize()  # weights and inputs were made on the default stream
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        stack.run(step.hook, stream)
    stream.synchronize()
    awa_b200.device_status()
    assert [r["b"] for r in step.log] == list(range(BLOCKS))
    return step


def test_every_block_matches_the_oracle(gpu_step, oracle):
    for rec in gpu_step.log:
        b = rec["b"]
        xv, xt = (host(x) for x in rec["x"])
        q, attn, y = oracle_block(oracle, b, gpu_step.w[b], xv, xt)
        for got, want in zip(rec["qkv"], q):
            assert rel_l2(host(got), want) < GEMM_REL_L2, (b, "qkv")
        # the AWA chain on the GPU's own QKV rows (so only the chain's error shows)
        cfg = LayerConfig(*GRID, *WINDOWS, text_tokens=TEXT, shifted=b % 2, heads=HEADS, head_dim=HEAD_DIM)
        chain = oracle.chain(cfg, host(rec["qkv"][0]), host(rec["qkv"][1]))
        tol = FP32_REL_L2 if b < FP32_BLOCKS else BF16_REL_L2
        assert rel_l2(host(rec["attn"][0]), chain["video"].reshape(-1, DIM)) < tol, (b, "awa video")
        assert rel_l2(host(rec["attn"][1]), chain["text"].reshape(-1, DIM)) < tol, (b, "awa text")
        # the block output from the GPU's own AWA output
        a16 = [round_bf16_rne(host(a)) for a in rec["attn"]]
        wn = {k: host(v) for k, v in gpu_step.w[b].items()}
        for got, a, x in zip(rec["y"], a16, (xv, xt)):
            want = round_bf16_rne(out_project(a, wn["wout"], wn["bias"], wn["gate"], x))
            assert rel_l2(host(got), want) < GEMM_REL_L2, (b, "block output")


def test_whole_step_matches_the_oracle_step(gpu_step, oracle):
    xv, xt = host(gpu_step.x0), host(gpu_step.t0)
    for b in range(BLOCKS):
        _, _, (xv, xt) = oracle_block(oracle, b, gpu_step.w[b], xv, xt)
    got_v, got_t = (host(y) for y in gpu_step.log[-1]["y"])
    assert rel_l2(got_v, xv) < BF16_REL_L2 and rel_l2(got_t, xt) < BF16_REL_L2

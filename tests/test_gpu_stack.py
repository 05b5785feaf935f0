"""The block-stack driver (include/awa_stack.h) on the GPU, through the C ABI.

A 32-block stack (odd blocks shifted, the first 9 in fp32 as the reference's
mixed-precision model, src/dit/dit_stack.cpp:519) runs a residual stream
through each block's attention path: QKV projection with the Q/K RMSNorm
(awa_qkv_project, fp32 rows in the fp32 blocks), the block's AWA chain, then
proj_out + gate + residual (awa_out_project). The hook enqueues the two GEMMs;
the stack runs the AWA chains. Checks:

* the stack's result is bit-identical to the same calls made block by block
  with separately built plans and workspace (same kernels, same order);
* a CUDA graph captured from the stack replays bit-identically, twice;
* the hook sees each block's precision (fp32 prefix, bf16 suffix) and a hook
  failure stops the run with the hook's error.
"""

import ctypes

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import awa_b200  # noqa: E402
from awa_b200 import AWA_BF16, AWA_F32, AWA_PREC_BF16, AWA_PREC_FP32, AWA_STACK_BEFORE  # noqa: E402

HEADS, HEAD_DIM, DIM = 20, 128, 2560
GRID, WINDOWS, TEXT = (2, 16, 16), (1, 2, 2), 58
BLOCKS, FP32_BLOCKS = 32, 9
N_V = GRID[0] * GRID[1] * GRID[2]


def block_params(b):
    return {"source_t": -1, "source_h": -1, "source_w": -1, "windows_t": WINDOWS[0], "windows_h": WINDOWS[1],
            "windows_w": WINDOWS[2], "text_tokens": TEXT, "shifted": b % 2, "rope_dim": 126}


class Blocks:
    """Weights and preallocated buffers of the stack's attention path."""

    def __init__(self, seed=7):
        dev = torch.device("cuda", 0)
        g = torch.Generator(device=dev).manual_seed(seed)

        def rnd(*shape, scale=1.0):
            return torch.randn(*shape, device=dev, generator=g) * scale

        self.x0 = rnd(N_V, DIM).bfloat16()
        self.t0 = rnd(TEXT, DIM).bfloat16()
        self.sets = []
        for _ in range(4):
            self.sets.append({
                "wqkv": rnd(3 * DIM, DIM, scale=DIM ** -0.5).bfloat16(), "wout": rnd(DIM, DIM, scale=DIM ** -0.5).bfloat16(),
                "gq": 1.0 + 0.2 * rnd(HEAD_DIM), "gk": 1.0 + 0.2 * rnd(HEAD_DIM),
                "bias": 0.02 * rnd(DIM), "gate": 0.1 * rnd(DIM)})
        self.xv = [torch.empty(N_V, DIM, device=dev, dtype=torch.bfloat16) for _ in range(2)]
        self.xt = [torch.empty(TEXT, DIM, device=dev, dtype=torch.bfloat16) for _ in range(2)]
        self.qkv = {dt: (torch.empty(N_V, 3, HEADS, HEAD_DIM, device=dev, dtype=dt),
                         torch.empty(TEXT, 3, HEADS, HEAD_DIM, device=dev, dtype=dt))
                    for dt in (torch.float32, torch.bfloat16)}
        self.attn_v = torch.empty(N_V, DIM, device=dev, dtype=torch.bfloat16)
        self.attn_t = torch.empty(TEXT, DIM, device=dev, dtype=torch.bfloat16)
        self.cur = 0
        self.seen = []

    def reset(self):
        self.xv[0].copy_(self.x0)
        self.xt[0].copy_(self.t0)
        self.cur = 0

    def project(self, b, precision, stream):
        """QKV rows of block b into the buffers of its precision; returns them."""
        lib, w = awa_b200.library(), self.sets[b % 4]
        dt = torch.float32 if precision == AWA_PREC_FP32 else torch.bfloat16
        code = AWA_F32 if dt == torch.float32 else AWA_BF16
        qv, qt = self.qkv[dt]
        for x, q, rows in ((self.xv[self.cur], qv, N_V), (self.xt[self.cur], qt, TEXT)):
            assert lib.awa_qkv_project(rows, DIM, HEADS, HEAD_DIM, x.data_ptr(), DIM, w["wqkv"].data_ptr(), DIM,
                                       w["gq"].data_ptr(), w["gk"].data_ptr(), 1e-5, code, q.data_ptr(), 3 * DIM,
                                       stream) == 0
        return code, qv, qt

    def residual(self, b, stream):
        lib, w = awa_b200.library(), self.sets[b % 4]
        nxt = 1 - self.cur
        for a, x, y, rows in ((self.attn_v, self.xv[self.cur], self.xv[nxt], N_V),
                              (self.attn_t, self.xt[self.cur], self.xt[nxt], TEXT)):
            assert lib.awa_out_project(rows, DIM, DIM, a.data_ptr(), DIM, w["wout"].data_ptr(), DIM,
                                       w["bias"].data_ptr(), w["gate"].data_ptr(), x.data_ptr(), DIM, AWA_BF16,
                                       AWA_BF16, y.data_ptr(), DIM, stream) == 0
        self.cur = nxt

    def hook(self, stage, io, stream):
        if stage == AWA_STACK_BEFORE:
            self.seen.append((io.block, io.precision))
            code, qv, qt = self.project(io.block, io.precision, stream)
            io.in_dtype = code
            io.video_qkv, io.video_token_stride, io.video_qkv_stride = qv.data_ptr(), 3 * DIM, DIM
            io.text_qkv, io.text_token_stride, io.text_qkv_stride = qt.data_ptr(), 3 * DIM, DIM
            io.out_dtype = AWA_BF16
            io.video_out, io.video_out_stride = self.attn_v.data_ptr(), DIM
            io.text_out, io.text_out_stride = self.attn_t.data_ptr(), DIM
        else:
            self.residual(io.block, stream)
        return 0

    def result(self):
        return self.xv[self.cur].clone(), self.xt[self.cur].clone()


@pytest.fixture(scope="module")
def stack():
    torch.cuda.set_device(0)
    return awa_b200.AwaStack([block_params(b) for b in range(BLOCKS)], runtime_spec=GRID, fp32_blocks=FP32_BLOCKS,
                             heads=HEADS, head_dim=HEAD_DIM)


def eager_reference(blocks, stream):
    """The same calls block by block, with their own plans and workspace."""
    lib = awa_b200.library()
    plans = [awa_b200.AwaPlan(-1, -1, -1, *WINDOWS, TEXT, s, 126, runtime_spec=GRID) for s in (0, 1)]
    ws_bytes = max(lib.awa_forward_workspace_bytes(p.handle, HEADS, HEAD_DIM) for p in plans)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    handle = stream.cuda_stream
    with torch.cuda.stream(stream):
        blocks.reset()
        for b in range(BLOCKS):
            prec = AWA_PREC_FP32 if b < FP32_BLOCKS else AWA_PREC_BF16
            code, qv, qt = blocks.project(b, prec, handle)
            assert lib.awa_forward(plans[b % 2].handle, prec, HEADS, HEAD_DIM, code, qv.data_ptr(), 3 * DIM, DIM,
                                   qt.data_ptr(), 3 * DIM, DIM, AWA_BF16, blocks.attn_v.data_ptr(), DIM,
                                   blocks.attn_t.data_ptr(), DIM, ws.data_ptr(), ws_bytes, handle) == 0
            blocks.residual(b, handle)
        out = blocks.result()
    stream.synchronize()
    return out


def test_stack_shares_two_plans(stack):
    plans, ws = stack.info()
    assert plans == 2 and ws > 0


def test_stack_run_matches_block_by_block_calls(stack):
    blocks = Blocks()
    stream = torch.cuda.Stream()
    ref_v, ref_t = eager_reference(blocks, stream)
    assert torch.isfinite(ref_v.float()).all() and torch.isfinite(ref_t.float()).all()
    with torch.cuda.stream(stream):
        blocks.reset()
        blocks.seen.clear()
        stack.run(blocks.hook, stream)
        got_v, got_t = blocks.result()
    stream.synchronize()
    awa_b200.device_status()
    assert blocks.seen == [(b, AWA_PREC_FP32 if b < FP32_BLOCKS else AWA_PREC_BF16) for b in range(BLOCKS)]
    assert torch.equal(got_v, ref_v) and torch.equal(got_t, ref_t)
    # the residual stream moved: the blocks did work
    assert not torch.equal(got_v, blocks.x0)


def test_stack_graph_replays_bit_identically(stack):
    blocks = Blocks()
    stream = torch.cuda.Stream()
    ref_v, ref_t = eager_reference(blocks, stream)
    with torch.cuda.stream(stream):
        blocks.reset()
        stack.run(blocks.hook, stream)  # eager first: first-use set-up stays outside the capture
        blocks.reset()
        graph = stack.capture(blocks.hook, stream)
    stream.synchronize()
    for _ in range(2):
        with torch.cuda.stream(stream):
            blocks.xv[0].fill_(0)
            blocks.xt[0].fill_(0)
            blocks.reset()
            graph.launch(stream)
            got_v, got_t = blocks.xv[blocks.cur].clone(), blocks.xt[blocks.cur].clone()
        stream.synchronize()
        assert torch.equal(got_v, ref_v) and torch.equal(got_t, ref_t)
    del graph
    awa_b200.device_status()


def test_stack_hook_failure_stops_the_run(stack):
    blocks = Blocks()
    stream = torch.cuda.Stream()
    calls = []

    def failing(stage, io, handle):
        calls.append(io.block)
        if io.block == 3 and stage == AWA_STACK_BEFORE:
            raise RuntimeError("hook failed at block 3")
        return blocks.hook(stage, io, handle)

    with torch.cuda.stream(stream):
        blocks.reset()
        with pytest.raises(RuntimeError, match="hook failed at block 3"):
            stack.run(failing, stream)
    stream.synchronize()
    assert max(calls) == 3
    # a nonzero return code is reported through the C status
    lib = awa_b200.library()
    cb = awa_b200.STACK_HOOK(lambda user, stage, io, handle: 5)
    assert lib.awa_stack_run(stack.handle, cb, None, stream.cuda_stream) == -1
    assert b"hook returned 5 before block 0" in lib.awa_last_error()
    awa_b200.device_status()


def test_stack_rejects_bad_arguments():
    lib = awa_b200.library()
    handle = ctypes.c_void_p()
    params = (awa_b200._LayerParams * 2)()
    assert lib.awa_stack_create(ctypes.cast(params, ctypes.c_void_p), 2, None, 3, HEADS, HEAD_DIM,
                                ctypes.byref(handle)) == -1
    assert lib.awa_stack_create(None, 2, None, 0, HEADS, HEAD_DIM, ctypes.byref(handle)) == -1
    # a dynamic grid needs the runtime spec (load_common, awa_layers.cpp:97-104)
    dyn = (awa_b200._LayerParams * 1)(awa_b200._LayerParams(-1, -1, -1, 1, 2, 2, TEXT, 0, 126))
    assert lib.awa_stack_create(ctypes.cast(dyn, ctypes.c_void_p), 1, None, 0, HEADS, HEAD_DIM,
                                ctypes.byref(handle)) == -1
    assert not handle.value

"""awa_forward_noalloc: the fused forward for callers that must not allocate.

Some hosts cannot let a library allocate device memory: a serving process
whose memory manager reserves the whole GPU, a plugin that may only use its
host framework's allocator, a latency-bound pipeline that cannot take the
device-wide synchronisation of cudaMalloc/cudaFree. awa_forward_noalloc
serves them from a fixed scratch array the library keeps in device memory.

These tests call it through the C ABI and compare it with awa_forward (which
takes a caller-provided workspace) on two calls in a row with different
inputs, so a result that leaned on the previous call's scratch contents would
show. They sit in a file of their own, collected last, and need nothing from
the other test files: they pass alone in a fresh process and after the rest.
"""

from __future__ import annotations

import ctypes

import pytest

import awa_b200
from awa_testlib import BF16_REL_L2, FP32_REL_L2, rel_l2, to_host

pytestmark = pytest.mark.gpu

HEADS = 20
HEAD_DIM = 128
TEXT = 58


def _forward(lib, plan, precision, v, t, video_out, text_out, workspace=None) -> int:
    """awa_forward (with `workspace`) or awa_forward_noalloc (without), through the C ABI."""
    import torch

    stream = torch.cuda.current_stream().cuda_stream
    common = [plan.handle, precision, HEADS, HEAD_DIM, awa_b200._dtype_code(v), v.data_ptr(), v.stride(0),
              v.stride(1), t.data_ptr(), t.stride(0), t.stride(1), awa_b200._dtype_code(video_out),
              video_out.data_ptr(), video_out.stride(0), text_out.data_ptr(), text_out.stride(0)]
    if workspace is None:
        return lib.awa_forward_noalloc(*common, stream)
    return lib.awa_forward(*common, workspace.data_ptr(), workspace.numel(), stream)


@pytest.mark.parametrize("precision", ["bf16", "fp32"])
def test_noalloc_matches_forward_on_two_calls(precision):
    import torch

    lib = awa_b200.library()
    bf16 = precision == "bf16"
    prec = awa_b200.AWA_PREC_BF16 if bf16 else awa_b200.AWA_PREC_FP32
    dtype = torch.bfloat16 if bf16 else torch.float32
    tol = BF16_REL_L2 if bf16 else FP32_REL_L2
    # 3 x 16 x 24 latent grid, shifted windows (partial edge windows included)
    plan = awa_b200.AwaPlan(3, 16, 24, 1, 2, 3, text_tokens=TEXT, shifted=True)
    assert 0 < plan.workspace_bytes(HEADS, HEAD_DIM) <= awa_b200.AWA_NOALLOC_SCRATCH_BYTES
    if bf16:
        assert plan.attention_kernel_kind(prec, HEADS, HEAD_DIM) == 1  # the tcgen05 kernel
    tokens = plan.info.source_tokens
    workspace = torch.empty(plan.workspace_bytes(HEADS, HEAD_DIM), dtype=torch.uint8, device="cuda")
    for call in range(2):
        gen = torch.Generator(device="cuda").manual_seed(7001 + call)
        v = torch.randn(tokens, 3, HEADS, HEAD_DIM, generator=gen, device="cuda").to(dtype)
        t = torch.randn(TEXT, 3, HEADS, HEAD_DIM, generator=gen, device="cuda").to(dtype)
        ref_video = torch.empty(tokens, HEADS, HEAD_DIM, dtype=dtype, device="cuda")
        ref_text = torch.empty(TEXT, HEADS, HEAD_DIM, dtype=dtype, device="cuda")
        video = torch.full_like(ref_video, float("nan"))
        text = torch.full_like(ref_text, float("nan"))
        assert _forward(lib, plan, prec, v, t, ref_video, ref_text, workspace) == awa_b200.AWA_OK
        rc = _forward(lib, plan, prec, v, t, video, text)
        assert rc == awa_b200.AWA_OK, lib.awa_last_error().decode()
        torch.cuda.synchronize()
        awa_b200.device_status()
        # Same kernels on the same inputs: the outputs must be bit-identical, so
        # even a small error from stale scratch contents would show.
        assert torch.equal(video, ref_video), \
            f"video, call {call}: rel_l2 {rel_l2(to_host(video), to_host(ref_video)):.3e} (tolerance {tol})"
        assert torch.equal(text, ref_text), \
            f"text, call {call}: rel_l2 {rel_l2(to_host(text), to_host(ref_text)):.3e} (tolerance {tol})"


def test_noalloc_rejects_layers_beyond_its_scratch():
    import torch

    lib = awa_b200.library()
    # 21 x 64 x 64 grid, 384 windows: 384 * 58 * 20 * 128 * 4 bytes of text partials
    plan = awa_b200.AwaPlan(21, 64, 64, 6, 8, 8, text_tokens=TEXT)
    assert plan.workspace_bytes(HEADS, HEAD_DIM) > awa_b200.AWA_NOALLOC_SCRATCH_BYTES
    small = torch.zeros(16, 3, HEADS, HEAD_DIM, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(16, HEADS, HEAD_DIM, dtype=torch.bfloat16, device="cuda")
    rc = _forward(lib, plan, awa_b200.AWA_PREC_BF16, small, small, out, out)
    assert rc == awa_b200.AWA_ERR_INVALID
    message = lib.awa_last_error().decode()
    assert "awa_forward_noalloc" in message and str(awa_b200.AWA_NOALLOC_SCRATCH_BYTES) in message

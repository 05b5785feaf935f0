"""Parity of the CUDA path with the oracle (the reference's CPU forward
restated, pinned bit-exact to it), through the C ABI.

Bit-exact: Pack, MMRoPE (fp32), Unpack (video rows and the text mean, given
identical attended input). Tolerance: attention and the fused chain, fp32
1e-5 relative L2, bf16 2e-2 relative L2.
"""

import zlib

import numpy as np
import pytest

from awa_testlib import BF16_REL_L2, FP32_REL_L2, make_inputs, plan_for, rel_l2, to_device, to_host
from oracle.oracle import LayerConfig

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import awa_b200  # noqa: E402
from awa_b200 import AWA_PREC_BF16, AWA_PREC_FP32  # noqa: E402

CASES = [
    # small generic shapes (scalar / fallback paths)
    LayerConfig(2, 5, 7, 2, 2, 3, text_tokens=3, shifted=1, heads=2, head_dim=8, rope_dim=6),
    LayerConfig(2, 19, 23, 4, 3, 3, text_tokens=5, shifted=0, heads=2, head_dim=12, rope_dim=12),
    LayerConfig(3, 9, 10, 2, 2, 3, text_tokens=7, shifted=1, heads=3, head_dim=24, rope_dim=18),
    # BASELINE config 1 (fp32, 4 windows) and its shifted layer, full 20 heads x 128
    LayerConfig(1, 16, 16, 1, 8, 8, shifted=0),
    LayerConfig(1, 16, 16, 1, 8, 8, shifted=1),
    # BASELINE config 2 (6x16x16, 3x8x8 windows), both shifts
    LayerConfig(6, 16, 16, 2, 8, 8, shifted=0),
    LayerConfig(6, 16, 16, 2, 8, 8, shifted=1),
    # product default window counts (4,3,3): 463-token windows (multi-block softmax)
    LayerConfig(1, 45, 80, 4, 3, 3, shifted=1, heads=2),
    # single text token; ragged windows of 48 and 54 tokens
    LayerConfig(2, 3, 17, 1, 1, 9, text_tokens=1, shifted=1, heads=2, head_dim=128),
    # 3600 one-token windows (shifted 1x1 windows on the 45x80 grid)
    LayerConfig(1, 45, 80, 1, 45, 80, text_tokens=3, shifted=1, heads=1, head_dim=128),
    # a single window holding a single video token
    LayerConfig(1, 1, 1, 1, 1, 1, text_tokens=2, shifted=0, heads=1, head_dim=128),
    # odd head count with 5 key blocks per window (two query tiles + an odd last
    # tile): head pairs (0, 1) and a lone head 2 on both kinds of work item
    LayerConfig(4, 16, 16, 1, 2, 2, shifted=1, heads=3, head_dim=128),
    # one 8x256 window (2106 rows, 1x64 boxes): a RoPE table of ~6.6K entries
    LayerConfig(1, 8, 256, 1, 1, 1, shifted=0, heads=2, head_dim=128),
]


def case_id(c):
    return f"{c.source_t}x{c.source_h}x{c.source_w}-{c.num_t}{c.num_h}{c.num_w}-s{c.shifted}-h{c.heads}d{c.head_dim}"


@pytest.fixture(scope="module")
def results(oracle):
    cache = {}

    def get(cfg, bf16):
        key = (cfg, bf16)
        if key not in cache:
            v, t = make_inputs(cfg, seed=zlib.crc32(case_id(cfg).encode()) % 1000 + int(bf16), bf16=bf16, oracle=oracle)
            cache[key] = (v, t, oracle.chain(cfg, v, t))
        return cache[key]

    return get


@pytest.mark.parametrize("cfg", CASES, ids=case_id)
def test_pack_rope_unpack_bitexact_fp32(cfg, results):
    v, t, ref = results(cfg, False)
    plan = plan_for(cfg)
    dv, dt = to_device(v, torch.float32), to_device(t, torch.float32)
    packed, cu = plan.pack(dv, dt)
    assert np.array_equal(to_host(packed), ref["packed"])
    assert np.array_equal(to_host(cu), ref["cu_seqlens"])
    roped = plan.mmrope(packed)
    assert np.array_equal(to_host(roped), ref["roped"])
    video, text = plan.unpack(to_device(ref["attended"], torch.float32))
    assert np.array_equal(to_host(video), ref["video"])
    assert np.array_equal(to_host(text), ref["text"])
    awa_b200.device_status()


@pytest.mark.parametrize("cfg", CASES, ids=case_id)
def test_attention_fp32(cfg, results):
    _, _, ref = results(cfg, False)
    plan = plan_for(cfg)
    attended = plan.window_attention(to_device(ref["roped"], torch.float32), AWA_PREC_FP32)
    assert rel_l2(to_host(attended), ref["attended"]) < FP32_REL_L2
    awa_b200.device_status()


@pytest.mark.parametrize("cfg", CASES, ids=case_id)
def test_attention_bf16(cfg, results):
    _, _, ref = results(cfg, True)
    plan = plan_for(cfg)
    roped_bf16 = to_device(ref["roped"], torch.bfloat16)
    attended = plan.window_attention(roped_bf16, AWA_PREC_BF16, out_dtype=torch.float32)
    err = rel_l2(to_host(attended), ref["attended"])
    assert err < BF16_REL_L2, err
    awa_b200.device_status()


@pytest.mark.parametrize("cfg", CASES, ids=case_id)
def test_fused_forward_fp32(cfg, results):
    v, t, ref = results(cfg, False)
    plan = plan_for(cfg)
    video, text = plan.forward(to_device(v, torch.float32), to_device(t, torch.float32), AWA_PREC_FP32)
    assert rel_l2(to_host(video), ref["video"]) < FP32_REL_L2
    assert rel_l2(to_host(text), ref["text"]) < FP32_REL_L2
    awa_b200.device_status()


@pytest.mark.parametrize("cfg", CASES, ids=case_id)
@pytest.mark.parametrize("out_dtype", ["bf16", "f32"])
def test_fused_forward_bf16(cfg, results, out_dtype):
    v, t, ref = results(cfg, True)
    plan = plan_for(cfg)
    odt = torch.bfloat16 if out_dtype == "bf16" else torch.float32
    video, text = plan.forward(to_device(v, torch.bfloat16), to_device(t, torch.bfloat16), AWA_PREC_BF16,
                               out_dtype=odt)
    assert rel_l2(to_host(video), ref["video"]) < BF16_REL_L2
    assert rel_l2(to_host(text), ref["text"]) < BF16_REL_L2
    awa_b200.device_status()


@pytest.mark.parametrize("cfg", [CASES[4], CASES[6]], ids=case_id)
def test_fused_equals_layer_chain_and_is_deterministic(cfg, results):
    v, t, _ = results(cfg, True)
    plan = plan_for(cfg)
    dv, dt = to_device(v, torch.bfloat16), to_device(t, torch.bfloat16)
    for prec, dtype in ((AWA_PREC_FP32, torch.float32), (AWA_PREC_BF16, torch.bfloat16)):
        packed, _ = plan.pack(dv.to(dtype), dt.to(dtype))
        attended = plan.window_attention(plan.mmrope(packed), prec)
        video_l, text_l = plan.unpack(attended)
        video_f, text_f = plan.forward(dv.to(dtype), dt.to(dtype), prec)
        video_f2, text_f2 = plan.forward(dv.to(dtype), dt.to(dtype), prec)
        assert torch.equal(video_f, video_f2) and torch.equal(text_f, text_f2)
        # Same arithmetic on the same rows: the two paths agree to rounding.
        tol = 1e-6 if prec == AWA_PREC_FP32 else 1e-2
        assert rel_l2(to_host(video_f), to_host(video_l)) < tol
        assert rel_l2(to_host(text_f), to_host(text_l)) < tol


def test_strided_blobs_like_ncnn(oracle):
    """QKV blobs in the (w=d, h=H, c=3N) encoding and padded token strides."""
    cfg = LayerConfig(2, 5, 7, 2, 2, 3, text_tokens=3, shifted=1, heads=2, head_dim=8, rope_dim=6)
    v, t = make_inputs(cfg, 5, False, oracle)
    ref = oracle.chain(cfg, v, t)
    plan = plan_for(cfg)
    # qkv-major storage [3][tokens][H][d] viewed as [tokens, 3, H, d]
    dv = to_device(np.ascontiguousarray(v.transpose(1, 0, 2, 3)), torch.float32).permute(1, 0, 2, 3)
    dt = to_device(np.ascontiguousarray(t.transpose(1, 0, 2, 3)), torch.float32).permute(1, 0, 2, 3)
    packed, _ = plan.pack(dv, dt)
    assert np.array_equal(to_host(packed), ref["packed"])
    video, text = plan.forward(dv, dt, AWA_PREC_FP32)
    assert rel_l2(to_host(video), ref["video"]) < FP32_REL_L2
    assert rel_l2(to_host(text), ref["text"]) < FP32_REL_L2


def test_invalid_arguments_rejected():
    plan = plan_for(LayerConfig(1, 16, 16, 1, 8, 8))
    lib = awa_b200.library()
    assert lib.awa_window_attention(plan.handle, 0, 20, 129, 0, 16, 7680, 0, 16, 2560, None) == -1
    assert lib.awa_window_attention(plan.handle, 0, 0, 128, 0, 16, 7680, 0, 16, 2560, None) == -1
    assert lib.awa_window_attention(plan.handle, 7, 20, 128, 0, 16, 7680, 0, 16, 2560, None) == -1
    # rope_dim > head_dim (awa_layers.cpp:920)
    assert lib.awa_mmrope(plan.handle, 2, 64, 0, 16, 384, 0, 16, 384, None) == -1
    awa_b200.device_status()


@pytest.mark.parametrize("cfg", [CASES[3], CASES[4], CASES[6], CASES[11]], ids=case_id)
def test_fp32_qkv_in_a_bf16_block_takes_the_tensor_cores(cfg, results):
    """A bf16 block fed fp32 QKV (the reference promotes QKV to fp32 ahead of
    Pack in its bf16 blocks, dit_precision.cpp:314-315): the fused forward
    converts the rows to bf16 in its workspace (one rounding, to nearest
    even) and runs the tcgen05 kernel -- the same result as handing it the
    bf16 rows, within the bf16 tolerance of the oracle on the fp32 rows."""
    v, t, ref = results(cfg, False)
    plan = plan_for(cfg)
    assert plan.attention_kernel_kind(AWA_PREC_BF16, cfg.heads, cfg.head_dim, torch.float32) == 1
    need = plan.workspace_bytes(cfg.heads, cfg.head_dim, AWA_PREC_BF16, torch.float32)
    assert need > plan.workspace_bytes(cfg.heads, cfg.head_dim)
    dv, dt = to_device(v, torch.float32), to_device(t, torch.float32)
    awa_b200.profile_reset()
    awa_b200.profile_enable(True)
    video, text = plan.forward(dv, dt, AWA_PREC_BF16, out_dtype=torch.float32)
    awa_b200.profile_enable(False)
    prof = awa_b200.profile_collect()
    assert "awa_attention_tc_fused" in prof and "awa_rows_to_bf16" in prof, prof
    video_b, text_b = plan.forward(dv.bfloat16(), dt.bfloat16(), AWA_PREC_BF16, out_dtype=torch.float32)
    assert torch.equal(video, video_b) and torch.equal(text, text_b)
    assert rel_l2(to_host(video), ref["video"]) < BF16_REL_L2
    assert rel_l2(to_host(text), ref["text"]) < BF16_REL_L2
    # a workspace that only holds the text partials is refused, not silently slower
    small = torch.empty(plan.workspace_bytes(cfg.heads, cfg.head_dim), dtype=torch.uint8, device="cuda")
    with pytest.raises(awa_b200.AwaError, match="awa_forward_workspace_bytes_for"):
        plan.forward(dv, dt, AWA_PREC_BF16, workspace=small)
    awa_b200.device_status()


@pytest.mark.parametrize("cfg", [CASES[4], CASES[1]], ids=case_id)
def test_forward_on_host_buffers(cfg, results):
    """awa_forward_host (host blobs, as the reference layers' CPU forward takes
    them): the same outputs as awa_forward on device copies, bit for bit, with
    dense host rows and with the qkv-major encoding's strides."""
    bf16 = cfg.head_dim == 128
    v, t, _ = results(cfg, bf16)
    plan = plan_for(cfg)
    prec, dtype = (AWA_PREC_BF16, torch.bfloat16) if bf16 else (AWA_PREC_FP32, torch.float32)
    ref_v, ref_t = plan.forward(to_device(v, dtype), to_device(t, dtype), prec, out_dtype=torch.float32)
    for layout in ("dense", "qkv-major"):
        hv = torch.from_numpy(np.ascontiguousarray(v)).to(dtype)
        ht = torch.from_numpy(np.ascontiguousarray(t)).to(dtype)
        if layout == "qkv-major":
            hv = hv.permute(1, 0, 2, 3).contiguous().permute(1, 0, 2, 3)
            ht = ht.permute(1, 0, 2, 3).contiguous().permute(1, 0, 2, 3)
        hv, ht = hv.pin_memory(), ht.pin_memory()
        out_v = torch.empty(cfg.source_tokens, cfg.heads, cfg.head_dim).pin_memory()
        out_t = torch.empty(cfg.text_tokens, cfg.heads, cfg.head_dim).pin_memory()
        stream = torch.cuda.Stream()
        plan.forward_host(hv, ht, out_v, out_t, prec, stream=stream)
        stream.synchronize()
        awa_b200.device_status()
        assert torch.equal(out_v, ref_v.cpu()), layout
        assert torch.equal(out_t, ref_t.cpu()), layout

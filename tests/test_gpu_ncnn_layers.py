"""The ncnn layer classes (the drop-in boundary) on the GPU, against the oracle.

The four classes SeedVR2AWAPack -> SeedVR2MMRoPE -> SeedVR2WindowAttention ->
SeedVR2AWAUnpack are driven the way a DiT block graph drives the reference's
(register_seedvr2_awa_layers, Net::create_custom_layer, load_param with
ParamDict ids 0-8, forward; awa_layers.cpp:1267-1291, dit_stack.cpp:180), by
awa_ncnn_run_chain in the compat library:

* host blobs (forward(Mat), the reference's CPU entry) and device blobs
  (forward_cuda(CudaBlob), the counterpart of its VkMat forward);
* fp32 blocks and bf16 blocks (ncnn Option use_bf16_storage,
  awa_layers.cpp:184-187), whose Unpack outputs are bf16 (:832-837), with
  bf16 QKV and with the promoted fp32 QKV of dit_precision.cpp:314-315;
* every QKV blob encoding describe_qkv_layout accepts (awa_layers.cpp:124-170):
  (w=d, h=3H, c=N), (w=d, h=H, c=3N), (w=d, h=H, d=3, c=N), and in the
  NCNN_BATCH build (w=d, h=H, c=3, n=N) with the 4-D batched video output;
* the grid from the creator's AwaRuntimeSpec (ParamDict 0-2 = -1).

Tolerances: fp32 blocks bit-exact for Pack, cu_seqlens and MMRoPE, 1e-5
relative L2 after attention; bf16 blocks bit-exact for Pack, 2e-2 relative L2
after attention.
"""

import numpy as np
import pytest

from awa_testlib import BF16_REL_L2, FP32_REL_L2, make_inputs, rel_l2
from oracle.oracle import LayerConfig

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import awa_b200  # noqa: E402

CFG1 = LayerConfig(1, 16, 16, 1, 8, 8, shifted=0)  # 4 windows, 20 heads x 128
SHIFTED = LayerConfig(2, 16, 24, 1, 2, 3, shifted=1, heads=4)  # partial edge windows


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 values that are exact bf16 -> their uint16 bit patterns."""
    return (np.ascontiguousarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def from_bits(x: np.ndarray) -> np.ndarray:
    return (x.astype(np.uint32) << 16).view(np.float32) if x.dtype == np.uint16 else x


_oracle_cache = {}


def oracle_chain(oracle, cfg, bf16_inputs, seed):
    key = (cfg, bf16_inputs, seed)
    if key not in _oracle_cache:
        v, t = make_inputs(cfg, seed, bf16_inputs, oracle)
        _oracle_cache[key] = (v, t, oracle.chain(cfg, v, t))
    return _oracle_cache[key]


def run_and_check(oracle, cfg, layout, bf16, device_blobs, batch_build=False, fp32_inputs_in_bf16=False,
                  runtime_spec=False):
    bf16_inputs = bf16 and not fp32_inputs_in_bf16
    v, t, ref = oracle_chain(oracle, cfg, bf16_inputs, seed=31 + layout)
    vin, tin = (bf16_bits(v), bf16_bits(t)) if bf16_inputs else (v, t)
    out = awa_b200.ncnn_run_chain(cfg.params, cfg.heads, cfg.head_dim, vin, tin, layout=layout,
                                  runtime_spec=runtime_spec, bf16=bf16, device_blobs=device_blobs,
                                  batch_build=batch_build)
    assert out["status"] == 0
    # the outputs' element size follows the block precision (bf16 blocks cast them)
    assert out["video"].dtype == (np.uint16 if bf16 else np.float32)
    assert np.array_equal(out["cu_seqlens"], ref["cu_seqlens"])
    if not bf16:
        assert np.array_equal(out["packed"], ref["packed"])
        assert np.array_equal(out["roped"], ref["roped"])
        tol = FP32_REL_L2
    else:
        packed = from_bits(out["packed"])
        assert np.array_equal(packed, oracle.round_bf16(ref["packed"]))
        if bf16_inputs:
            # fp32 rotation of bf16 values, rounded once
            assert np.array_equal(from_bits(out["roped"]), oracle.round_bf16(ref["roped"]))
        tol = BF16_REL_L2
    for key in ("attended", "video", "text"):
        err = rel_l2(from_bits(out[key]), ref[key])
        assert err <= tol, f"{key}: rel_l2 {err:.3e} > {tol}"


@pytest.mark.parametrize("device_blobs", [False, True], ids=["host-mat", "cuda-blob"])
@pytest.mark.parametrize("bf16", [False, True], ids=["fp32-block", "bf16-block"])
@pytest.mark.parametrize("layout", [0, 1, 2])
def test_ncnn_chain_encodings(oracle, layout, bf16, device_blobs):
    run_and_check(oracle, CFG1, layout, bf16, device_blobs, runtime_spec=layout == 1)


@pytest.mark.parametrize("device_blobs", [False, True], ids=["host-mat", "cuda-blob"])
@pytest.mark.parametrize("bf16", [False, True], ids=["fp32-block", "bf16-block"])
@pytest.mark.parametrize("layout", [3, 0])
def test_ncnn_batch_build(oracle, layout, bf16, device_blobs):
    """The NCNN_BATCH build: the batched QKV encoding (c=3, n=N) and the 4-D
    batched video output (w=d, h=H, d=W, c=H_grid, n=T), whose frames sit on
    4 KiB batch boundaries."""
    run_and_check(oracle, SHIFTED, layout, bf16, device_blobs, batch_build=True)


@pytest.mark.parametrize("device_blobs", [False, True], ids=["host-mat", "cuda-blob"])
def test_ncnn_bf16_block_with_fp32_qkv(oracle, device_blobs):
    """A bf16 block fed fp32 QKV (the reference promotes QKV to fp32 ahead of
    Pack in its bf16 blocks, dit_precision.cpp:314-315)."""
    run_and_check(oracle, SHIFTED, 0, True, device_blobs, fp32_inputs_in_bf16=True)


def test_ncnn_shifted_windows_runtime_spec(oracle):
    run_and_check(oracle, SHIFTED, 2, False, True, runtime_spec=True)


def test_ncnn_rejects_unknown_encoding(oracle):
    v, t, _ = oracle_chain(oracle, SHIFTED, False, 5)
    out = awa_b200.ncnn_run_chain(SHIFTED.params, SHIFTED.heads, SHIFTED.head_dim, v, t, layout=3)
    assert out["status"] == -1  # the batched encoding needs an NCNN_BATCH build

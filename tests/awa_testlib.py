"""Shared helpers of the GPU parity tests: seeded inputs, the oracle's results,
and tolerance checks. Tolerances are the ones the reference port states:
fp32 blocks 1e-5 relative L2, bf16 blocks 2e-2 relative L2."""

from __future__ import annotations

import numpy as np

from oracle.oracle import LayerConfig, Oracle

FP32_REL_L2 = 1e-5
BF16_REL_L2 = 2e-2


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def make_inputs(cfg: LayerConfig, seed: int, bf16: bool, oracle: Oracle):
    """QKV ~ N(0, 1) (fp32 draws, rounded RNE to bf16 for bf16 cases)."""
    rng = np.random.default_rng(seed)
    v = rng.standard_normal((cfg.source_tokens, 3, cfg.heads, cfg.head_dim), dtype=np.float32)
    t = rng.standard_normal((cfg.text_tokens, 3, cfg.heads, cfg.head_dim), dtype=np.float32)
    if bf16:
        v = oracle.round_bf16(v)
        t = oracle.round_bf16(t)
    return v, t


def to_device(array, dtype):
    import torch

    return torch.from_numpy(np.ascontiguousarray(array)).to(device="cuda", dtype=dtype)


def to_host(tensor) -> np.ndarray:
    import torch

    return tensor.detach().to(torch.float32).cpu().numpy()


def plan_for(cfg: LayerConfig):
    import awa_b200

    return awa_b200.AwaPlan(*cfg.params[:6], text_tokens=cfg.text_tokens, shifted=cfg.shifted, rope_dim=cfg.rope_dim)

"""Write the golden fixtures of tests/golden/ from the reference's PyTorch mirror.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden.py --reference <reference checkout>

It imports ``tools/reference/{seedvr2_baseline,awa_attention,dit_block}.py`` of
HGinkgo/SeedVR2-ncnn and records, for each configuration:

* ``windows.json``: the window list of ``make_windows`` (seedvr2_baseline.py:37-79),
  the SHA-256 of the target and reverse index maps exactly as
  ``awa_round_trip`` reports them (seedvr2_baseline.py:92-114), the SHA-256 of
  the Pack ``sequence_index``/``video_positions``/``text_positions`` buffers
  (awa_attention.py:46-74) and ``cu_seqlens``.
* ``chain_*.npz``: one seeded forward of AwaAttentionPack -> 3D RoPE
  (dit_block.py:70-96 frequencies, :223-231 rotation, gathered as in :268-278)
  -> AwaWindowAttention -> AwaAttentionUnpack, with its inputs.
* ``qkv_project.npz``: the producer of the AWA input, run with the modules of
  FixedMMAttention (dit_block.py:234-263) as its forward does (:280-287): the
  bf16 proj_qkv Linear, then norm_q / norm_k (FixedRMSNorm) on Q and K.

* ``out_project.npz``: the consumer of the AWA output, run with the modules of
  FixedDitBlock (dit_block.py:302-349): attn.proj_out (a Linear with bias), the
  Ada "out" gate of ada.vid (:178-190) and the residual add (:345-347).

``--only gemms`` writes just these two.

The fixtures are small (a few hundred KB) and are what the CPU tests compare the
C oracle against; the GPU tests never read the reference.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# (size, num_windows, shifted) triples: the BASELINE configs, the exporter
# defaults (tools/export_awa_attention.py, seedvr2_baseline.py awa), the product
# default window counts (4,3,3) and ragged / non-divisible grids.
WINDOW_CASES = [
    ((1, 16, 16), (1, 8, 8)),
    ((6, 16, 16), (2, 8, 8)),
    ((6, 16, 16), (4, 3, 3)),
    ((21, 64, 64), (6, 8, 8)),
    ((21, 64, 64), (21, 8, 8)),
    ((9, 45, 80), (3, 6, 10)),
    ((1, 45, 80), (4, 3, 3)),
    ((2, 19, 23), (4, 3, 3)),
    ((1, 45, 80), (1, 1, 1)),
    ((3, 7, 11), (2, 3, 5)),
    ((40, 9, 13), (3, 2, 2)),
    ((33, 30, 52), (4, 3, 3)),
    ((1, 1, 1), (1, 1, 1)),
    ((5, 2, 97), (2, 1, 9)),
]

ROPE_STRIDE = 5

CHAIN_CASES = [
    # name, size, num_windows, text_tokens, heads, shifted, seed
    ("chain_small_unshifted", (2, 5, 7), (2, 2, 3), 3, 2, False, 20260823),
    ("chain_small_shifted", (2, 5, 7), (2, 2, 3), 3, 2, True, 20260824),
    ("chain_cfg1_1head", (1, 16, 16), (1, 8, 8), 58, 1, False, 0),
]


def sha(array) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


# tokens (not a multiple of the 128-row tile), model_dim (not a multiple of the
# 64-wide K slice), heads, eps, seed
QKV_CASE = (70, 160, 2, 1e-5, 20261202)


def make_qkv_fixture(torch) -> None:
    from tools.reference.dit_block import FixedMMAttention

    tokens, model_dim, heads, eps, seed = QKV_CASE
    head_dim = 128
    gen = torch.Generator().manual_seed(seed)
    block = FixedMMAttention((1, 2, 2), (1, 1, 1), 1, model_dim, model_dim, heads, head_dim, eps)
    with torch.no_grad():
        block.proj_qkv.vid.weight.copy_(torch.randn(3 * heads * head_dim, model_dim, generator=gen) * 0.08)
        block.norm_q.vid.weight.copy_(1.0 + 0.25 * torch.randn(head_dim, generator=gen))
        block.norm_k.vid.weight.copy_(1.0 + 0.25 * torch.randn(head_dim, generator=gen))
        block.proj_qkv.vid.to(torch.bfloat16)  # the bf16 blocks: bf16 Linear, fp32 RMSNorm weights
        x = torch.randn(tokens, model_dim, generator=gen).bfloat16()
        # FixedMMAttention.forward, dit_block.py:280-287 (video branch)
        qkv = block.proj_qkv.vid(x).reshape(-1, 3, heads, head_dim)
        q, k, v = qkv.unbind(dim=1)
        out = torch.stack((block.norm_q.vid(q), block.norm_k.vid(k), v.float()), dim=1)
    np.savez_compressed(
        os.path.join(HERE, "qkv_project.npz"), tokens=tokens, model_dim=model_dim, heads=heads, eps=eps, seed=seed,
        x=x.float().numpy(), w=block.proj_qkv.vid.weight.detach().float().numpy(),
        gamma_q=block.norm_q.vid.weight.detach().float().numpy(),
        gamma_k=block.norm_k.vid.weight.detach().float().numpy(), out=out.float().numpy())


# tokens (not a multiple of 128), in_dim (heads * 128), out_dim (= vid_dim), seed
OUT_CASE = (70, 256, 256, 20261203)


def make_out_fixture(torch) -> None:
    from tools.reference.dit_block import FixedDitBlock

    tokens, in_dim, dim, seed = OUT_CASE
    gen = torch.Generator().manual_seed(seed)
    block = FixedDitBlock(source_shape=(1, 2, 2), window_shape=(1, 1, 1), text_tokens=1, vid_dim=dim, txt_dim=dim,
                          emb_dim=6 * dim, heads=in_dim // 128, head_dim=128)
    with torch.no_grad():
        proj = block.attn.proj_out.vid
        proj.weight.copy_(torch.randn(dim, in_dim, generator=gen) * 0.06)
        proj.bias.copy_(torch.randn(dim, generator=gen) * 0.1)
        block.ada.vid.attn_gate.copy_(torch.randn(dim, generator=gen) * 0.2)
        proj.to(torch.bfloat16)  # the bf16 blocks
        emb = torch.randn(1, 6 * dim, generator=gen)
        attn_out = torch.randn(tokens, in_dim, generator=gen).bfloat16()
        vid = torch.randn(tokens, dim, generator=gen)  # the block input (residual), fp32
        # FixedDitBlock.forward :340-347 after the attention: proj_out, Ada "out", residual
        hidden = proj(attn_out)
        gated = block.ada.vid(hidden, emb, "attn", "out")
        out = gated + vid
        modulation = emb.reshape(1, dim, 2, 3)[0, :, 0, :]
        gate = modulation[:, 2] + block.ada.vid.attn_gate
    np.savez_compressed(
        os.path.join(HERE, "out_project.npz"), tokens=tokens, in_dim=in_dim, dim=dim, seed=seed,
        x=attn_out.float().numpy(), w=proj.weight.detach().float().numpy(), bias=proj.bias.detach().float().numpy(),
        gate=gate.detach().float().numpy(), residual=vid.numpy(), out=out.float().numpy())


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="root of a reference checkout")
    parser.add_argument("--only", choices=["gemms"], default=None)
    args = parser.parse_args()
    sys.path.insert(0, args.reference)
    import torch

    make_qkv_fixture(torch)
    make_out_fixture(torch)
    if args.only == "gemms":
        print("wrote qkv_project.npz and out_project.npz to", HERE)
        return
    from tools.reference.awa_attention import AwaAttentionPack, AwaAttentionUnpack, AwaWindowAttention
    from tools.reference.dit_block import _apply_fixed_rotary, build_mmrope_frequencies
    from tools.reference.seedvr2_baseline import awa_round_trip, make_windows

    records = []
    for size, num in WINDOW_CASES:
        for shifted in (False, True):
            windows = make_windows(size, num, shifted=shifted)
            source = torch.zeros(*size, 1)
            _, meta = awa_round_trip(source, num, shifted=shifted)
            pack = AwaAttentionPack(size, num, 58, shifted=shifted)
            records.append({
                "size": list(size), "num_windows": list(num), "shifted": shifted, "text_tokens": 58,
                "windows": [[a for axis in w for a in axis] for w in windows],
                "target_index_sha256": meta["target_index_sha256"],
                "reverse_index_sha256": meta["reverse_index_sha256"],
                "sequence_index_int64_sha256": sha(pack.sequence_index.numpy()),
                "video_positions_int64_sha256": sha(pack.video_positions.numpy()),
                "text_positions_int64_sha256": sha(pack.text_positions.numpy()),
                "cu_seqlens": [int(v) for v in pack.cu_seqlens.tolist()],
            })
    with open(os.path.join(HERE, "windows.json"), "w") as handle:
        json.dump({"generator": "tests/golden/make_golden.py", "cases": records}, handle, indent=1)

    for name, size, num, text_tokens, heads, shifted, seed in CHAIN_CASES:
        head_dim = 128  # dit_block.py's RoPE frequencies are fixed to 126 of 128 dims
        gen = torch.Generator().manual_seed(seed)
        tokens = size[0] * size[1] * size[2]
        vid = torch.randn(tokens, 3, heads, head_dim, generator=gen)
        txt = torch.randn(text_tokens, 3, heads, head_dim, generator=gen)
        pack = AwaAttentionPack(size, num, text_tokens, shifted=shifted)
        unpack = AwaAttentionUnpack(size, num, text_tokens, shifted=shifted)
        attention = AwaWindowAttention(pack.cu_seqlens, head_dim=head_dim)
        video_freqs, text_freqs = build_mmrope_frequencies(
            size, text_tokens, window_shape=num, shifted=shifted, device=torch.device("cpu"), dtype=torch.float32)
        # dit_block.py:276-278: frequencies in packed order.
        source_freqs = torch.cat((video_freqs.index_select(0, pack.reverse_index), text_freqs), dim=0)
        rope_freqs = source_freqs.index_select(0, pack.sequence_index)
        packed, cu = pack(vid.reshape(*size, 3, heads, head_dim), txt)
        q, k, v = packed.unbind(dim=1)
        roped = torch.stack((_apply_fixed_rotary(q, rope_freqs), _apply_fixed_rotary(k, rope_freqs), v), dim=1)
        attended = attention(roped)
        video, text = unpack(attended)
        rope_rows = torch.arange(0, packed.shape[0], ROPE_STRIDE)
        np.savez_compressed(
            os.path.join(HERE, name + ".npz"),
            size=np.array(size), num_windows=np.array(num), text_tokens=text_tokens, heads=heads,
            head_dim=head_dim, shifted=int(shifted), seed=seed,
            video_qkv=vid.numpy(), text_qkv=txt.numpy(), cu_seqlens=cu.numpy(),
            # Pack is a pure copy: its bytes are pinned by hash. RoPE is pinned on
            # the Q/K rows of every ROPE_STRIDE-th packed position to keep the file small.
            packed_fp32_sha256=sha(packed.numpy()), rope_positions=rope_rows.numpy(),
            roped_qk=roped[rope_rows, :2].numpy(), attended=attended.numpy(),
            video=video.reshape(tokens, heads, head_dim).numpy(), text=text.numpy())
    print("wrote", len(records), "window cases and", len(CHAIN_CASES), "chain cases to", HERE)


if __name__ == "__main__":
    main()

"""Write tests/golden/param_templates.json from the reference's own
normalize_dynamic_awa_template (tools/export_dit_block.py:38-124).

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_param_golden.py --reference <reference checkout>

Each case is an ncnn .param text built here (block graphs shaped the way the
exporter writes its AWA lines, tools/export_dit_block.py:578-644, plus broken
variants); the reference function rewrites a temporary copy of it, and the
fixture records the bytes it wrote or the message it raised. The library's
awa_graph_make_dynamic is checked against these records; the tests never read
the reference.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))


def awa_lines(grid="1 16 16", windows="1 8 8", text=58, shifted=0, suffix="", rope=True, attention=True):
    t, h, w = grid.split()
    wt, wh, ww = windows.split()
    common = f"0={t} 1={h} 2={w} 3={wt} 4={wh} 5={ww} 6={text} 7={shifted}"
    lines = [f"SeedVR2AWAPack awa_pack{suffix} 2 2 vid_qkv{suffix} txt_qkv{suffix} packed{suffix} "
             f"awa_cu_seqlens{suffix} {common}"]
    src = f"packed{suffix}"
    if rope:
        lines.append(f"SeedVR2MMRoPE mmrope{suffix} 1 1 {src} roped{suffix} {common} 8=126")
        src = f"roped{suffix}"
    if attention:
        lines.append(f"SeedVR2WindowAttention awa_attention{suffix} 1 1 {src} attended{suffix} {common}")
        src = f"attended{suffix}"
    else:
        # attention kept as ordinary ncnn layers (a static split/concat pair)
        lines.append(f"Slice attention_split{suffix} 1 1 {src} window_rows{suffix} -23300=1,-233 1=0")
        lines.append(f"Concat attention_concat{suffix} 1 1 window_rows{suffix} attended{suffix} 0=0")
        src = f"attended{suffix}"
    lines.append(f"SeedVR2AWAUnpack awa_unpack{suffix} 1 2 {src} vid_out{suffix} txt_out{suffix} {common}")
    return lines


def block(body, header="7767517", counts=None):
    layers = [
        "Input in_vid 0 1 vid_in",
        "Input in_txt 0 1 txt_in",
        "Gemm gemm_0 1 1 vid_in vid_qkv 10=-1 2=0 3=1 4=0 5=1 6=1 7=0 8=7680 9=2560",
        "MemoryData constant_p_ada_0 0 1 ada_0 0=2560",
        "Gemm gemm_1 1 1 txt_in txt_qkv 10=-1 2=0 3=1 4=0 5=1 6=1 7=0 8=7680 9=2560",
        *body,
        "Reshape reshape_awa_video_batch 1 1 vid_out awa_video_batch 0=2560 1=256",
        "Gemm gemm_2 1 1 awa_video_batch vid_proj 10=-1 2=0 3=1 4=0 5=1 6=1 7=0 8=2560 9=2560",
        "BinaryOp add_0 2 1 vid_proj ada_0 out_vid 0=0 -23303=2,1.5e+00,2.0",
    ]
    lines = [header, counts or f"{len(layers)} {len(layers) * 2}", *layers]
    return "\n".join(lines) + "\n"


def cases():
    out = {}
    out["static_block"] = block(awa_lines())
    out["static_shifted_45x80"] = block(awa_lines("9 45 80", "4 3 3", 58, 1)).replace("1=256", "1=32400")
    out["already_dynamic"] = block(awa_lines("-1 -1 -1")).replace("1=256", "1=-1")
    out["pack_unpack_only"] = block(awa_lines(rope=False, attention=False))
    out["no_attention"] = block(awa_lines(attention=False))
    out["crlf_tabs_spaces"] = block(awa_lines()).replace("\n", "\r\n").replace(
        "SeedVR2MMRoPE mmrope", "SeedVR2MMRoPE\tmmrope").replace("awa_attention 1 1", "awa_attention   1  1")
    out["params_reordered"] = block([
        "SeedVR2AWAPack awa_pack 2 2 vid_qkv txt_qkv packed awa_cu_seqlens 7=0 6=58 2=16 5=8 1=16 4=8 0=1 3=1",
        "SeedVR2MMRoPE mmrope 1 1 packed roped 8=126 0=1 1=16 2=16 3=1 4=8 5=8 6=58 7=0",
        "SeedVR2WindowAttention awa_attention 1 1 roped attended 0=1 1=16 2=16 3=1 4=8 5=8 6=58 7=0",
        "SeedVR2AWAUnpack awa_unpack 1 2 attended vid_out txt_out 0=1 1=16 2=16 3=1 4=8 5=8 6=58 7=0 9=3",
    ])
    out["trailing_whitespace_kept"] = block(awa_lines()).replace("Input in_txt 0 1 txt_in", "Input in_txt 0 1 txt_in  ")
    out["no_final_newline"] = block(awa_lines())[:-1]
    out["reshape_other_name_ignored"] = block(awa_lines()).replace(
        "Reshape reshape_awa_video_batch 1 1 vid_out awa_video_batch 0=2560 1=256",
        "Reshape reshape_awa_video_batch 1 1 vid_out awa_video_batch 0=2560 1=256\n"
        "Reshape reshape_other 1 1 vid_out other 0=2560 1=256")
    # failures the reference raises on
    out["bad_header"] = block(awa_lines(), header="7767518")
    out["one_line"] = "7767517\n"
    out["no_awa"] = block([])
    out["short_layer_line"] = block(awa_lines() + ["Split split"])
    out["bad_blob_counts"] = block(awa_lines() + ["Split split x 1 a b"])
    out["negative_blob_count"] = block(awa_lines() + ["Split split -1 1 a b"])
    out["missing_blobs"] = block(awa_lines() + ["Concat cat 3 1 a b"])
    out["blank_line"] = block(awa_lines() + [""])
    out["unpack_one_output"] = block(awa_lines()[:-1] + [
        "SeedVR2AWAUnpack awa_unpack 1 1 attended vid_out 0=1 1=16 2=16 3=1 4=8 5=8 6=58 7=0"])
    out["duplicate_grid_param"] = block([awa_lines()[0] + " 1=16"] + awa_lines()[1:])
    out["incomplete_grid"] = block([awa_lines()[0].replace(" 2=16", "")] + awa_lines()[1:])
    out["two_unpacks"] = block(awa_lines() + awa_lines(suffix="_1"))
    out["no_reshape"] = block(awa_lines()).replace("reshape_awa_video_batch", "reshape_awa_video_other")
    out["two_reshapes"] = block(awa_lines()).replace(
        "Reshape reshape_awa_video_batch 1 1 vid_out awa_video_batch 0=2560 1=256",
        "Reshape reshape_awa_video_batch 1 1 vid_out awa_video_batch 0=2560 1=256\n"
        "Reshape reshape_awa_video_batch 1 1 vid_out awa_video_batch2 0=2560 1=256")
    out["reshape_two_heights"] = block(awa_lines()).replace("0=2560 1=256", "0=2560 1=256 1=256")
    out["reshape_no_height"] = block(awa_lines()).replace("0=2560 1=256", "0=2560")
    return out


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="root of a reference checkout")
    args = parser.parse_args()
    sys.path.insert(0, args.reference)
    from tools.export_dit_block import normalize_dynamic_awa_template  # noqa: E402
    from pathlib import Path

    records = []
    with tempfile.TemporaryDirectory(dir=HERE) as tmp:
        for name, text in cases().items():
            path = Path(tmp) / f"{name}.ncnn.param"
            path.write_bytes(text.encode())
            record = {"name": name, "input": text}
            try:
                normalize_dynamic_awa_template(path)
                record["output"] = path.read_bytes().decode()
            except ValueError as exc:
                record["error"] = str(exc).replace(str(path), "<path>")
            records.append(record)
    with open(os.path.join(HERE, "param_templates.json"), "w") as f:
        json.dump({"source": "tools/export_dit_block.py:38-124 normalize_dynamic_awa_template", "cases": records},
                  f, indent=1)
        f.write("\n")
    print(f"wrote {len(records)} cases")


if __name__ == "__main__":
    main()

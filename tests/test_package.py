"""Model-package side of the library, host only (no GPU):

* awa_graph_make_dynamic against the reference's normalize_dynamic_awa_template
  (tools/export_dit_block.py:38-124): same bytes out, same failures, on the
  fixture tests/golden/param_templates.json that the reference function wrote;
* awa_graph_find_chains: the ParamDict values and line numbers of each chain,
  plans built from them equal plans built from the same values directly, and
  the graphs that ncnn's loader or the layers' load_param would reject;
* awa_manifest_validate against validate_manifest's rules
  (src/model/model_registry.cpp:248-362), on packages written the way the
  reference's _write_manifest writes them
  (tools/materialize_dynamic_model_package.py:47-54);
* SHA-256 against hashlib.
"""

import hashlib
import json
import os
import tempfile

import numpy as np
import pytest

import awa_b200
from awa_b200 import AwaError

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
with open(os.path.join(ROOT, "tests", "golden", "param_templates.json")) as _f:
    TEMPLATES = {c["name"]: c for c in json.load(_f)["cases"]}


@pytest.fixture
def scratch():
    """A temporary directory inside the checkout (under .pytest_cache)."""
    base = os.path.join(ROOT, ".pytest_cache", "awa_package")
    os.makedirs(base, exist_ok=True)
    with tempfile.TemporaryDirectory(dir=base) as path:
        yield path


# ---------------------------------------------------------------- SHA-256
@pytest.mark.parametrize("size", [0, 1, 3, 55, 56, 57, 63, 64, 65, 119, 120, 127, 128, 1000, 65536 + 7])
def test_sha256_matches_hashlib(size):
    data = np.random.default_rng(size).integers(0, 256, size, dtype=np.uint8).tobytes()
    assert awa_b200.sha256(data) == hashlib.sha256(data).hexdigest()


def test_sha256_file_matches_hashlib(scratch):
    data = np.random.default_rng(5).integers(0, 256, (3 << 20) + 11, dtype=np.uint8).tobytes()
    path = os.path.join(scratch, "blob.bin")
    with open(path, "wb") as f:
        f.write(data)
    assert awa_b200.sha256_file(path) == hashlib.sha256(data).hexdigest()
    with pytest.raises(AwaError, match="failed to open model package artifact"):
        awa_b200.sha256_file(os.path.join(scratch, "absent.bin"))


# ---------------------------------------------------------------- make_dynamic
def _reference_message(message):
    # The reference names the file it read; the text entry point has no path.
    return message.replace(": <path>", "").replace(" in <path>", "")


@pytest.mark.parametrize("name", sorted(TEMPLATES))
def test_make_dynamic_matches_reference(name):
    case = TEMPLATES[name]
    if "output" in case:
        assert awa_b200.graph_make_dynamic(case["input"]) == case["output"]
    else:
        with pytest.raises(AwaError) as err:
            awa_b200.graph_make_dynamic(case["input"])
        assert err.value.code == -1
        assert str(err.value).endswith(_reference_message(case["error"])), (str(err.value), case["error"])


def test_make_dynamic_is_idempotent():
    for case in TEMPLATES.values():
        if "output" in case:
            once = awa_b200.graph_make_dynamic(case["input"])
            assert awa_b200.graph_make_dynamic(once) == once


def test_make_dynamic_reports_the_size_it_needs():
    import ctypes

    lib = awa_b200.library()
    text = TEMPLATES["static_block"]["input"].encode()
    needed = ctypes.c_size_t(0)
    small = ctypes.create_string_buffer(16)
    rc = lib.awa_graph_make_dynamic(text, len(text), ctypes.cast(small, ctypes.c_void_p), 16, ctypes.byref(needed))
    assert rc == awa_b200.AWA_ERR_ALLOC
    assert needed.value == len(TEMPLATES["static_block"]["output"].encode())


# ---------------------------------------------------------------- find_chains
def test_chain_of_static_and_dynamic_block():
    static = awa_b200.graph_find_chains(TEMPLATES["static_block"]["input"])
    dynamic = awa_b200.graph_find_chains(TEMPLATES["static_block"]["output"])
    assert len(static) == len(dynamic) == 1
    s, d = static[0], dynamic[0]
    assert s["params"] == {"source_t": 1, "source_h": 16, "source_w": 16, "windows_t": 1, "windows_h": 8,
                           "windows_w": 8, "text_tokens": 58, "shifted": 0, "rope_dim": 126}
    assert s["dynamic"] == 0 and d["dynamic"] == 1
    assert d["params"]["source_t"] == d["params"]["source_h"] == d["params"]["source_w"] == -1
    # header 2 lines + 5 block layers before the Pack; file lines are 1-based
    assert (s["pack_line"], s["rope_line"], s["attention_line"], s["unpack_line"], s["reshape_line"]) == (8, 9, 10,
                                                                                                        11, 12)
    assert s["reshape_height"] == 256 and d["reshape_height"] == -1


def test_chain_without_rope_and_attention_layers():
    (c,) = awa_b200.graph_find_chains(TEMPLATES["pack_unpack_only"]["input"])
    assert c["rope_line"] == 0 and c["attention_line"] == 0 and c["params"]["rope_dim"] == 126
    # a Pack wired straight into its Unpack does no attention at all
    text = TEMPLATES["pack_unpack_only"]["input"]
    with pytest.raises(AwaError, match="no attention between"):
        awa_b200.graph_find_chains(text.replace("awa_unpack 1 2 attended", "awa_unpack 1 2 packed"))


def test_chain_from_file_and_crlf(scratch):
    path = os.path.join(scratch, "dit_block_00.ncnn.param")
    with open(path, "wb") as f:
        f.write(TEMPLATES["crlf_tabs_spaces"]["input"].encode())
    chains = awa_b200.graph_find_chains_file(path)
    assert chains == awa_b200.graph_find_chains(TEMPLATES["static_block"]["input"])


def test_plan_from_graph_equals_plan_from_params():
    """The dynamic template plus the session's runtime spec gives the same plan
    as the static graph of that resolution (awa_layers.cpp:90-114)."""
    static_text = TEMPLATES["static_shifted_45x80"]["input"]
    dynamic_text = TEMPLATES["static_shifted_45x80"]["output"]
    (s,) = awa_b200.graph_find_chains(static_text)
    (d,) = awa_b200.graph_find_chains(dynamic_text)
    p = s["params"]
    assert (p["source_t"], p["source_h"], p["source_w"], p["shifted"]) == (9, 45, 80, 1)
    plan_static = awa_b200.AwaPlan(**{k: v for k, v in p.items()}, host_only=True)
    plan_dynamic = awa_b200.AwaPlan(**d["params"], runtime_spec=(9, 45, 80), host_only=True)
    a, b = plan_static.maps(), plan_dynamic.maps()
    for key in ("sequence_index", "cu_seqlens", "video_positions", "text_positions"):
        assert np.array_equal(a[key], b[key]), key
    assert a["windows"] == b["windows"]
    # without the runtime spec the dynamic grid is rejected, as load_common does
    with pytest.raises(AwaError):
        awa_b200.AwaPlan(**d["params"], host_only=True)


def two_block_graph():
    """Two consecutive blocks in one graph (the exporter's multi-block rewrite,
    tools/export_dit_block.py:806-831): layer-name suffix per block, odd blocks
    shifted, no video batch reshape."""
    lines = []
    for block, suffix in enumerate(("", "_1")):
        common = f"0=1 1=16 2=16 3=1 4=8 5=8 6=58 7={block % 2}"
        src = "vid_in" if block == 0 else "vid_out"
        lines += [
            f"Gemm gemm_qkv{suffix} 1 1 {src} vid_qkv{suffix} 8=7680 9=2560",
            f"SeedVR2AWAPack awa_pack{suffix} 2 2 vid_qkv{suffix} txt_qkv packed{suffix} cu{suffix} {common}",
            f"SeedVR2MMRoPE mmrope{suffix} 1 1 packed{suffix} roped{suffix} {common} 8=126",
            f"SeedVR2WindowAttention awa_attention{suffix} 1 1 roped{suffix} attended{suffix} {common}",
            f"SeedVR2AWAUnpack awa_unpack{suffix} 1 2 attended{suffix} vid_out{suffix} txt_out{suffix} {common}",
        ]
    lines = ["Input in_vid 0 1 vid_in", "Input in_txt 0 1 txt_qkv"] + lines
    return "\n".join(["7767517", f"{len(lines)} 40", *lines]) + "\n"


def test_multi_block_graph_has_one_chain_per_block():
    chains = awa_b200.graph_find_chains(two_block_graph())
    assert [c["params"]["shifted"] for c in chains] == [0, 1]
    assert chains[0]["unpack_line"] < chains[1]["pack_line"]
    assert all(c["reshape_line"] == 0 for c in chains)


def test_graph_without_awa_layers():
    assert awa_b200.graph_find_chains(TEMPLATES["no_awa"]["input"]) == []


def _mutate(old, new, count=1):
    text = TEMPLATES["static_block"]["input"]
    assert text.count(old) >= count, old
    return text.replace(old, new, count)


BAD_GRAPHS = {
    "header": ("7767517\n", "7767518\n", "unexpected ncnn param header"),
    "layer count": ("\n12 24\n", "\n13 24\n", "declares 13 layers but holds 12"),
    "count line": ("\n12 24\n", "\n12\n", "invalid ncnn layer/blob count line"),
    "partial dynamic grid": ("awa_cu_seqlens 0=1", "awa_cu_seqlens 0=-1", "invalid AWA grid metadata in awa_pack"),
    "zero windows": ("awa_cu_seqlens 0=1 1=16 2=16 3=1", "awa_cu_seqlens 0=1 1=16 2=16 3=0",
                     "invalid AWA grid metadata in awa_pack"),
    "missing text tokens": ("roped attended 0=1 1=16 2=16 3=1 4=8 5=8 6=58", "roped attended 0=1 1=16 2=16 3=1 4=8 5=8",
                            "invalid AWA grid metadata in awa_attention"),
    # three grid values that each fit an int but whose product is near 2^93:
    # the T*H*W <= INT_MAX rule must hold without the product overflowing
    "grid product overflow": ("awa_cu_seqlens 0=1 1=16 2=16", "awa_cu_seqlens 0=2147483647 1=2147483646 2=2147483645",
                              "invalid AWA grid metadata in awa_pack"),
    "grid product just past int": ("awa_cu_seqlens 0=1 1=16 2=16", "awa_cu_seqlens 0=2 1=32768 2=32768",
                                   "invalid AWA grid metadata in awa_pack"),
    "float parameter": ("8=126", "8=126.0", "parameter 8 of mmrope is not an integer"),
    "rope dim": ("8=126", "8=125", "invalid rope dimension 125 in mmrope"),
    "duplicate id": ("8=126", "8=126 5=8", "duplicate AWA parameter 5 in mmrope"),
    "malformed pair": ("8=126", "8=126 junk", "invalid parameter 'junk' in mmrope"),
    "pack arity": ("awa_pack 2 2 vid_qkv txt_qkv packed awa_cu_seqlens", "awa_pack 2 1 vid_qkv txt_qkv packed",
                   "SeedVR2AWAPack awa_pack must have 2 inputs and 2 outputs"),
    "parameters disagree": ("attended 0=1 1=16 2=16 3=1 4=8 5=8 6=58 7=0", "attended 0=1 1=16 2=16 3=1 4=8 5=8 6=57 7=0",
                            "awa_attention disagrees with awa_pack on parameter 6"),
    "shift disagrees": ("vid_out txt_out 0=1 1=16 2=16 3=1 4=8 5=8 6=58 7=0",
                        "vid_out txt_out 0=1 1=16 2=16 3=1 4=8 5=8 6=58 7=1",
                        "awa_unpack disagrees with awa_pack on parameter 7"),
    "rope wiring": ("mmrope 1 1 packed roped", "mmrope 1 1 vid_qkv roped", "does not read awa_pack's packed output"),
    "attention wiring": ("awa_attention 1 1 roped", "awa_attention 1 1 packed", "does not read mmrope's output"),
    "unpack wiring": ("awa_unpack 1 2 attended", "awa_unpack 1 2 roped", "does not read awa_attention's output"),
    "reshape height": ("0=2560 1=256", "0=2560 1=255", "height 255 does not match the 256 video tokens"),
    "reshape two heights": ("0=2560 1=256", "0=2560 1=256 1=256", "must have exactly one integer height parameter"),
}


@pytest.mark.parametrize("name", sorted(BAD_GRAPHS))
def test_find_chains_rejects(name):
    old, new, message = BAD_GRAPHS[name]
    with pytest.raises(AwaError, match=message.replace("(", r"\(").replace(")", r"\)")) as err:
        awa_b200.graph_find_chains(_mutate(old, new))
    assert err.value.code == -1


def test_find_chains_rejects_unpaired_and_stray_layers():
    text = two_block_graph()
    lines = text.splitlines()
    # drop the second Unpack
    dropped = [ln for ln in lines if not ln.startswith("SeedVR2AWAUnpack awa_unpack_1")]
    dropped[1] = f"{len(dropped) - 2} 40"
    with pytest.raises(AwaError, match="2 SeedVR2AWAPack layers but 1 SeedVR2AWAUnpack"):
        awa_b200.graph_find_chains("\n".join(dropped) + "\n")
    # an MMRoPE after the last Unpack belongs to no chain
    stray = lines + ["SeedVR2MMRoPE stray 1 1 x y 0=1 1=16 2=16 3=1 4=8 5=8 6=58 7=0"]
    stray[1] = f"{len(stray) - 2} 40"
    with pytest.raises(AwaError, match="stray lies outside every Pack..Unpack chain"):
        awa_b200.graph_find_chains("\n".join(stray) + "\n")


# ---------------------------------------------------------------- manifest
def _write_package(root, files, extra_lines=(), upper=False, crlf=False):
    """Files plus a manifest.sha256 in the reference's writer format."""
    for name, data in files.items():
        path = os.path.join(root, name)
        os.makedirs(os.path.dirname(path), exist_ok=True)
        with open(path, "wb") as f:
            f.write(data)
    lines = []
    for name in sorted(files):
        digest = hashlib.sha256(files[name]).hexdigest()
        lines.append(f"{digest.upper() if upper else digest}  {name}")
    lines.extend(extra_lines)
    end = "\r\n" if crlf else "\n"
    with open(os.path.join(root, "manifest.sha256"), "w", newline="") as f:
        f.write(end.join(lines) + end)


def _files(count=75):
    rng = np.random.default_rng(count)
    names = [f"dit_block_{i:02d}.ncnn.param" for i in range(count - 3)] + ["vae_encode.ncnn.bin",
                                                                           "conditioning/pos_emb.bin", "dit_input.ncnn.param"]
    return {n: rng.integers(0, 256, int(rng.integers(0, 3000)), dtype=np.uint8).tobytes() for n in names}


def test_manifest_of_a_75_record_package(scratch):
    _write_package(scratch, _files(75))
    awa_b200.manifest_validate(scratch)
    awa_b200.manifest_validate(scratch, 75)
    with pytest.raises(AwaError, match="must contain 74 records, got 75"):
        awa_b200.manifest_validate(scratch, 74)


def test_manifest_accepts_crlf_uppercase_and_blank_lines(scratch):
    files = _files(5)
    _write_package(scratch, files, extra_lines=("", ""), upper=True, crlf=True)
    awa_b200.manifest_validate(scratch, -1)
    with pytest.raises(AwaError, match=r"must contain 75 records \(positive\) or 146 records \(positive \+ CFG\), got 5"):
        awa_b200.manifest_validate(scratch)


MANIFEST_FAULTS = {
    "missing manifest": "missing model package manifest",
    "short separator": "invalid model package manifest record at line 1",
    "non-hex digest": "invalid model package manifest record at line 2",
    "parent path": "invalid model package manifest path at line 6",
    "absolute path": "invalid model package manifest path at line 6",
    "dot component": "invalid model package manifest path at line 6",
    "backslash": "invalid model package manifest path at line 6",
    "double slash": "invalid model package manifest path at line 6",
    "trailing slash": "manifest artifact is missing: sub/",
    "duplicate record": "duplicate model package manifest path: a.bin",
    "missing artifact": "manifest artifact is missing: zz.bin",
    "hash mismatch": "manifest hash mismatch for artifact: b.bin",
    "unlisted artifact": "artifact is not listed in model package manifest: ",
    "symbolic link": "model package must not contain symbolic links: ",
}


@pytest.mark.parametrize("fault", sorted(MANIFEST_FAULTS))
def test_manifest_rejects(fault, scratch):
    files = {"a.bin": b"alpha", "b.bin": b"beta", "sub/c.bin": b"gamma", "sub/d.bin": b"", "e.bin": b"e" * 70000}
    good = hashlib.sha256(b"x").hexdigest()
    extra = {
        "parent path": [f"{good}  ../a.bin"],
        "absolute path": [f"{good}  /a.bin"],
        "dot component": [f"{good}  sub/./c.bin"],
        "backslash": [f"{good}  sub\\c.bin"],
        "double slash": [f"{good}  sub//c.bin"],
        "trailing slash": [f"{good}  sub/"],
        "duplicate record": [f"{hashlib.sha256(b'alpha').hexdigest()}  a.bin"],
        "missing artifact": [f"{good}  zz.bin"],
    }.get(fault, [])
    _write_package(scratch, files, extra_lines=extra)
    manifest = os.path.join(scratch, "manifest.sha256")
    if fault == "missing manifest":
        os.remove(manifest)
    elif fault in ("short separator", "non-hex digest"):
        lines = open(manifest).read().splitlines()
        index = 0 if fault == "short separator" else 1
        lines[index] = lines[index].replace("  ", " ", 1) if fault == "short separator" else "g" + lines[index][1:]
        open(manifest, "w").write("\n".join(lines) + "\n")
    elif fault == "hash mismatch":
        open(os.path.join(scratch, "b.bin"), "wb").write(b"BETA")
    elif fault == "unlisted artifact":
        open(os.path.join(scratch, "sub", "new.bin"), "wb").write(b"new")
    elif fault == "symbolic link":
        os.symlink(os.path.join(scratch, "a.bin"), os.path.join(scratch, "link.bin"))
    with pytest.raises(AwaError, match=MANIFEST_FAULTS[fault].replace("\\", "\\\\")) as err:
        awa_b200.manifest_validate(scratch, -1)
    assert err.value.code == -1

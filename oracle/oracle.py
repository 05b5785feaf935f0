"""ctypes access to the AWA parity checkers (TEST INFRASTRUCTURE ONLY).

Two CPU implementations of the SeedVR2-ncnn AWA chain live here:

* ``Oracle``: the C restatement in ``awa_oracle.c`` (always built).
* ``Reference``: the reference's own ``src/awa/awa_layers.cpp`` compiled
  unmodified against the library's ncnn API subset
  (``seedvr2-ncnn_b200/ncnn_compat/ncnn``; ``_ref/libawa_ref.so``, built only
  where a reference checkout is given, then carried with the repository copy).

Only ``tests/``, ``__graft_entry__`` (build and smoke) and ``bench.py``'s
CPU-baseline and reference legs import this module; the product never does.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libawa_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libawa_ref.so")
REF_BATCH_SO = os.path.join(HERE, "_ref", "libawa_ref_batch.so")  # built with NCNN_BATCH=1
# Root of a reference checkout (its src/awa/awa_layers.cpp is compiled into
# _ref/); unset means "use the prebuilt _ref/ library if it is there".
REFERENCE_ROOT = os.environ.get("SEEDVR2_REFERENCE_ROOT", "")

_i = ctypes.c_int
_p = ctypes.c_void_p


def build(reference: bool = True, reference_root: Optional[str] = None) -> None:
    """Compile the C restatement, and the reference's CPU forward when a
    reference checkout is given (argument, else SEEDVR2_REFERENCE_ROOT) and
    holds src/awa/awa_layers.cpp."""
    root = reference_root or REFERENCE_ROOT
    targets = ["oracle"]
    if reference and root and os.path.isfile(os.path.join(root, "src", "awa", "awa_layers.cpp")):
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", HERE, f"REFERENCE={root}", *targets], check=True)


def _ptr(array: Optional[np.ndarray]):
    if array is None:
        return None
    assert array.flags["C_CONTIGUOUS"]
    return array.ctypes.data_as(_p)


@dataclass(frozen=True)
class LayerConfig:
    """ParamDict ids 0-8 of the four AWA layers plus the blob geometry."""

    source_t: int
    source_h: int
    source_w: int
    num_t: int
    num_h: int
    num_w: int
    text_tokens: int = 58
    shifted: int = 0
    rope_dim: int = 126
    heads: int = 20
    head_dim: int = 128

    @property
    def source_tokens(self) -> int:
        return self.source_t * self.source_h * self.source_w

    @property
    def params(self) -> List[int]:
        return [self.source_t, self.source_h, self.source_w, self.num_t, self.num_h, self.num_w,
                self.text_tokens, self.shifted, self.rope_dim]


class Oracle:
    """The C restatement (awa_oracle.c)."""

    def __init__(self, path: str = ORACLE_SO) -> None:
        if not os.path.isfile(path):
            build(reference=False)
        lib = ctypes.CDLL(path)
        i7 = [_i] * 7
        sig = {
            "oracle_make_windows": (_i, i7 + [_p, _i]),
            "oracle_index_maps": (_i, i7 + [_i, _p, _p, _p, _p]),
            "oracle_pack": (None, [_p, _p, _i, _i, _i, _p, _i, _p]),
            "oracle_rope_table": (_i, i7 + [_i, _i, _p]),
            "oracle_rope": (None, [_p, _i, _i, _i, _i, _p, _p]),
            "oracle_attention": (None, [_p, _i, _p, _i, _i, _p, _i]),
            "oracle_attention_range": (None, [_p, _i, _i, _p, _i, _i, _p, _i]),
            "oracle_unpack": (_i, [_p, _i, _i, _i, _i, _i, _i, _p, _p, _p, _p]),
            "oracle_round_bf16": (None, [_p, _p, ctypes.c_int64]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        self.lib = lib

    def make_windows(self, size: Sequence[int], num: Sequence[int], shifted: bool) -> List[Tuple[int, ...]]:
        n = self.lib.oracle_make_windows(*size, *num, int(shifted), None, 0)
        out = np.zeros((max(n, 1), 6), dtype=np.int32)
        self.lib.oracle_make_windows(*size, *num, int(shifted), _ptr(out), n)
        return [tuple(int(v) for v in row) for row in out[:n]]

    def index_maps(self, cfg: LayerConfig):
        windows = self.make_windows((cfg.source_t, cfg.source_h, cfg.source_w),
                                    (cfg.num_t, cfg.num_h, cfg.num_w), bool(cfg.shifted))
        count = len(windows)
        seq_len = sum((w[1] - w[0]) * (w[3] - w[2]) * (w[5] - w[4]) + cfg.text_tokens for w in windows)
        seq = np.zeros(seq_len, np.int32)
        cu = np.zeros(count + 1, np.int32)
        vpos = np.zeros(cfg.source_tokens, np.int32)
        tpos = np.zeros(count * cfg.text_tokens, np.int32)
        s = self.lib.oracle_index_maps(*cfg.params[:6], cfg.text_tokens, cfg.shifted, _ptr(seq), _ptr(cu),
                                       _ptr(vpos), _ptr(tpos))
        assert s == seq_len
        return {"windows": windows, "sequence_index": seq, "cu_seqlens": cu,
                "video_positions": vpos, "text_positions": tpos}

    def chain(self, cfg: LayerConfig, video_qkv: np.ndarray, text_qkv: np.ndarray, threads: int = 0):
        """Pack -> MMRoPE -> WindowAttention -> Unpack; returns every intermediate."""
        maps = self.index_maps(cfg)
        heads, d = cfg.heads, cfg.head_dim
        video_qkv = np.ascontiguousarray(video_qkv, dtype=np.float32)
        text_qkv = np.ascontiguousarray(text_qkv, dtype=np.float32)
        seq_len = len(maps["sequence_index"])
        packed = np.empty((seq_len, 3, heads, d), np.float32)
        self.lib.oracle_pack(_ptr(video_qkv), _ptr(text_qkv), cfg.source_tokens, heads, d,
                             _ptr(maps["sequence_index"]), seq_len, _ptr(packed))
        table = self.rope_table(cfg)
        roped = np.empty_like(packed)
        self.lib.oracle_rope(_ptr(packed), seq_len, heads, d, cfg.rope_dim, _ptr(table), _ptr(roped))
        attended = np.empty((seq_len, heads, d), np.float32)
        threads = threads or (os.cpu_count() or 1)
        self.lib.oracle_attention(_ptr(roped), len(maps["windows"]), _ptr(maps["cu_seqlens"]), heads, d,
                                  _ptr(attended), threads)
        video = np.empty((cfg.source_tokens, heads, d), np.float32)
        text = np.empty((cfg.text_tokens, heads, d), np.float32)
        rc = self.lib.oracle_unpack(_ptr(attended), seq_len, cfg.source_tokens, heads, d, len(maps["windows"]),
                                    cfg.text_tokens, _ptr(maps["video_positions"]), _ptr(maps["text_positions"]),
                                    _ptr(video), _ptr(text))
        assert rc == 0
        return {"packed": packed, "cu_seqlens": maps["cu_seqlens"].astype(np.float32), "roped": roped,
                "attended": attended, "video": video, "text": text, "maps": maps}

    def rope_table(self, cfg: LayerConfig) -> np.ndarray:
        maps_len = self.lib.oracle_index_maps(*cfg.params[:6], cfg.text_tokens, cfg.shifted, None, None, None, None)
        table = np.empty((maps_len, 2 * cfg.rope_dim), np.float32)
        rc = self.lib.oracle_rope_table(*cfg.params[:6], cfg.text_tokens, cfg.shifted, cfg.rope_dim, _ptr(table))
        assert rc == maps_len
        return table

    def rope(self, packed: np.ndarray, table: np.ndarray, heads: int, head_dim: int, rope_dim: int) -> np.ndarray:
        """MMRoPE of packed rows [n, 3, H, d] with their table rows [n, 2*rope_dim]."""
        packed = np.ascontiguousarray(packed, dtype=np.float32)
        table = np.ascontiguousarray(table, dtype=np.float32)
        out = np.empty_like(packed)
        self.lib.oracle_rope(_ptr(packed), packed.shape[0], heads, head_dim, rope_dim, _ptr(table), _ptr(out))
        return out

    def attention_range(self, packed: np.ndarray, cu: np.ndarray, first: int, last: int, heads: int, head_dim: int,
                        attended: np.ndarray, threads: int = 1) -> None:
        cu = np.ascontiguousarray(cu, dtype=np.int32)
        packed = np.ascontiguousarray(packed, dtype=np.float32)
        assert attended.flags["C_CONTIGUOUS"] and attended.dtype == np.float32
        self.lib.oracle_attention_range(_ptr(packed), first, last, _ptr(cu), heads, head_dim, _ptr(attended), threads)

    def round_bf16(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty_like(x)
        self.lib.oracle_round_bf16(_ptr(x), _ptr(out), ctypes.c_int64(x.size))
        return out


def round_bf16_rne(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest bf16 (ties to even), returned as fp32 (finite inputs)."""
    bits = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounded = (bits + np.uint32(0x7FFF) + ((bits >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return rounded.view(np.float32)


def qkv_project(x: np.ndarray, w: np.ndarray, gamma_q: np.ndarray, gamma_k: np.ndarray, eps: float, heads: int,
                head_dim: int = 128) -> np.ndarray:
    """The producer of the AWA input: a DiT block's QKV projection and the
    per-head RMSNorm of Q and K (tools/reference/dit_block.py:280-287).

    proj_qkv is a bias-free Linear (dit_block.py:252-253) whose output, in the
    bf16 blocks, is bf16: x @ w.T accumulated in fp32, rounded to bf16.
    norm_q / norm_k are nn.RMSNorm(head_dim, eps, affine) (FixedRMSNorm,
    dit_block.py:157-166), computed as DitRMSNorm does (src/dit/
    dit_precision.cpp:22-90, shader dit_rmsnorm.comp:23-48): fp32 squares and
    sum, inversesqrt(sum / head_dim + eps), times gamma; V is left as is.
    x [tokens, model_dim] and w [3*heads*head_dim, model_dim] hold bf16 values
    as fp32. Returns [tokens, 3, heads, head_dim] fp32.
    """
    acc = np.asarray(x, np.float32) @ np.asarray(w, np.float32).T
    y = round_bf16_rne(acc).reshape(acc.shape[0], 3, heads, head_dim)
    for part, gamma in ((0, gamma_q), (1, gamma_k)):
        v = y[:, part]
        ss = np.einsum("thd,thd->th", v, v, dtype=np.float32)
        coef = (np.float32(1) / np.sqrt(ss / np.float32(head_dim) + np.float32(eps))).astype(np.float32)
        y[:, part] = v * coef[..., None] * np.asarray(gamma, np.float32)
    return y


def out_project(x: np.ndarray, w: np.ndarray, bias: np.ndarray, gate: np.ndarray, residual: np.ndarray) -> np.ndarray:
    """The consumer of the AWA output: a DiT block's proj_out, Ada "out" gate
    and residual (tools/reference/dit_block.py:299 -- nn.Linear with bias, bf16
    output in the bf16 blocks; FixedAdaBranch.forward mode "out" :187-190 --
    hidden * (gate_a + gate_b); FixedDitBlock.forward :345-347 -- + the block
    input). x [tokens, in_dim], w [out_dim, in_dim] hold bf16 values as fp32;
    gate is gate_a + gate_b. Returns [tokens, out_dim] fp32: the product and the
    sum each rounded to fp32."""
    linear = round_bf16_rne(np.asarray(x, np.float32) @ np.asarray(w, np.float32).T + np.asarray(bias, np.float32))
    gated = (linear * np.asarray(gate, np.float32)).astype(np.float32)
    return (gated + np.asarray(residual, np.float32)).astype(np.float32)


class Reference:
    """The reference's own awa_layers.cpp CPU forward (oracle/_ref)."""

    def __init__(self, path: str = REF_SO) -> None:
        if not os.path.isfile(path):
            build(reference=True)
        if not os.path.isfile(path):
            raise FileNotFoundError(path)
        lib = ctypes.CDLL(path)
        lib.ref_make_windows.restype = _i
        lib.ref_chain_create.restype = _p
        lib.ref_chain_create.argtypes = [_p, _i, _i, _i, _i, ctypes.POINTER(_i)]
        lib.ref_chain_forward.restype = _i
        lib.ref_chain_forward.argtypes = [_p] * 9
        lib.ref_chain_destroy.argtypes = [_p]
        lib.ref_chain_seconds.argtypes = [_p, _p]
        lib.ref_layer_forward.restype = _i
        lib.ref_layer_forward.argtypes = [_p, _i, _p, _p, _i, _i, _p, _p]
        lib.ref_batch_build.restype = _i
        self.lib = lib
        self.batch_build = bool(lib.ref_batch_build())

    @staticmethod
    def available(path: str = REF_SO) -> bool:
        return os.path.isfile(path)

    def make_windows(self, size: Sequence[int], num: Sequence[int], shifted: bool) -> List[Tuple[int, ...]]:
        n = self.lib.ref_make_windows(*size, *num, int(shifted), None, 0)
        out = np.zeros((max(n, 1), 6), dtype=np.int32)
        self.lib.ref_make_windows(*size, *num, int(shifted), _ptr(out), n)
        return [tuple(int(v) for v in row) for row in out[:n]]

    def create(self, cfg: LayerConfig, layout: int = 0, runtime_spec: bool = False):
        params = (_i * 9)(*cfg.params)
        status = _i(0)
        handle = self.lib.ref_chain_create(ctypes.cast(params, _p), cfg.heads, cfg.head_dim, layout,
                                           int(runtime_spec), ctypes.byref(status))
        return handle, status.value

    def chain(self, cfg: LayerConfig, video_qkv: np.ndarray, text_qkv: np.ndarray, layout: int = 0,
              runtime_spec: bool = False):
        handle, status = self.create(cfg, layout, runtime_spec)
        if not handle:
            raise RuntimeError(f"reference load_param failed: {status}")
        try:
            windows = self.make_windows((cfg.source_t, cfg.source_h, cfg.source_w),
                                        (cfg.num_t, cfg.num_h, cfg.num_w), bool(cfg.shifted))
            seq_len = sum((w[1] - w[0]) * (w[3] - w[2]) * (w[5] - w[4]) + cfg.text_tokens for w in windows)
            h, d = cfg.heads, cfg.head_dim
            out = {
                "packed": np.empty((seq_len, 3, h, d), np.float32),
                "cu_seqlens": np.empty(len(windows) + 1, np.float32),
                "roped": np.empty((seq_len, 3, h, d), np.float32),
                "attended": np.empty((seq_len, h, d), np.float32),
                "video": np.empty((cfg.source_tokens, h, d), np.float32),
                "text": np.empty((cfg.text_tokens, h, d), np.float32),
            }
            v = np.ascontiguousarray(video_qkv, np.float32)
            t = np.ascontiguousarray(text_qkv, np.float32)
            rc = self.lib.ref_chain_forward(handle, _ptr(v), _ptr(t), *(_ptr(out[k]) for k in
                                            ("packed", "cu_seqlens", "roped", "attended", "video", "text")))
            if rc != 0:
                raise RuntimeError(f"reference forward failed: {rc}")
            secs = (ctypes.c_double * 4)()
            self.lib.ref_chain_seconds(handle, ctypes.cast(secs, _p))
            out["seconds"] = list(secs)
            return out
        finally:
            self.lib.ref_chain_destroy(handle)

"""Python binding of the B200 AWA library (include/awa_b200.h) over ctypes.

The library is the CUDA implementation of SeedVR2-ncnn's adaptive window
attention layers (src/awa): ``AwaPlan`` is what the four ncnn layers build in
``load_param``; its methods are the layers' forwards (``pack``, ``mmrope``,
``window_attention``, ``unpack``) and the fused chain (``forward``). Tensors
are torch CUDA tensors; torch is used only for device memory and streams.

There is no CPU fallback: importing this module on a machine without the
built library raises, and every call needs a CUDA device.
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libawa_b200.so")
COMPAT_PATH = os.path.join(PKG_DIR, "lib", "libawa_ncnn_compat.so")
COMPAT_BATCH_PATH = os.path.join(PKG_DIR, "lib", "libawa_ncnn_compat_batch.so")  # built with NCNN_BATCH

AWA_F32 = 0
AWA_BF16 = 1
AWA_PREC_FP32 = 0
AWA_PREC_BF16 = 1
AWA_OK = 0
AWA_ERR_INVALID = -1
AWA_ERR_CUDA = -2
AWA_ERR_DEVICE = -3
AWA_ERR_ALLOC = -100
AWA_NOALLOC_SCRATCH_BYTES = 32 << 20  # scratch of awa_forward_noalloc, per GPU
AWA_BRANCH_VIDEO = 0
AWA_BRANCH_TEXT = 1
AWA_PUSH_AUTO = 0
AWA_PUSH_COPY_ENGINES = 1
AWA_PUSH_KERNEL = 2

# Every symbol declared in include/awa_b200.h, include/awa_package.h and include/awa_stack.h.
EXPORTED_SYMBOLS = (
    "awa_make_windows", "awa_plan_create", "awa_plan_create_host", "awa_plan_destroy", "awa_plan_get_info", "awa_plan_get_maps",
    "awa_pack", "awa_mmrope", "awa_window_attention", "awa_unpack", "awa_forward_workspace_bytes", "awa_forward",
    "awa_forward_workspace_bytes_for",
    "awa_forward_noalloc", "awa_forward_prerotated", "awa_qkv_project_rotated", "awa_forward_host",
    "awa_forward_host_workspace_bytes",
    "awa_forward_windows", "awa_text_finalize", "awa_scatter_video_shard", "awa_gather_video_shard",
    "awa_window_range_video_rows", "awa_partition_windows", "awa_qkv_project", "awa_out_project", "awa_device_status",
    "awa_selftest_bounded_wait", "awa_attention_kernel_kind",
    "awa_comm_unique_id", "awa_comm_create", "awa_comm_wrap", "awa_comm_destroy", "awa_comm_info", "awa_shard_split",
    "awa_comm_alloc_shared", "awa_comm_free_shared", "awa_shard_windows", "awa_comm_set_push", "awa_shard_runs",
    "awa_forward_sharded_workspace_bytes", "awa_forward_sharded",
    "awa_profile_enable", "awa_profile_reset", "awa_profile_collect", "awa_last_error", "awa_version",
    "awa_graph_find_chains", "awa_graph_find_chains_file", "awa_graph_make_dynamic", "awa_manifest_validate",
    "awa_sha256", "awa_sha256_file",
    "awa_stack_create", "awa_stack_destroy", "awa_stack_get_info", "awa_stack_block_plan", "awa_stack_forward_block",
    "awa_stack_run", "awa_stack_capture", "awa_stack_graph_launch", "awa_stack_graph_destroy",
)


class AwaError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"awa error {code}: {message}")
        self.code = code


class _LayerParams(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("source_t", "source_h", "source_w", "windows_t", "windows_h",
                                             "windows_w", "text_tokens", "shifted", "rope_dim")]


class _RuntimeSpec(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("source_t", "source_h", "source_w", "video_tokens")]


class _Window(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("t0", "t1", "h0", "h1", "w0", "w1")]


class _GraphChain(ctypes.Structure):
    _fields_ = [("params", _LayerParams)] + [(n, ctypes.c_int) for n in (
        "dynamic", "pack_line", "rope_line", "attention_line", "unpack_line", "reshape_line", "reshape_height")]


class StackIO(ctypes.Structure):
    """awa_stack_io: one block's AWA input and output (include/awa_stack.h)."""
    _fields_ = [("block", ctypes.c_int), ("precision", ctypes.c_int), ("in_dtype", ctypes.c_int),
                ("video_qkv", ctypes.c_void_p), ("video_token_stride", ctypes.c_int64),
                ("video_qkv_stride", ctypes.c_int64), ("text_qkv", ctypes.c_void_p),
                ("text_token_stride", ctypes.c_int64), ("text_qkv_stride", ctypes.c_int64),
                ("out_dtype", ctypes.c_int), ("video_out", ctypes.c_void_p), ("video_out_stride", ctypes.c_int64),
                ("text_out", ctypes.c_void_p), ("text_out_stride", ctypes.c_int64)]


# int (*awa_stack_hook)(void* user, int stage, awa_stack_io* io, awa_stream_t stream)
STACK_HOOK = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(StackIO), ctypes.c_void_p)
AWA_STACK_BEFORE = 0
AWA_STACK_AFTER = 1


class _PlanInfo(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("source_t", "source_h", "source_w", "source_tokens", "text_tokens",
                                             "window_count", "sequence_tokens", "max_window_length", "rope_dim",
                                             "shifted", "device")]


_lib = None


def library() -> ctypes.CDLL:
    """Load lib/libawa_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.isfile(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {PKG_DIR}` (no CPU fallback exists)")
    lib = ctypes.CDLL(LIB_PATH)
    i, p, i64, sz = ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_size_t
    sig = {
        "awa_make_windows": (i, [i, i, i, i, i, i, i, p, i]),
        "awa_plan_create": (i, [p, p, ctypes.POINTER(p)]),
        "awa_plan_create_host": (i, [p, p, ctypes.POINTER(p)]),
        "awa_plan_destroy": (None, [p]),
        "awa_plan_get_info": (i, [p, p]),
        "awa_plan_get_maps": (i, [p, p, p, p, p, p]),
        "awa_pack": (i, [p, i, i, i, p, i64, i64, p, i64, i64, i, p, i64, p, p]),
        "awa_mmrope": (i, [p, i, i, i, p, i64, i, p, i64, p]),
        "awa_window_attention": (i, [p, i, i, i, i, p, i64, i, p, i64, p]),
        "awa_unpack": (i, [p, i, i, i, p, i64, i, p, i64, p, i64, p]),
        "awa_forward_workspace_bytes": (sz, [p, i, i]),
        "awa_forward_workspace_bytes_for": (sz, [p, i, i, i, i]),
        "awa_forward": (i, [p, i, i, i, i, p, i64, i64, p, i64, i64, i, p, i64, p, i64, p, sz, p]),
        "awa_forward_noalloc": (i, [p, i, i, i, i, p, i64, i64, p, i64, i64, i, p, i64, p, i64, p]),
        "awa_forward_prerotated": (i, [p, i, i, i, i, p, i64, i64, p, i64, i64, i, p, i64, p, i64, p, sz, p]),
        "awa_forward_host": (i, [p, i, i, i, i, p, i64, i64, p, i64, i64, i, p, i64, p, i64, p, sz, p]),
        "awa_forward_host_workspace_bytes": (sz, [p, i, i, i, i, i]),
        "awa_qkv_project_rotated": (i, [i, i, i, i, p, i64, p, i64, p, p, ctypes.c_float, p, i, i, p, i64, p]),
        "awa_qkv_project": (i, [i, i, i, i, p, i64, p, i64, p, p, ctypes.c_float, i, p, i64, p]),
        "awa_out_project": (i, [i, i, i, p, i64, p, i64, p, p, p, i64, i, i, p, i64, p]),
        "awa_forward_windows": (i, [p, i, i, i, i, i, i, p, i64, i64, p, i64, i64, i, p, i64, p, p, sz, p]),
        "awa_text_finalize": (i, [p, i, i, p, i, p, i64, p]),
        "awa_scatter_video_shard": (i, [p, i, i, i, i, i, p, p, i64, p]),
        "awa_gather_video_shard": (i, [p, i, i, i, i, i, p, i64, p, p]),
        "awa_window_range_video_rows": (i64, [p, i, i]),
        "awa_partition_windows": (i, [p, i, p]),
        "awa_device_status": (i, []),
        "awa_selftest_bounded_wait": (i, [ctypes.c_uint, ctypes.POINTER(i), p]),
        "awa_comm_unique_id": (i, [p, sz]),
        "awa_comm_create": (i, [p, sz, i, i, ctypes.POINTER(p)]),
        "awa_comm_wrap": (i, [p, ctypes.POINTER(p)]),
        "awa_comm_destroy": (None, [p]),
        "awa_comm_alloc_shared": (i, [p, sz, ctypes.POINTER(p)]),
        "awa_comm_free_shared": (i, [p, p]),
        "awa_comm_set_push": (i, [p, i]),
        "awa_comm_info": (i, [p, ctypes.POINTER(i), ctypes.POINTER(i)]),
        "awa_shard_split": (i, [p, i, i, ctypes.POINTER(i), p]),
        "awa_shard_windows": (i, [p, i, i, i, p, i]),
        "awa_shard_runs": (i, [p, i, i, i, p, i]),
        "awa_forward_sharded_workspace_bytes": (sz, [p, i, i, i, i]),
        "awa_forward_sharded": (i, [p, p, i, i, i, i, p, i64, i64, p, i64, i64, i, p, i64, p, i64, p, sz, p]),
        "awa_attention_kernel_kind": (i, [p, i, i, i, i]),
        "awa_profile_enable": (None, [i]),
        "awa_profile_reset": (None, []),
        "awa_profile_collect": (i, [p, sz]),
        "awa_last_error": (ctypes.c_char_p, []),
        "awa_version": (ctypes.c_char_p, []),
        "awa_graph_find_chains": (i, [ctypes.c_char_p, sz, p, i]),
        "awa_graph_find_chains_file": (i, [ctypes.c_char_p, p, i]),
        "awa_graph_make_dynamic": (i, [ctypes.c_char_p, sz, p, sz, ctypes.POINTER(sz)]),
        "awa_manifest_validate": (i, [ctypes.c_char_p, i]),
        "awa_sha256": (i, [ctypes.c_char_p, sz, p]),
        "awa_sha256_file": (i, [ctypes.c_char_p, p]),
        "awa_stack_create": (i, [p, i, p, i, i, i, ctypes.POINTER(p)]),
        "awa_stack_destroy": (None, [p]),
        "awa_stack_get_info": (i, [p, p, p]),
        "awa_stack_block_plan": (p, [p, i]),
        "awa_stack_forward_block": (i, [p, i, p, p]),
        "awa_stack_run": (i, [p, STACK_HOOK, p, p]),
        "awa_stack_capture": (i, [p, STACK_HOOK, p, p, ctypes.POINTER(p)]),
        "awa_stack_graph_launch": (i, [p, p]),
        "awa_stack_graph_destroy": (None, [p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def _check(rc: int) -> None:
    if rc != AWA_OK:
        raise AwaError(rc, library().awa_last_error().decode())


def make_windows(size: Sequence[int], num_windows: Sequence[int], shifted: bool) -> List[Tuple[int, ...]]:
    """Window bounds (t0, t1, h0, h1, w0, w1) in layer order (host only, no GPU needed)."""
    lib = library()
    n = lib.awa_make_windows(*size, *num_windows, int(shifted), None, 0)
    arr = (_Window * max(n, 1))()
    lib.awa_make_windows(*size, *num_windows, int(shifted), ctypes.cast(arr, ctypes.c_void_p), n)
    return [(w.t0, w.t1, w.h0, w.h1, w.w0, w.w1) for w in arr[:n]]


def _torch():
    import torch

    return torch


def _dtype_code(t) -> int:
    torch = _torch()
    if t.dtype == torch.float32:
        return AWA_F32
    if t.dtype == torch.bfloat16:
        return AWA_BF16
    raise TypeError(f"unsupported dtype {t.dtype}")


def _torch_dtype(code: int):
    torch = _torch()
    return torch.float32 if code == AWA_F32 else torch.bfloat16


def _stream_ptr(stream) -> Optional[int]:
    torch = _torch()
    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream


def _qkv_strides(t) -> Tuple[int, int]:
    """(token_stride, qkv_stride) of a [tokens, 3, H, d] view with dense (H, d)."""
    if t.dim() != 4 or t.shape[1] != 3 or t.stride(3) != 1 or t.stride(2) != t.shape[3]:
        raise ValueError("QKV tensors must be [tokens, 3, heads, head_dim] with dense heads x head_dim")
    return t.stride(0), t.stride(1)


@dataclass(frozen=True)
class PlanInfo:
    source_t: int
    source_h: int
    source_w: int
    source_tokens: int
    text_tokens: int
    window_count: int
    sequence_tokens: int
    max_window_length: int
    rope_dim: int
    shifted: int
    device: int


class AwaPlan:
    """Index maps, window table and RoPE table of one AWA layer configuration.

    Arguments are the layers' ParamDict ids 0-8 (awa_layers.cpp:90-114, 872):
    grid (``-1, -1, -1`` with ``runtime_spec`` = grid of the session), window
    counts, text token count, shift flag and rotated feature count.
    """

    def __init__(self, source_t: int, source_h: int, source_w: int, windows_t: int, windows_h: int,
                 windows_w: int, text_tokens: int = 58, shifted: bool = False, rope_dim: int = 126,
                 runtime_spec: Optional[Tuple[int, int, int]] = None, host_only: bool = False):
        lib = library()
        params = _LayerParams(source_t, source_h, source_w, windows_t, windows_h, windows_w, text_tokens,
                              int(bool(shifted)), rope_dim)
        spec = None
        if runtime_spec is not None:
            t, h, w = runtime_spec
            spec = _RuntimeSpec(t, h, w, t * h * w)
        handle = ctypes.c_void_p()
        create = lib.awa_plan_create_host if host_only else lib.awa_plan_create
        rc = create(ctypes.byref(params), ctypes.byref(spec) if spec is not None else None, ctypes.byref(handle))
        _check(rc)
        self._handle = handle
        info = _PlanInfo()
        _check(lib.awa_plan_get_info(handle, ctypes.byref(info)))
        self.info = PlanInfo(*(getattr(info, f[0]) for f in _PlanInfo._fields_))

    def __del__(self):
        handle = getattr(self, "_handle", None)
        if handle and _lib is not None:
            _lib.awa_plan_destroy(handle)
            self._handle = None

    @property
    def handle(self):
        return self._handle

    def maps(self):
        """Host copies of the index maps (numpy int32) and the window list."""
        import numpy as np

        inf = self.info
        seq = np.empty(inf.sequence_tokens, np.int32)
        cu = np.empty(inf.window_count + 1, np.int32)
        vpos = np.empty(inf.source_tokens, np.int32)
        tpos = np.empty(inf.window_count * inf.text_tokens, np.int32)
        wins = (_Window * inf.window_count)()
        _check(library().awa_plan_get_maps(self._handle, seq.ctypes.data, cu.ctypes.data, vpos.ctypes.data,
                                           tpos.ctypes.data, ctypes.cast(wins, ctypes.c_void_p)))
        return {"sequence_index": seq, "cu_seqlens": cu, "video_positions": vpos, "text_positions": tpos,
                "windows": [(w.t0, w.t1, w.h0, w.h1, w.w0, w.w1) for w in wins]}

    # ---------------------------------------------------------------- layers
    def pack(self, video_qkv, text_qkv, out_dtype=None, stream=None):
        """SeedVR2AWAPack: returns (packed [S, 3, H, d], cu_seqlens float [W+1])."""
        torch = _torch()
        heads, hd = video_qkv.shape[2], video_qkv.shape[3]
        out_dtype = video_qkv.dtype if out_dtype is None else out_dtype
        packed = torch.empty(self.info.sequence_tokens, 3, heads, hd, dtype=out_dtype, device=video_qkv.device)
        cu = torch.empty(self.info.window_count + 1, dtype=torch.float32, device=video_qkv.device)
        vts, vqs = _qkv_strides(video_qkv)
        tts, tqs = _qkv_strides(text_qkv)
        if video_qkv.dtype != text_qkv.dtype:
            raise TypeError("video and text QKV must share a dtype")
        _check(library().awa_pack(self._handle, heads, hd, _dtype_code(video_qkv), video_qkv.data_ptr(), vts, vqs,
                                  text_qkv.data_ptr(), tts, tqs, _dtype_code(packed), packed.data_ptr(),
                                  packed.stride(0), cu.data_ptr(), _stream_ptr(stream)))
        return packed, cu

    def mmrope(self, packed, out_dtype=None, stream=None):
        """SeedVR2MMRoPE on a packed [S, 3, H, d] tensor."""
        torch = _torch()
        heads, hd = packed.shape[2], packed.shape[3]
        out = torch.empty(packed.shape, dtype=packed.dtype if out_dtype is None else out_dtype, device=packed.device)
        _check(library().awa_mmrope(self._handle, heads, hd, _dtype_code(packed), packed.data_ptr(), packed.stride(0),
                                    _dtype_code(out), out.data_ptr(), out.stride(0), _stream_ptr(stream)))
        return out

    def window_attention(self, packed, precision=AWA_PREC_FP32, out_dtype=None, stream=None):
        """SeedVR2WindowAttention: packed [S, 3, H, d] -> attended [S, H, d]."""
        torch = _torch()
        s, _, heads, hd = packed.shape
        out = torch.empty(s, heads, hd, dtype=packed.dtype if out_dtype is None else out_dtype, device=packed.device)
        _check(library().awa_window_attention(self._handle, precision, heads, hd, _dtype_code(packed),
                                              packed.data_ptr(), packed.stride(0), _dtype_code(out), out.data_ptr(),
                                              out.stride(0), _stream_ptr(stream)))
        return out

    def unpack(self, attended, out_dtype=None, stream=None):
        """SeedVR2AWAUnpack: attended [S, H, d] -> (video [N_v, H, d], text [T, H, d])."""
        torch = _torch()
        _, heads, hd = attended.shape
        dt = attended.dtype if out_dtype is None else out_dtype
        video = torch.empty(self.info.source_tokens, heads, hd, dtype=dt, device=attended.device)
        text = torch.empty(self.info.text_tokens, heads, hd, dtype=dt, device=attended.device)
        _check(library().awa_unpack(self._handle, heads, hd, _dtype_code(attended), attended.data_ptr(),
                                    attended.stride(0), _dtype_code(video), video.data_ptr(), video.stride(0),
                                    text.data_ptr(), text.stride(0), _stream_ptr(stream)))
        return video, text

    # ---------------------------------------------------------------- fused chain
    def workspace_bytes(self, heads: int, head_dim: int, precision=None, in_dtype=None) -> int:
        """awa_forward's workspace; with precision and in_dtype (a torch dtype)
        it includes the bf16 copy that fp32 rows on the tensor-core path need."""
        if precision is None:
            return int(library().awa_forward_workspace_bytes(self._handle, heads, head_dim))
        return int(library().awa_forward_workspace_bytes_for(self._handle, precision, _dtype_code_of(in_dtype),
                                                             heads, head_dim))

    def forward(self, video_qkv, text_qkv, precision=AWA_PREC_BF16, out_dtype=None, workspace=None,
                video_out=None, text_out=None, stream=None):
        """Pack -> MMRoPE -> WindowAttention -> Unpack in one pass: (video, text)."""
        torch = _torch()
        heads, hd = video_qkv.shape[2], video_qkv.shape[3]
        dt = video_qkv.dtype if out_dtype is None else out_dtype
        if video_out is None:
            video_out = torch.empty(self.info.source_tokens, heads, hd, dtype=dt, device=video_qkv.device)
        if text_out is None:
            text_out = torch.empty(self.info.text_tokens, heads, hd, dtype=dt, device=video_qkv.device)
        need = self.workspace_bytes(heads, hd, precision, video_qkv.dtype)
        if workspace is None:
            workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=video_qkv.device)
        vts, vqs = _qkv_strides(video_qkv)
        tts, tqs = _qkv_strides(text_qkv)
        _check(library().awa_forward(self._handle, precision, heads, hd, _dtype_code(video_qkv), video_qkv.data_ptr(),
                                     vts, vqs, text_qkv.data_ptr(), tts, tqs, _dtype_code(video_out),
                                     video_out.data_ptr(), video_out.stride(0), text_out.data_ptr(), text_out.stride(0),
                                     workspace.data_ptr(), workspace.numel() * workspace.element_size(),
                                     _stream_ptr(stream)))
        return video_out, text_out

    def host_workspace_bytes(self, precision, in_dtype, out_dtype, heads: int, head_dim: int) -> int:
        return int(library().awa_forward_host_workspace_bytes(self._handle, precision, _dtype_code_of(in_dtype),
                                                              _dtype_code_of(out_dtype), heads, head_dim))

    def forward_host(self, video_qkv, text_qkv, video_out, text_out, precision=AWA_PREC_BF16, workspace=None,
                     stream=None):
        """awa_forward_host: inputs and outputs are CPU tensors (pin them for
        full-rate copies); enqueues copy in, forward and copy out on `stream`
        without waiting. Returns the device workspace used (keep it alive until
        the stream is done)."""
        torch = _torch()
        heads, hd = video_qkv.shape[2], video_qkv.shape[3]
        if workspace is None:
            need = self.host_workspace_bytes(precision, video_qkv.dtype, video_out.dtype, heads, hd)
            workspace = torch.empty(max(need, 16), dtype=torch.uint8, device="cuda")
        vts, vqs = _qkv_strides(video_qkv)
        tts, tqs = _qkv_strides(text_qkv)
        _check(library().awa_forward_host(self._handle, precision, heads, hd, _dtype_code(video_qkv),
                                          video_qkv.data_ptr(), vts, vqs, text_qkv.data_ptr(), tts, tqs,
                                          _dtype_code(video_out), video_out.data_ptr(), video_out.stride(0),
                                          text_out.data_ptr(), text_out.stride(0), workspace.data_ptr(),
                                          workspace.numel() * workspace.element_size(), _stream_ptr(stream)))
        return workspace

    def forward_prerotated(self, video_qkv, text_qkv, precision=AWA_PREC_BF16, out_dtype=None, workspace=None,
                           video_out=None, text_out=None, stream=None):
        """forward() for Q/K rows already rotated by qkv_project_rotated with this plan."""
        torch = _torch()
        heads, hd = video_qkv.shape[2], video_qkv.shape[3]
        dt = video_qkv.dtype if out_dtype is None else out_dtype
        if video_out is None:
            video_out = torch.empty(self.info.source_tokens, heads, hd, dtype=dt, device=video_qkv.device)
        if text_out is None:
            text_out = torch.empty(self.info.text_tokens, heads, hd, dtype=dt, device=video_qkv.device)
        if workspace is None:
            workspace = torch.empty(max(self.workspace_bytes(heads, hd, precision, video_qkv.dtype), 16),
                                    dtype=torch.uint8, device=video_qkv.device)
        vts, vqs = _qkv_strides(video_qkv)
        tts, tqs = _qkv_strides(text_qkv)
        _check(library().awa_forward_prerotated(self._handle, precision, heads, hd, _dtype_code(video_qkv),
                                                video_qkv.data_ptr(), vts, vqs, text_qkv.data_ptr(), tts, tqs,
                                                _dtype_code(video_out), video_out.data_ptr(), video_out.stride(0),
                                                text_out.data_ptr(), text_out.stride(0), workspace.data_ptr(),
                                                workspace.numel() * workspace.element_size(), _stream_ptr(stream)))
        return video_out, text_out

    def forward_windows(self, video_qkv, text_qkv, window_begin: int, window_end: int, video_out, text_partial,
                        precision=AWA_PREC_BF16, workspace=None, stream=None):
        """Windows [begin, end) only: writes their video rows and the fp32 text partial sum."""
        torch = _torch()
        heads, hd = video_qkv.shape[2], video_qkv.shape[3]
        need = (window_end - window_begin) * self.info.text_tokens * heads * hd * 4
        if workspace is None:
            workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=video_qkv.device)
        vts, vqs = _qkv_strides(video_qkv)
        tts, tqs = _qkv_strides(text_qkv)
        _check(library().awa_forward_windows(self._handle, precision, heads, hd, window_begin, window_end,
                                             _dtype_code(video_qkv), video_qkv.data_ptr(), vts, vqs,
                                             text_qkv.data_ptr(), tts, tqs, _dtype_code(video_out),
                                             video_out.data_ptr(), video_out.stride(0), text_partial.data_ptr(),
                                             workspace.data_ptr(), workspace.numel() * workspace.element_size(),
                                             _stream_ptr(stream)))

    def text_finalize(self, text_sum, out_dtype, stream=None):
        torch = _torch()
        t, heads, hd = text_sum.shape
        out = torch.empty(t, heads, hd, dtype=out_dtype, device=text_sum.device)
        _check(library().awa_text_finalize(self._handle, heads, hd, text_sum.data_ptr(), _dtype_code(out),
                                           out.data_ptr(), out.stride(0), _stream_ptr(stream)))
        return out

    # ---------------------------------------------------------------- multi-GPU
    def shard_split(self, nranks: int, heads: int) -> Tuple[bool, List[int]]:
        """(by_heads, bounds): how awa_forward_sharded splits this layer over
        nranks ranks -- window bounds, or head bounds when windows are few."""
        by_heads = ctypes.c_int(0)
        bounds = (ctypes.c_int * (nranks + 1))()
        _check(library().awa_shard_split(self._handle, nranks, heads, ctypes.byref(by_heads),
                                         ctypes.cast(bounds, ctypes.c_void_p)))
        return bool(by_heads.value), list(bounds)

    def shard_windows(self, nranks: int, heads: int, rank: int) -> List[int]:
        """The windows `rank` computes (ascending plan indices)."""
        lib = library()
        n = lib.awa_shard_windows(self._handle, nranks, heads, rank, None, 0)
        _check(min(n, 0))
        buf = (ctypes.c_int * max(n, 1))()
        lib.awa_shard_windows(self._handle, nranks, heads, rank, ctypes.cast(buf, ctypes.c_void_p), n)
        return list(buf[:n])

    def shard_runs(self, nranks: int, heads: int, rank: int) -> List[Tuple[int, int]]:
        """The (first token, tokens) runs of video rows `rank` reads and writes."""
        lib = library()
        n = lib.awa_shard_runs(self._handle, nranks, heads, rank, None, 0)
        _check(min(n, 0))
        buf = (ctypes.c_int64 * max(2 * n, 2))()
        lib.awa_shard_runs(self._handle, nranks, heads, rank, ctypes.cast(buf, ctypes.c_void_p), n)
        return [(buf[2 * i], buf[2 * i + 1]) for i in range(n)]

    def sharded_workspace_bytes(self, nranks: int, heads: int, head_dim: int, out_dtype) -> int:
        code = out_dtype if isinstance(out_dtype, int) else _dtype_code_of(out_dtype)
        return int(library().awa_forward_sharded_workspace_bytes(self._handle, nranks, heads, head_dim, code))

    def forward_sharded(self, comm: "AwaComm", video_qkv, text_qkv, precision=AWA_PREC_BF16, out_dtype=None,
                        workspace=None, video_out=None, text_out=None, stream=None):
        """awa_forward over the ranks of `comm` (every rank passes the full
        inputs and gets the full outputs): (video, text)."""
        torch = _torch()
        heads, hd = video_qkv.shape[2], video_qkv.shape[3]
        dt = video_qkv.dtype if out_dtype is None else out_dtype
        if video_out is None:
            video_out = torch.empty(self.info.source_tokens, heads, hd, dtype=dt, device=video_qkv.device)
        if text_out is None:
            text_out = torch.empty(self.info.text_tokens, heads, hd, dtype=dt, device=video_qkv.device)
        if workspace is None:
            need = self.sharded_workspace_bytes(comm.nranks, heads, hd, dt)
            workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=video_qkv.device)
        vts, vqs = _qkv_strides(video_qkv)
        tts, tqs = _qkv_strides(text_qkv)
        _check(library().awa_forward_sharded(self._handle, comm.handle, precision, heads, hd, _dtype_code(video_qkv),
                                             video_qkv.data_ptr(), vts, vqs, text_qkv.data_ptr(), tts, tqs,
                                             _dtype_code(video_out), video_out.data_ptr(), video_out.stride(0),
                                             text_out.data_ptr(), text_out.stride(0), workspace.data_ptr(),
                                             workspace.numel() * workspace.element_size(), _stream_ptr(stream)))
        return video_out, text_out

    def partition(self, parts: int) -> List[int]:
        bounds = (ctypes.c_int * (parts + 1))()
        _check(library().awa_partition_windows(self._handle, parts, ctypes.cast(bounds, ctypes.c_void_p)))
        return list(bounds)

    def range_video_rows(self, begin: int, end: int) -> int:
        return int(library().awa_window_range_video_rows(self._handle, begin, end))

    def gather_video_shard(self, video, begin: int, end: int, shard, stream=None):
        _, heads, hd = video.shape
        _check(library().awa_gather_video_shard(self._handle, heads, hd, begin, end, _dtype_code(video),
                                                video.data_ptr(), video.stride(0), shard.data_ptr(),
                                                _stream_ptr(stream)))

    def scatter_video_shard(self, shard, begin: int, end: int, video, stream=None):
        _, heads, hd = video.shape
        _check(library().awa_scatter_video_shard(self._handle, heads, hd, begin, end, _dtype_code(video),
                                                 shard.data_ptr(), video.data_ptr(), video.stride(0),
                                                 _stream_ptr(stream)))

    def attention_kernel_kind(self, precision: int, heads: int, head_dim: int, in_dtype=None) -> int:
        """1 = tcgen05 kernel, 2 = fp32 SIMT kernel. `in_dtype` (a torch dtype) defaults to bf16 at
        AWA_PREC_BF16 and fp32 otherwise."""
        torch = _torch()
        if in_dtype is None:
            in_dtype = torch.bfloat16 if precision == AWA_PREC_BF16 else torch.float32
        code = AWA_BF16 if in_dtype == torch.bfloat16 else AWA_F32
        return int(library().awa_attention_kernel_kind(self._handle, precision, code, heads, head_dim))


def qkv_project(x, w, gamma_q, gamma_k, eps: float, heads: int, out_dtype=None, out=None, stream=None):
    """The block's QKV projection with the per-head RMSNorm of Q and K
    (awa_qkv_project): x [tokens, model_dim] bf16, w [3*heads*128, model_dim]
    bf16 (nn.Linear layout), gamma_q / gamma_k [128] fp32 -> [tokens, 3, heads,
    128] in out_dtype (bf16 by default), the rows awa_forward reads."""
    torch = _torch()
    tokens, model_dim = x.shape
    if out is None:
        out = torch.empty(tokens, 3, heads, 128, dtype=out_dtype or torch.bfloat16, device=x.device)
    _check(library().awa_qkv_project(tokens, model_dim, heads, 128, x.data_ptr(), x.stride(0), w.data_ptr(),
                                     w.stride(0), gamma_q.data_ptr(), gamma_k.data_ptr(), float(eps),
                                     _dtype_code(out), out.data_ptr(), out.stride(0), _stream_ptr(stream)))
    return out


def qkv_project_rotated(x, w, gamma_q, gamma_k, eps: float, heads: int, plan: "AwaPlan", branch: int,
                        out_dtype=None, out=None, stream=None):
    """qkv_project with the layer's MMRoPE in the epilogue
    (awa_qkv_project_rotated): Q and K heads rotated in fp32 with the
    window-local coordinates `plan` gives each row of `branch`
    (AWA_BRANCH_VIDEO: the plan's video tokens; AWA_BRANCH_TEXT: its text
    tokens), rounded once. The rows feed AwaPlan.forward_prerotated."""
    torch = _torch()
    tokens, model_dim = x.shape
    if out is None:
        out = torch.empty(tokens, 3, heads, 128, dtype=out_dtype or torch.bfloat16, device=x.device)
    _check(library().awa_qkv_project_rotated(tokens, model_dim, heads, 128, x.data_ptr(), x.stride(0), w.data_ptr(),
                                             w.stride(0), gamma_q.data_ptr(), gamma_k.data_ptr(), float(eps),
                                             plan.handle, branch, _dtype_code(out), out.data_ptr(), out.stride(0),
                                             _stream_ptr(stream)))
    return out


def out_project(x, w, bias, gate, residual, out_dtype=None, out=None, stream=None):
    """The block's proj_out + Ada "out" gate + residual (awa_out_project):
    x [tokens, in_dim] bf16, w [out_dim, in_dim] bf16, bias / gate [out_dim]
    fp32, residual [tokens, out_dim] bf16 or fp32 -> residual + bf16(x W^T +
    bias) * gate, [tokens, out_dim] in out_dtype (the residual's by default)."""
    torch = _torch()
    tokens, in_dim = x.shape
    out_dim = w.shape[0]
    if out is None:
        out = torch.empty(tokens, out_dim, dtype=out_dtype or residual.dtype, device=x.device)
    _check(library().awa_out_project(tokens, in_dim, out_dim, x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0),
                                     bias.data_ptr(), gate.data_ptr(), residual.data_ptr(), residual.stride(0),
                                     _dtype_code(residual), _dtype_code(out), out.data_ptr(), out.stride(0),
                                     _stream_ptr(stream)))
    return out


class AwaStack:
    """The AWA chains of a DiT block stack on one stream (include/awa_stack.h).

    block_params: one dict of awa_layer_params fields per block (e.g. the
    "params" of graph_find_chains for each block graph); fp32_blocks leading
    blocks run in fp32, the rest in bf16. Built on the current device.
    """

    def __init__(self, block_params, runtime_spec=None, fp32_blocks: int = 0, heads: int = 20, head_dim: int = 128):
        lib = library()
        arr = (_LayerParams * len(block_params))()
        for i, p in enumerate(block_params):
            arr[i] = _LayerParams(*(int(p.get(f, 126 if f == "rope_dim" else 0)) for f, _ in _LayerParams._fields_))
        spec = None
        if runtime_spec is not None:
            t, h, w = runtime_spec
            spec = _RuntimeSpec(t, h, w, t * h * w)
        handle = ctypes.c_void_p()
        _check(lib.awa_stack_create(ctypes.cast(arr, ctypes.c_void_p), len(block_params),
                                    ctypes.byref(spec) if spec is not None else None, int(fp32_blocks), int(heads),
                                    int(head_dim), ctypes.byref(handle)))
        self._handle = handle
        self.blocks = len(block_params)

    def __del__(self):
        handle = getattr(self, "_handle", None)
        if handle and _lib is not None:
            _lib.awa_stack_destroy(handle)
            self._handle = None

    @property
    def handle(self):
        return self._handle

    def info(self) -> Tuple[int, int]:
        """(distinct plans, workspace bytes)."""
        plans, ws = ctypes.c_int(0), ctypes.c_size_t(0)
        _check(library().awa_stack_get_info(self._handle, ctypes.byref(plans), ctypes.byref(ws)))
        return plans.value, ws.value

    def _callback(self, hook, errors):
        def call(_user, stage, io, stream):
            try:
                return int(hook(stage, io.contents, stream) or 0)
            except BaseException as exc:  # reported after the C call returns
                errors.append(exc)
                return 1
        return STACK_HOOK(call)

    def run(self, hook, stream) -> None:
        """hook(stage, io: StackIO, stream_handle) enqueues the caller's work
        on the raw stream handle and fills io at AWA_STACK_BEFORE."""
        errors = []
        cb = self._callback(hook, errors)
        rc = library().awa_stack_run(self._handle, cb, None, _stream_ptr(stream))
        if errors:
            raise errors[0]
        _check(rc)

    def capture(self, hook, stream) -> "StackGraph":
        """run() captured into a CUDA graph on stream (not the default stream)."""
        errors = []
        cb = self._callback(hook, errors)
        graph = ctypes.c_void_p()
        rc = library().awa_stack_capture(self._handle, cb, None, _stream_ptr(stream), ctypes.byref(graph))
        if errors:
            raise errors[0]
        _check(rc)
        return StackGraph(graph)


class StackGraph:
    """An instantiated CUDA graph of one stack run (awa_stack_capture)."""

    def __init__(self, handle):
        self._handle = handle

    def launch(self, stream) -> None:
        _check(library().awa_stack_graph_launch(self._handle, _stream_ptr(stream)))

    def __del__(self):
        handle = getattr(self, "_handle", None)
        if handle and _lib is not None:
            _lib.awa_stack_graph_destroy(handle)
            self._handle = None


def _dtype_code_of(torch_dtype) -> int:
    torch = _torch()
    return AWA_BF16 if torch_dtype == torch.bfloat16 else AWA_F32


class AwaComm:
    """An NCCL communicator for awa_forward_sharded (one rank per GPU, on the
    current device). Every rank passes the same 128-byte id, made once by
    AwaComm.unique_id() on rank 0 and handed to the others by the caller."""

    def __init__(self, unique_id: bytes, nranks: int, rank: int):
        handle = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(bytes(unique_id), len(unique_id))
        _check(library().awa_comm_create(ctypes.cast(buf, ctypes.c_void_p), len(unique_id), nranks, rank,
                                         ctypes.byref(handle)))
        self._handle = handle
        self.nranks, self.rank = nranks, rank

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        _check(library().awa_comm_unique_id(ctypes.cast(buf, ctypes.c_void_p), 128))
        return buf.raw

    @property
    def handle(self):
        return self._handle

    def set_push(self, mode: int) -> None:
        """How the direct mode moves video rows (AWA_PUSH_AUTO / _COPY_ENGINES / _KERNEL)."""
        _check(library().awa_comm_set_push(self._handle, mode))

    def shared_tensor(self, shape, dtype):
        """Collective: a torch tensor over a buffer shared by every rank
        (awa_comm_alloc_shared). A video output in such a buffer lets
        forward_sharded store rows straight into every rank's copy. Release
        with free_shared (collective)."""
        torch = _torch()
        import math as _math

        nbytes = _math.prod(shape) * torch.tensor([], dtype=dtype).element_size()
        ptr = ctypes.c_void_p()
        _check(library().awa_comm_alloc_shared(self._handle, nbytes, ctypes.byref(ptr)))
        typestr = {torch.bfloat16: "<i2", torch.float32: "<f4"}[dtype]

        class _Iface:
            __cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr.value, False),
                                        "version": 3, "strides": None}

        t = torch.as_tensor(_Iface(), device="cuda")
        if dtype == torch.bfloat16:
            t = t.view(torch.bfloat16)
        self._shared = getattr(self, "_shared", [])
        self._shared.append(ptr.value)
        return t

    def free_shared(self, tensor) -> None:
        ptr = tensor.data_ptr()
        _check(library().awa_comm_free_shared(self._handle, ctypes.c_void_p(ptr)))
        self._shared = [p for p in getattr(self, "_shared", []) if p != ptr]

    def destroy(self) -> None:
        if getattr(self, "_handle", None) and _lib is not None:
            _lib.awa_comm_destroy(self._handle)
            self._handle = None

    def __del__(self):
        self.destroy()


def device_status() -> None:
    """Raise if a device-side check of the library failed since the last call."""
    _check(library().awa_device_status())


def profile_enable(enabled: bool = True) -> None:
    """Bracket every library kernel launch with CUDA events on its stream."""
    library().awa_profile_enable(int(enabled))


def profile_reset() -> None:
    library().awa_profile_reset()


def profile_collect() -> dict:
    """{kernel name: (launches, total device ms)} since the last reset."""
    lib = library()
    n = lib.awa_profile_collect(None, 0)
    buf = ctypes.create_string_buffer(n + 1)
    lib.awa_profile_collect(buf, n + 1)
    out = {}
    for line in buf.value.decode().splitlines():
        fields = dict(item.split("=", 1) for item in line.split()[1:])
        out[fields["name"]] = (int(fields["launches"]), float(fields["ms"]))
    return out


# ---------------------------------------------------------------- ncnn layer classes
_compat = {}


def ncnn_compat(batch: bool = False) -> ctypes.CDLL:
    """The ncnn layer classes' library: built against the ncnn API subset
    without NCNN_BATCH, or (batch=True) with it."""
    if batch not in _compat:
        library()
        path = COMPAT_BATCH_PATH if batch else COMPAT_PATH
        if not os.path.isfile(path):
            raise ImportError(f"{path} is missing")
        lib = ctypes.CDLL(path)
        p, i = ctypes.c_void_p, ctypes.c_int
        lib.awa_ncnn_run_chain.restype = i
        lib.awa_ncnn_run_chain.argtypes = [p, i, i, i, i, i, i, i, p, p, p, p, p, p, p, p]
        lib.awa_ncnn_batch_build.restype = i
        assert bool(lib.awa_ncnn_batch_build()) == batch, path
        _compat[batch] = lib
    return _compat[batch]


def ncnn_run_chain(params: Sequence[int], heads: int, head_dim: int, video_qkv, text_qkv, layout: int = 0,
                   runtime_spec: bool = False, bf16: bool = False, device_blobs: bool = False,
                   batch_build: bool = False):
    """Run SeedVR2AWAPack -> MMRoPE -> WindowAttention -> AWAUnpack through the
    ncnn layer classes (register_seedvr2_awa_layers + Net + ParamDict + forward).

    video_qkv / text_qkv: host numpy arrays [tokens, 3, H, d] (float32, or
    uint16 holding bf16 bits), written into QKV blob encoding `layout` (0: w=d,
    h=3H, c=N; 1: w=d, h=H, c=3N; 2: w=d, h=H, d=3, c=N; 3: w=d, h=H, c=3, n=N,
    which needs batch_build). batch_build selects the classes built with
    NCNN_BATCH, whose video output is the 4-D batched blob. Returns a dict of
    dense numpy outputs (video rows in t, h, w order) and the status.
    """
    import numpy as np

    lib = ncnn_compat(batch_build)
    params = list(params)
    elem = 2 if video_qkv.dtype == np.uint16 else 4
    out_np = np.uint16 if bf16 else np.float32
    n_v = params[0] * params[1] * params[2]
    windows = make_windows(params[0:3], params[3:6], bool(params[7]))
    s = n_v + len(windows) * params[6]
    out = {
        "packed": np.empty((s, 3, heads, head_dim), out_np),
        "cu_seqlens": np.empty(len(windows) + 1, np.float32),
        "roped": np.empty((s, 3, heads, head_dim), out_np),
        "attended": np.empty((s, heads, head_dim), out_np),
        "video": np.empty((n_v, heads, head_dim), out_np),
        "text": np.empty((params[6], heads, head_dim), out_np),
    }
    arr = (ctypes.c_int * 9)(*params)
    v = np.ascontiguousarray(video_qkv)
    t = np.ascontiguousarray(text_qkv)
    rc = lib.awa_ncnn_run_chain(ctypes.cast(arr, ctypes.c_void_p), heads, head_dim, layout, int(runtime_spec),
                                int(bf16), int(device_blobs), elem, v.ctypes.data, t.ctypes.data,
                                *(out[k].ctypes.data for k in ("packed", "cu_seqlens", "roped", "attended", "video",
                                                               "text")))
    out["status"] = rc
    return out


def _chains(count_fn) -> List[dict]:
    n = count_fn(None, 0)
    if n < 0:
        _check(n)
    arr = (_GraphChain * max(n, 1))()
    _check(min(0, count_fn(ctypes.cast(arr, ctypes.c_void_p), n)))
    out = []
    for c in arr[:n]:
        params = {f: getattr(c.params, f) for f, _ in _LayerParams._fields_}
        out.append({"params": params, **{f: getattr(c, f) for f, _ in _GraphChain._fields_[1:]}})
    return out


def graph_find_chains(text) -> List[dict]:
    """AWA chains of an ncnn .param text (str or bytes): per chain its ParamDict
    values ("params", the awa_layer_params fields), "dynamic" and the 1-based
    line numbers of its layers (awa_graph_find_chains). Host only."""
    data = text.encode() if isinstance(text, str) else bytes(text)
    return _chains(lambda buf, cap: library().awa_graph_find_chains(data, len(data), buf, cap))


def graph_find_chains_file(path) -> List[dict]:
    """graph_find_chains on a .param file."""
    raw = os.fsencode(path)
    return _chains(lambda buf, cap: library().awa_graph_find_chains_file(raw, buf, cap))


def graph_make_dynamic(text) -> str:
    """The resolution-independent form of a block graph's .param text: the
    exporter's normalize_dynamic_awa_template (awa_graph_make_dynamic)."""
    data = text.encode() if isinstance(text, str) else bytes(text)
    lib = library()
    needed = ctypes.c_size_t(0)
    rc = lib.awa_graph_make_dynamic(data, len(data), None, 0, ctypes.byref(needed))
    if rc not in (AWA_OK, AWA_ERR_ALLOC):
        _check(rc)
    out = ctypes.create_string_buffer(needed.value + 1)
    _check(lib.awa_graph_make_dynamic(data, len(data), ctypes.cast(out, ctypes.c_void_p), len(out),
                                      ctypes.byref(needed)))
    return out.raw[:needed.value].decode()


def manifest_validate(package_dir, expected_records: int = 0) -> None:
    """Raise AwaError unless package_dir matches its manifest.sha256
    (awa_manifest_validate; expected_records 0 = the reference's 75/146 rule)."""
    _check(library().awa_manifest_validate(os.fsencode(package_dir), int(expected_records)))


def sha256(data: bytes) -> str:
    buf = ctypes.create_string_buffer(65)
    data = bytes(data)
    _check(library().awa_sha256(data, len(data), ctypes.cast(buf, ctypes.c_void_p)))
    return buf.value.decode()


def sha256_file(path) -> str:
    buf = ctypes.create_string_buffer(65)
    _check(library().awa_sha256_file(os.fsencode(path), ctypes.cast(buf, ctypes.c_void_p)))
    return buf.value.decode()


__all__ = ["AwaPlan", "AwaComm", "AwaError", "PlanInfo", "library", "make_windows", "device_status", "ncnn_run_chain",
           "EXPORTED_SYMBOLS", "qkv_project", "qkv_project_rotated", "out_project", "graph_find_chains", "graph_find_chains_file",
           "graph_make_dynamic", "manifest_validate", "sha256", "sha256_file", "AwaStack", "StackGraph", "StackIO",
           "AWA_STACK_BEFORE", "AWA_STACK_AFTER", "AWA_F32", "AWA_BF16", "AWA_PREC_FP32", "AWA_PREC_BF16",
           "AWA_BRANCH_VIDEO", "AWA_BRANCH_TEXT"]

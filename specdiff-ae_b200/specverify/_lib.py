"""ctypes binding of libspecverify.so (the C ABI declared in include/specverify.h).

The library is loaded from this package directory.  There is no fallback:
if it is missing or cannot be loaded, every entry point raises
:class:`SpecVerifyError` -- the CUDA kernels are the product path.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libspecverify.so"

TV_OK = 0
TV_BF16, TV_F16, TV_F32 = 0, 1, 2

_DTYPE_CODE = {torch.bfloat16: TV_BF16, torch.float16: TV_F16, torch.float32: TV_F32}


class SpecVerifyError(RuntimeError):
    """Raised when a library call returns a non-zero status."""

    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} (status {status})"
                         + (f" [{last_cuda_error()}]" if status == -4 else ""))


c_i32, c_i64, c_f32, c_u64, c_size, c_vp = (ctypes.c_int32, ctypes.c_int64, ctypes.c_float,
                                            ctypes.c_uint64, ctypes.c_size_t, ctypes.c_void_p)


class AttnArgs(ctypes.Structure):
    """Mirror of ``tv_attn_args``."""
    _fields_ = [
        ("dtype", c_i32), ("batch", c_i32), ("rows", c_i32), ("heads", c_i32), ("kv_heads", c_i32),
        ("head_dim", c_i32), ("scale", c_f32),
        ("q", c_vp), ("q_sb", c_i64), ("q_sm", c_i64), ("q_sh", c_i64),
        ("k", c_vp), ("v", c_vp),
        ("k_sb", c_i64), ("k_sn", c_i64), ("k_sh", c_i64),
        ("v_sb", c_i64), ("v_sn", c_i64), ("v_sh", c_i64),
        ("page_table", c_vp), ("pt_sb", c_i64), ("page_size", c_i32), ("num_pages", c_i32),
        ("kv_lens", c_vp), ("num_keys", c_i32), ("mask_len", c_i32),
        ("mask", c_vp), ("mask_sb", c_i64), ("mask_sm", c_i64),
        ("out", c_vp), ("o_sb", c_i64), ("o_sm", c_i64), ("o_sh", c_i64), ("out_f32", c_i32),
        ("lse", c_vp), ("lse_sb", c_i64), ("lse_sm", c_i64), ("lse_sh", c_i64),
        ("aux_lse", c_vp), ("aux_sb", c_i64), ("aux_sm", c_i64), ("aux_sh", c_i64),
        ("weight", c_vp), ("w_sb", c_i64), ("w_sm", c_i64), ("w_sh", c_i64),
        ("num_splits", c_i32), ("kernel", c_i32),
        ("workspace", c_vp), ("workspace_bytes", c_size), ("status", c_vp),
        ("mask_words_full", c_vp), ("mask_words_full_sb", c_i64),
    ]


class AcceptArgs(ctypes.Structure):
    """Mirror of ``tv_accept_args``."""
    _fields_ = [
        ("mode", c_i32), ("logits_dtype", c_i32), ("logits", c_vp), ("logits_sm", c_i64),
        ("rows", c_i32), ("vocab", c_i32),
        ("draft", c_vp), ("parent", c_vp), ("pos", c_vp), ("max_depth", c_i32),
        ("sampled", c_vp), ("temperature", c_f32), ("seed", c_u64), ("offset", c_u64),
        ("next_tokens", c_vp), ("result", c_vp), ("workspace", c_vp), ("workspace_bytes", c_size),
    ]


class RopeArgs(ctypes.Structure):
    """Mirror of ``tv_rope_args``."""
    _fields_ = [
        ("dtype", c_i32), ("batch", c_i32), ("tokens", c_i32), ("heads", c_i32), ("kv_heads", c_i32),
        ("head_dim", c_i32),
        ("q", c_vp), ("q_sb", c_i64), ("q_sh", c_i64), ("q_st", c_i64),
        ("k", c_vp), ("k_sb", c_i64), ("k_sh", c_i64), ("k_st", c_i64),
        ("v", c_vp), ("v_sb", c_i64), ("v_sh", c_i64), ("v_st", c_i64),
        ("cos", c_vp), ("sin", c_vp), ("cs_sb", c_i64), ("cs_sr", c_i64), ("cs_rows", c_i64),
        ("pos", c_vp), ("pos_sb", c_i64),
        ("q_out", c_vp), ("qo_sb", c_i64), ("qo_sh", c_i64), ("qo_st", c_i64),
        ("k_out", c_vp), ("ko_sb", c_i64), ("ko_sh", c_i64), ("ko_st", c_i64),
        ("k_cache", c_vp), ("kc_sb", c_i64), ("kc_sh", c_i64), ("kc_st", c_i64),
        ("v_cache", c_vp), ("vc_sb", c_i64), ("vc_sh", c_i64), ("vc_st", c_i64),
        ("start", c_i64), ("capacity", c_i64),
        ("page_table", c_vp), ("pt_sb", c_i64), ("page_size", c_i32), ("num_pages", c_i32),
        ("status", c_vp),
    ]


class LmheadArgs(ctypes.Structure):
    """Mirror of ``tv_lmhead_args``."""
    _fields_ = [
        ("dtype", c_i32), ("rows", c_i32), ("hidden", c_i32), ("vocab", c_i32),
        ("x", c_vp), ("x_sm", c_i64), ("weight", c_vp), ("w_sv", c_i64),
        ("mode", c_i32), ("temperature", c_f32), ("seed", c_u64), ("offset", c_u64),
        ("draft", c_vp), ("parent", c_vp), ("pos", c_vp), ("max_depth", c_i32),
        ("next_tokens", c_vp), ("result", c_vp), ("workspace", c_vp), ("workspace_bytes", c_size),
    ]


# name -> (restype, argtypes)
_SIGNATURES = {
    "tv_status_string": (ctypes.c_char_p, [c_i32]),
    "tv_version": (ctypes.c_char_p, []),
    "tv_last_cuda_error": (ctypes.c_char_p, []),
    "tv_attn_workspace_size": (c_i32, [ctypes.POINTER(AttnArgs), ctypes.POINTER(c_size)]),
    "tv_attn_describe": (c_i32, [ctypes.POINTER(AttnArgs), ctypes.POINTER(c_i32)]),
    "tv_verify_attn": (c_i32, [ctypes.POINTER(AttnArgs), c_vp]),
    "tv_verify_attn_static": (c_i32, [ctypes.POINTER(AttnArgs), c_vp]),
    "tv_merge_partials": (c_i32, [c_i32, c_i64, c_i32, c_vp, c_i64, c_vp, c_i64, c_i32, c_vp, c_vp, c_vp]),
    "tv_sharded_exchange_bytes": (c_i32, [c_i32, c_i64, c_i32, ctypes.POINTER(c_i64)]),
    "tv_verify_attn_sharded_workspace_size": (c_i32, [ctypes.POINTER(AttnArgs), ctypes.POINTER(c_size)]),
    "tv_verify_attn_sharded": (c_i32, [ctypes.POINTER(AttnArgs), c_i32, c_i32, ctypes.POINTER(c_vp), c_i64, c_vp]),
    "tv_pack_mask": (c_i32, [c_i32, c_vp, c_i64, c_i64, c_i64, c_i32, c_i32, c_i32, c_vp, c_i64, c_i64, c_vp]),
    "tv_mask_word_summary": (c_i32, [c_vp, c_i32, c_i32, c_i32, c_i64, c_i64, c_vp, c_i64, c_vp]),
    "tv_accept_workspace_size": (c_i32, [ctypes.POINTER(AcceptArgs), ctypes.POINTER(c_size)]),
    "tv_accept": (c_i32, [ctypes.POINTER(AcceptArgs), c_vp]),
    "tv_compact_contig": (c_i32, [c_vp, c_i64, c_i64, c_i64, c_i32, c_i64, c_vp, c_i32, c_vp]),
    "tv_copy_pages": (c_i32, [c_vp, c_i32, c_i64, c_i64, c_i64, c_vp, c_i32, c_i32, c_vp]),
    "tv_compact_paged": (c_i32, [c_vp, c_i32, c_i32, c_i64, c_i64, c_i64, c_i64, c_i32, c_i32, c_vp, c_vp,
                                 c_i32, c_i32, c_i64, c_vp, c_i32, c_vp]),
    "tv_arena_gather": (c_i32, [c_i32, c_i32, c_vp, c_vp, c_i64, c_i64, c_i32, c_vp, c_i64, c_i64, c_i64, c_i32,
                                c_i32, c_i32, c_vp, c_i32, c_vp]),
    "tv_gather_page_table": (c_i32, [c_vp, c_i32, c_vp, c_i32, c_i32, c_vp, c_vp]),
    "tv_rope_append": (c_i32, [ctypes.POINTER(RopeArgs), c_vp]),
    "tv_lmhead_accept_workspace_size": (c_i32, [ctypes.POINTER(LmheadArgs), ctypes.POINTER(c_size)]),
    "tv_lmhead_accept": (c_i32, [ctypes.POINTER(LmheadArgs), c_vp]),
    "tv_tree_finalize": (c_i32, [c_i32, c_i32, c_i32, c_vp, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp,
                                 c_vp, c_vp, c_vp, c_vp]),
    "tv_chunk_select_workspace_size": (c_i32, [c_i32, c_i64, ctypes.POINTER(c_size)]),
    "tv_chunk_select": (c_i32, [c_vp, c_i64, c_vp, c_vp, c_i32, c_i32, c_i64, c_vp, c_vp, c_i64, c_vp, c_vp, c_size,
                                c_vp, c_vp]),
    "tv_gather_rows": (c_i32, [c_i32, c_i32, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i32, c_vp, c_vp, c_i64, c_vp]),
    "tv_rms_norm": (c_i32, [c_vp, c_i64, c_vp, c_vp, c_i64, c_i32, c_i32, c_f32, c_i32, c_vp]),
    "tv_silu_mul": (c_i32, [c_vp, c_vp, c_i64, c_vp, c_i64, c_i32, c_i32, c_i32, c_vp]),
}

EXPORTED = tuple(_SIGNATURES)

_lib = None
_load_error = None


def load():
    """Load the library once; raise SpecVerifyError if it is unavailable."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    if _load_error is not None:
        raise _load_error
    path = os.environ.get("SPECVERIFY_LIB", str(LIB_PATH))
    try:
        lib = ctypes.CDLL(path)
    except OSError as e:
        _load_error = SpecVerifyError(-7, f"cannot load {path} ({e}); build it with "
                                          f"`python specdiff-ae_b200/build.py`")
        raise _load_error
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def available() -> bool:
    try:
        load()
        return True
    except SpecVerifyError:
        return False


def status_string(status: int) -> str:
    try:
        return load().tv_status_string(status).decode()
    except SpecVerifyError:
        return "library not loaded"


def last_cuda_error() -> str:
    try:
        return load().tv_last_cuda_error().decode()
    except SpecVerifyError:
        return ""


def check(status: int, what: str) -> None:
    if status != TV_OK:
        raise SpecVerifyError(status, what)


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dtype]
    except KeyError:
        raise SpecVerifyError(-2, f"dtype {dtype}") from None


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def require_cuda(*tensors) -> torch.device:
    """All tensors on one CUDA device; no CPU path exists."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise SpecVerifyError(-7, "specverify runs on CUDA tensors only (got a CPU tensor)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise SpecVerifyError(-1, f"tensors on different devices: {dev} and {t.device}")
    return dev

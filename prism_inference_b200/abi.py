"""ctypes mirror of include/prism_moe.h and the loader of libprism_moe.so.

The shared library is built in-tree (prism_inference_b200/libprism_moe.so) by
prism_inference_b200/build.py.  Loading fails loudly when it is missing: there is no
CPU or PyTorch fallback for any entry point.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

from .layout import StackLayout

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libprism_moe.so"

PRISM_OK, PRISM_E_ARG, PRISM_E_ALIGN, PRISM_E_RANGE, PRISM_E_CUDA, PRISM_E_TIMEOUT, \
    PRISM_E_NOMEM, PRISM_E_UNSUPPORTED = range(8)
STATUS_NAMES = ["PRISM_OK", "PRISM_E_ARG", "PRISM_E_ALIGN", "PRISM_E_RANGE", "PRISM_E_CUDA",
                "PRISM_E_TIMEOUT", "PRISM_E_NOMEM", "PRISM_E_UNSUPPORTED"]
PRISM_BLOCK_MOE, PRISM_BLOCK_DENSE = 0, 1


def _fields(names):
    return [(n, C.c_int32) for n in names.split()]


class AttnParams(C.Structure):
    _fields_ = _fields("n_tokens dim n_heads head_dim spatial_w spatial_h window_size "
                       "qkv_w qkv_b out_w out_b input_offset output_offset")


class RouterParams(C.Structure):
    _fields_ = _fields("n_tokens dim n_experts router_w router_b input_offset "
                       "assignment_offset count_offset")


class ExpertParams(C.Structure):
    _fields_ = _fields("n_tokens dim expert_id w1_offset b1_offset w2_offset b2_offset "
                       "input_offset output_offset assignment_offset")


class ProjParams(C.Structure):
    _fields_ = _fields("n_tokens w_offset b_offset input_offset output_offset")


class DenseParams(C.Structure):
    _fields_ = _fields("n_tokens dim n_heads head_dim spatial_w spatial_h window_size "
                       "qkv_w_offset qkv_b_offset out_w_offset out_b_offset ffn_w1_offset "
                       "ffn_b1_offset ffn_w2_offset ffn_b2_offset input_offset output_offset")


class BlockDesc(C.Structure):
    _fields_ = _fields("kind qkv_w qkv_b out_w out_b n_experts router_w router_b expert_w1 "
                       "expert_b1 expert_w2 expert_b2 expert_stride ffn_hidden ffn_chunk ffn_w1 "
                       "ffn_b1 ffn_w2 ffn_b2")


class StackDesc(C.Structure):
    _fields_ = _fields("dim n_heads head_dim spatial_w spatial_h window_size in_dim up_w up_b "
                       "out_dim down_w down_b n_blocks") + [("blocks", C.POINTER(BlockDesc))]


def stack_desc(L: StackLayout):
    """(StackDesc, keep-alive block array) for a StackLayout."""
    arr = (BlockDesc * max(1, len(L.blocks)))()
    for i, b in enumerate(L.blocks):
        d = arr[i]
        d.kind = PRISM_BLOCK_MOE if b.kind == "moe" else PRISM_BLOCK_DENSE
        for f in ("qkv_w", "qkv_b", "out_w", "out_b", "n_experts", "router_w", "router_b",
                  "expert_w1", "expert_b1", "expert_w2", "expert_b2", "expert_stride",
                  "ffn_hidden", "ffn_chunk", "ffn_w1", "ffn_b1", "ffn_w2", "ffn_b2"):
            setattr(d, f, getattr(b, f))
    s = StackDesc(dim=L.dim, n_heads=L.n_heads, head_dim=L.head_dim, spatial_w=L.spatial_w,
                  spatial_h=L.spatial_h, window_size=L.window_size, in_dim=L.in_dim,
                  up_w=L.up_w, up_b=L.up_b, out_dim=L.out_dim, down_w=L.down_w,
                  down_b=L.down_b, n_blocks=len(L.blocks))
    s.blocks = C.cast(arr, C.POINTER(BlockDesc))
    return s, arr


# Every symbol include/prism_moe.h declares (checked by tests without a GPU).
EXPORTS = ("prism_create", "prism_destroy", "prism_last_error_string", "prism_abi_version",
           "prism_attn_window", "prism_router", "prism_expert", "prism_proj_up",
           "prism_proj_down", "prism_dense_block", "prism_stack_create", "prism_stack_destroy",
           "prism_stack_forward", "prism_stack_status", "prism_stack_launch_count",
           "prism_stack_tokens_per_frame", "prism_stack_profile", "prism_stack_profile_read", "prism_stack_set_option",
           "prism_expert_all_static", "prism_stack_inject_stall", "prism_stack_infer",
           "prism_stack_submit", "prism_stack_wait", "prism_moe_block", "prism_stack_infer_gpu",
           "prism_codec_pass", "prism_ctx_status")
# prism_codec_kind order = the shaders of oracle.CODEC_KINDS
CODEC_KINDS = ("conv3x3_coopvec_9ch", "strided_conv_coopvec_32ch", "strided_conv_split_64ch",
               "strided_conv_split_128ch", "dec3_fused", "dec2_fused", "dec1_fused",
               "pw_conv_coopvec_32to12", "pixelshuffle_sigmoid")
STATIC_MAX_TOKENS = 65536  # PRISM_STATIC_MAX_TOKENS
# prism_stack_option
OPT_PAIR_ATTENTION = 1
OPT_BUCKET_ROUTING = 2
KERNEL_KINDS = ("proj_up", "attn", "router", "route", "expert", "dense_ffn", "proj_down", "copy")

_lib = None


def load(path: os.PathLike | None = None) -> C.CDLL:
    """Load libprism_moe.so (raises if it has not been built)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(f"{p} is missing: build it with python -m prism_inference_b200.build "
                           "(there is no CPU fallback)")
    lib = C.CDLL(str(p))
    vp, sz, i32, i32p = C.c_void_p, C.c_size_t, C.c_int, C.POINTER(C.c_int32)
    sig = {
        "prism_create": (i32, [i32, C.POINTER(vp)]),
        "prism_destroy": (i32, [vp]),
        "prism_last_error_string": (C.c_char_p, []),
        "prism_abi_version": (i32, []),
        "prism_attn_window": (i32, [vp, C.POINTER(AttnParams), vp, sz, vp, sz, vp]),
        "prism_router": (i32, [vp, C.POINTER(RouterParams), vp, sz, vp, sz, vp, sz, vp]),
        "prism_expert": (i32, [vp, C.POINTER(ExpertParams), vp, sz, vp, sz, vp, sz, vp]),
        "prism_proj_up": (i32, [vp, C.POINTER(ProjParams), vp, sz, vp, sz, vp]),
        "prism_proj_down": (i32, [vp, C.POINTER(ProjParams), vp, sz, vp, sz, vp]),
        "prism_dense_block": (i32, [vp, C.POINTER(DenseParams), C.c_int32, C.c_int32, vp, sz, vp,
                                    sz, vp]),
        "prism_stack_create": (i32, [vp, C.POINTER(StackDesc), vp, sz, i32, i32, C.POINTER(vp)]),
        "prism_stack_destroy": (i32, [vp]),
        "prism_stack_forward": (i32, [vp, vp, vp, i32, vp, vp]),
        "prism_stack_status": (i32, [vp, vp]),
        "prism_stack_inject_stall": (i32, [vp, vp]),
        "prism_stack_infer": (i32, [vp, vp, vp, i32, C.POINTER(C.c_float)]),
        "prism_stack_infer_gpu": (i32, [vp, vp, sz, vp, sz, i32, C.POINTER(C.c_float)]),
        "prism_codec_pass": (i32, [vp, i32, C.POINTER(C.c_int32), i32, vp, sz, vp, sz, vp, sz, vp]),
        "prism_ctx_status": (i32, [vp, vp]),
        "prism_moe_block": (i32, [vp, vp, vp, i32, vp, vp, vp]),
        "prism_stack_submit": (i32, [vp, vp, vp, i32, vp, C.POINTER(C.c_int64)]),
        "prism_stack_wait": (i32, [vp, C.c_int64, vp]),
        "prism_stack_launch_count": (i32, [vp, i32]),
        "prism_stack_tokens_per_frame": (i32, [vp]),
        "prism_stack_profile": (i32, [vp, i32]),
        "prism_stack_set_option": (i32, [vp, i32, i32]),
        "prism_expert_all_static": (i32, [vp, C.POINTER(ExpertParams), C.c_int32, C.c_int32, vp, sz, vp, sz, vp,
                                          sz, vp]),
        "prism_stack_profile_read": (i32, [vp, C.POINTER(C.c_double), C.POINTER(C.c_int64), i32]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    if path is None:
        _lib = lib
    return lib


class PrismError(RuntimeError):
    def __init__(self, status: int, msg: str):
        self.status = status
        name = STATUS_NAMES[status] if 0 <= status < len(STATUS_NAMES) else str(status)
        super().__init__(f"{name}: {msg}")


def check(lib, status: int):
    if status != PRISM_OK:
        raise PrismError(status, lib.prism_last_error_string().decode())
    return status

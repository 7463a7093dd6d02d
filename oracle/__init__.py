"""TEST INFRASTRUCTURE, NOT THE PRODUCT.

ctypes access to the two CPU checkers:
  * liboracle.so       - the C++ restatement of the reference GLSL (prism_oracle.cpp)
  * _ref/libglsl_ref.so - the reference's own shader sources compiled as C++ through
                          glsl_ref/ (built only where the reference tree exists; the
                          built library travels with the repository snapshot)

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, and only as the checker or the timed CPU baseline, never as the product.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

from prism_inference_b200.abi import (AttnParams, DenseParams, ExpertParams, ProjParams,
                                      RouterParams, StackDesc, stack_desc)
from prism_inference_b200.layout import StackLayout

ORACLE_DIR = Path(__file__).resolve().parent
LIB = ORACLE_DIR / "liboracle.so"
REF_LIB = ORACLE_DIR / "_ref" / "libglsl_ref.so"
REF_SHADERS = ("split2_qkv_attn_d256", "moe_router", "moe_expert_skip", "moe_ffn_16exp",
               "pw_project_128to256", "pw_project_256to128", "attention_windowed_d256",
               "attention_windowed",
               # the encoder / decoder around the stack (prism_moe_bench.cpp:386-471)
               "conv3x3_coopvec_9ch", "strided_conv_coopvec_32ch", "strided_conv_split_64ch",
               "strided_conv_split_128ch", "dec3_fused", "dec2_fused", "dec1_fused",
               "pw_conv_coopvec_32to12", "pixelshuffle_sigmoid")

# order of enum oracle_codec_kind (prism_oracle.h)
CODEC_KINDS = ("conv3x3_coopvec_9ch", "strided_conv_coopvec_32ch", "strided_conv_split_64ch",
               "strided_conv_split_128ch", "dec3_fused", "dec2_fused", "dec1_fused",
               "pw_conv_coopvec_32to12", "pixelshuffle_sigmoid")

_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")


def build(ref: bool = False):
    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)] + (["ref"] if ref else []), check=True)


class Oracle:
    def __init__(self):
        if not LIB.exists():
            build()
        L = C.CDLL(str(LIB))
        vp = C.c_void_p
        L.oracle_attn_window.argtypes = [C.POINTER(AttnParams), _u16p, _u16p]
        L.oracle_router.argtypes = [C.POINTER(RouterParams), _u16p, _u16p, _i32p, vp]
        L.oracle_expert.argtypes = [C.POINTER(ExpertParams), _u16p, _u16p, _i32p]
        L.oracle_proj_up.argtypes = [C.POINTER(ProjParams), _u16p, _u16p]
        L.oracle_proj_down.argtypes = [C.POINTER(ProjParams), _u16p, _u16p]
        L.oracle_dense_block.argtypes = [C.POINTER(DenseParams), C.c_int32, C.c_int32, _u16p, _u16p]
        L.oracle_stack_forward.argtypes = [C.POINTER(StackDesc), _u16p, C.c_size_t, _u16p, _u16p,
                                           C.c_int, vp, vp, C.c_float, vp]
        L.oracle_stack_forward.restype = C.c_int
        L.oracle_f2h.argtypes, L.oracle_f2h.restype = [C.c_float], C.c_uint16
        L.oracle_h2f.argtypes, L.oracle_h2f.restype = [C.c_uint16], C.c_float
        L.oracle_gelu_h.argtypes, L.oracle_gelu_h.restype = [C.c_float], C.c_float
        L.oracle_codec_pass.argtypes = [C.c_int, _i32p, C.c_int, _u16p, _u16p, C.c_void_p]
        L.oracle_codec_pass.restype = C.c_int
        L.oracle_num_threads.restype = C.c_int
        L.oracle_set_num_threads.argtypes = [C.c_int]
        self.lib = L

    # per-pass (arena semantics: features / aux are updated in place)
    def attn(self, p: AttnParams, weights, features):
        self.lib.oracle_attn_window(C.byref(p), _u16(weights), _u16(features))

    def router(self, p: RouterParams, weights, features, aux, want_margin=False):
        m = np.zeros(p.n_tokens, np.float32) if want_margin else None
        self.lib.oracle_router(C.byref(p), _u16(weights), _u16(features), aux,
                               m.ctypes.data if m is not None else None)
        return m

    def expert(self, p: ExpertParams, weights, features, aux):
        self.lib.oracle_expert(C.byref(p), _u16(weights), _u16(features), aux)

    def proj_up(self, p: ProjParams, weights, features):
        self.lib.oracle_proj_up(C.byref(p), _u16(weights), _u16(features))

    def proj_down(self, p: ProjParams, weights, features):
        self.lib.oracle_proj_down(C.byref(p), _u16(weights), _u16(features))

    def dense(self, p: DenseParams, hidden, chunk, weights, features):
        self.lib.oracle_dense_block(C.byref(p), hidden, chunk, _u16(weights), _u16(features))

    def stack(self, L: StackLayout, blob, frames_in, forced=None, tie_thr=1e-3):
        """Run the whole stack.  Returns (out fp16 [F][T][out_dim], assign int32
        [n_moe][F*T], stats int64[4])."""
        F = frames_in.shape[0]
        T = L.tokens
        out = np.zeros((F, T, L.out_dim), np.float16)
        assign = np.zeros((max(1, L.n_moe_blocks), F * T), np.int32)
        stats = np.zeros(4, np.int64)
        desc, keep = stack_desc(L)
        fa = None
        if forced is not None:
            fa = np.ascontiguousarray(forced, dtype=np.int32)
        rc = self.lib.oracle_stack_forward(C.byref(desc), _u16(blob), blob.size,
                                           _u16(np.ascontiguousarray(frames_in)), _u16(out), F,
                                           assign.ctypes.data, fa.ctypes.data if fa is not None else None,
                                           tie_thr, stats.ctypes.data)
        if rc != 0:
            raise RuntimeError("oracle_stack_forward: invalid descriptor")
        return out, assign, stats

    def codec_pass(self, shader: str, push, weights, features, rgb=None):
        """One encoder / decoder pass (CODEC_KINDS) with the shader's push constants, on the
        feature arena in place; rgb receives pixelshuffle_sigmoid's output."""
        pc = np.ascontiguousarray(np.asarray(push, dtype=np.int32))
        rc = self.lib.oracle_codec_pass(CODEC_KINDS.index(shader), pc, pc.size, _u16(weights), _u16(features),
                                        _u16(rgb).ctypes.data if rgb is not None else None)
        if rc != 0:
            raise ValueError(f"oracle_codec_pass({shader}): bad push constants")

    def f2h(self, x):
        return self.lib.oracle_f2h(x)

    def gelu_h(self, x):
        return self.lib.oracle_gelu_h(x)


def use_host_threads(n: int | None = None) -> int:
    """Let the OpenMP runtime of the host libraries (the system libgomp, which reads
    OMP_NUM_THREADS once at start-up - torchrun sets it to 1) use n threads (default: all
    host cores) in parallel regions started from this thread.  Returns n."""
    import os
    n = n or os.cpu_count() or 1
    C.CDLL("libgomp.so.1").omp_set_num_threads(C.c_int(n))
    return n


class GlslRef:
    """The reference's shader sources, executed on the host (see glsl_ref/)."""

    def __init__(self):
        if not REF_LIB.exists():
            raise FileNotFoundError(REF_LIB)
        L = C.CDLL(str(REF_LIB))
        self.fns = {}
        for s in REF_SHADERS:
            f = getattr(L, f"glslref_{s}")
            f.argtypes = [_i32p, C.c_int, _u16p, _u16p, C.c_void_p, C.c_int]
            f.restype = C.c_int
            n = getattr(L, f"glslref_{s}_n_push")
            n.restype = C.c_int
            ls = getattr(L, f"glslref_{s}_local_size")
            ls.restype = C.c_int
            ly = getattr(L, f"glslref_{s}_local_size_y")
            ly.restype = C.c_int
            if ly() > 1:  # 2-D workgroups: the _2d entry takes the group grid
                f = getattr(L, f"glslref_{s}_2d")
                f.argtypes = [_i32p, C.c_int, _u16p, _u16p, C.c_void_p, C.c_int, C.c_int]
                f.restype = C.c_int
            self.fns[s] = (f, n(), ls(), ly())
        self.lib = L

    def dispatch(self, shader: str, push, weights, features, aux=None, n_groups=1):
        """n_groups: an int, or (groups_x, groups_y) for a shader with 2-D workgroups.  aux is
        binding 2 (int32 for the router / experts, fp16 for pixelshuffle's RGB output)."""
        f, n_push, _, ly = self.fns[shader]
        pc = np.ascontiguousarray(np.asarray(push, dtype=np.int32))
        if pc.size != n_push:
            raise ValueError(f"{shader}: {n_push} push constants expected, got {pc.size}")
        grid = tuple(n_groups) if isinstance(n_groups, (tuple, list)) else (n_groups,)
        if (len(grid) == 2) != (ly > 1):
            raise ValueError(f"{shader}: workgroup grid {grid} does not match its workgroup shape")
        rc = f(pc, pc.size, _u16(weights), _u16(features),
               aux.ctypes.data if aux is not None else None, *grid)
        if rc != 0:
            raise RuntimeError(f"{shader}: dispatch failed")

    def local_size(self, shader: str) -> int:
        return self.fns[shader][2]


def _u16(a):
    """View an fp16/uint16 numpy array as uint16 without copying."""
    if a.dtype == np.float16:
        return a.view(np.uint16)
    return a

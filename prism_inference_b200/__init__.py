"""prism_inference_b200 - B200 (sm_100a) implementation of Prism's bottleneck
transformer / MoE stack behind the C ABI of include/prism_moe.h.

The Python layer is a thin host mirror over libprism_moe.so (ctypes): PyTorch is
used only to own device memory and streams.  Two interfaces:

* the per-pass drop-ins, one call per reference vkCmdDispatch, taking the same
  push-constant blocks (AttnParams, RouterParams, ExpertParams, ProjParams,
  DenseParams) and the three arenas (fp16 weight blob, fp16 feature arena, int32 aux
  arena) - the dispatch contract of prism_moe_bench.cpp:213-505;
* Stack: the whole stack of a StackLayout over a batch of frames (the fast path).

No entry point falls back to the CPU: a missing libprism_moe.so raises.
"""
from __future__ import annotations

import ctypes as C

from . import abi, configs, layout, synth
from .abi import (AttnParams, DenseParams, ExpertParams, PrismError, ProjParams, RouterParams,
                  check)
from .layout import StackLayout, build_stack

__all__ = ["Prism", "Stack", "AttnParams", "RouterParams", "ExpertParams", "ProjParams",
           "DenseParams", "PrismError", "StackLayout", "build_stack", "configs", "layout", "synth"]


def _ptr(t) -> int:
    return t.data_ptr()


def _host_ptr(a) -> int | None:
    """Address of a host array (CPU tensor or numpy array); None passes through."""
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        if a.is_cuda or not a.is_contiguous():
            raise ValueError("expected a contiguous host tensor")
        return a.data_ptr()
    if not a.flags["C_CONTIGUOUS"]:
        raise ValueError("expected a C-contiguous array")
    return a.ctypes.data


def _stream(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return getattr(stream, "cuda_stream", stream)


class Prism:
    """One context per CUDA device (prism_create)."""

    def __init__(self, device: int = 0):
        self.lib = abi.load()
        self.device = device
        h = C.c_void_p()
        check(self.lib, self.lib.prism_create(device, C.byref(h)))
        self.h = h

    def close(self):
        if self.h:
            self.lib.prism_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- per-pass drop-ins (tensors are flat CUDA arenas) ------------------------
    def attn_window(self, p: AttnParams, weights, features, stream=None):
        check(self.lib, self.lib.prism_attn_window(self.h, C.byref(p), _ptr(weights), weights.numel(),
                                                   _ptr(features), features.numel(), _stream(stream)))

    def router(self, p: RouterParams, weights, features, aux, stream=None):
        check(self.lib, self.lib.prism_router(self.h, C.byref(p), _ptr(weights), weights.numel(),
                                              _ptr(features), features.numel(), _ptr(aux), aux.numel(),
                                              _stream(stream)))

    def expert(self, p: ExpertParams, weights, features, aux, stream=None):
        check(self.lib, self.lib.prism_expert(self.h, C.byref(p), _ptr(weights), weights.numel(),
                                              _ptr(features), features.numel(), _ptr(aux), aux.numel(),
                                              _stream(stream)))

    def expert_all_static(self, p: ExpertParams, n_experts: int, expert_stride: int, weights, features, aux,
                          stream=None):
        """All experts of one pass in one call without device allocation
        (prism_expert_all_static): scratch lives in a fixed per-device array."""
        check(self.lib, self.lib.prism_expert_all_static(self.h, C.byref(p), n_experts, expert_stride, _ptr(weights),
                                                         weights.numel(), _ptr(features), features.numel(), _ptr(aux),
                                                         aux.numel(), _stream(stream)))

    def proj_up(self, p: ProjParams, weights, features, stream=None):
        check(self.lib, self.lib.prism_proj_up(self.h, C.byref(p), _ptr(weights), weights.numel(),
                                               _ptr(features), features.numel(), _stream(stream)))

    def proj_down(self, p: ProjParams, weights, features, stream=None):
        check(self.lib, self.lib.prism_proj_down(self.h, C.byref(p), _ptr(weights), weights.numel(),
                                                 _ptr(features), features.numel(), _stream(stream)))

    def dense_block(self, p: DenseParams, ffn_hidden: int, ffn_chunk: int, weights, features, stream=None):
        check(self.lib, self.lib.prism_dense_block(self.h, C.byref(p), ffn_hidden, ffn_chunk, _ptr(weights),
                                                   weights.numel(), _ptr(features), features.numel(),
                                                   _stream(stream)))

    def codec_pass(self, shader: str, push, weights, features, rgb=None, stream=None):
        """prism_codec_pass: one dispatch of an encoder / decoder shader (abi.CODEC_KINDS) with
        its push constants, on CUDA fp16 tensors (weights = binding 0, features = binding 1,
        rgb = binding 2 for pixelshuffle_sigmoid)."""
        pc = (C.c_int32 * len(push))(*[int(v) for v in push])
        check(self.lib, self.lib.prism_codec_pass(self.h, abi.CODEC_KINDS.index(shader), pc, len(push),
                                                  _ptr(weights), weights.numel(), _ptr(features), features.numel(),
                                                  _ptr(rgb) if rgb is not None else None,
                                                  rgb.numel() if rgb is not None else 0, _stream(stream)))

    def status(self, stream=None):
        """prism_ctx_status: raises PrismError if a per-pass kernel's bounded wait gave up."""
        check(self.lib, self.lib.prism_ctx_status(self.h, _stream(stream)))


class Stack:
    """The whole stack of a StackLayout (prism_stack_create / prism_stack_forward).

    blob: numpy fp16/uint16 array (host) or a CUDA fp16 tensor (device)."""

    def __init__(self, ctx: Prism, L: StackLayout, blob, max_frames: int):
        self.ctx, self.lib, self.layout, self.max_frames = ctx, ctx.lib, L, max_frames
        self._desc, self._keep = abi.stack_desc(L)
        h = C.c_void_p()
        if hasattr(blob, "data_ptr"):
            ptr, n, on_host = blob.data_ptr(), blob.numel(), 0
        else:
            ptr, n, on_host = blob.ctypes.data, blob.size, 1
        check(self.lib, self.lib.prism_stack_create(ctx.h, C.byref(self._desc), ptr, n, on_host, max_frames,
                                                    C.byref(h)))
        self.h = h

    def forward(self, x, out, assign=None, stream=None):
        """x: CUDA fp16 [F, T, in_dim]; out: CUDA fp16 [F, T, out_dim];
        assign: optional CUDA int32 [n_moe_blocks, F*T]."""
        F = x.shape[0]
        check(self.lib, self.lib.prism_stack_forward(self.h, _ptr(x), _ptr(out), F,
                                                     _ptr(assign) if assign is not None else None,
                                                     _stream(stream)))
        return out

    def moe_block(self, x, out, assign=None, counts=None, stream=None):
        """prism_moe_block (a stack of one MoE block, no adapters): x / out CUDA fp16
        [F, T, dim] (views into a feature arena work), assign CUDA int32 [F*T] and counts
        CUDA int32 [n_experts], both optional."""
        check(self.lib, self.lib.prism_moe_block(self.h, _ptr(x), _ptr(out), x.shape[0],
                                                 _ptr(assign) if assign is not None else None,
                                                 _ptr(counts) if counts is not None else None,
                                                 _stream(stream)))
        return out

    def infer(self, host_in, host_out=None) -> float:
        """prism_stack_infer: host_in [F, T, in_dim] / host_out [F, T, out_dim] fp16 host
        arrays (CPU tensors, page-locked for DMA, or numpy arrays); synchronous.  Returns
        the forward's device time in ms."""
        ms = C.c_float()
        check(self.lib, self.lib.prism_stack_infer(self.h, _host_ptr(host_in), _host_ptr(host_out),
                                                   host_in.shape[0], C.byref(ms)))
        return ms.value

    def infer_gpu(self, in_buf, out_buf, frames: int, in_offset: int = 0, out_offset: int = 0) -> float:
        """prism_stack_infer_gpu (the reference's InferGPU): in_buf / out_buf are CUDA tensors
        (any dtype) holding [frames, T, in_dim] / [frames, T, out_dim] fp16 at the given BYTE
        offsets; synchronous.  Returns the forward's device time in ms."""
        ms = C.c_float()
        check(self.lib, self.lib.prism_stack_infer_gpu(self.h, in_buf.data_ptr(), in_offset, out_buf.data_ptr(),
                                                       out_offset, frames, C.byref(ms)))
        return ms.value

    def submit(self, host_in, host_out=None, stream=None) -> int:
        """prism_stack_submit: enqueue upload, forward and download; returns the ticket."""
        t = C.c_int64()
        check(self.lib, self.lib.prism_stack_submit(self.h, _host_ptr(host_in), _host_ptr(host_out),
                                                    host_in.shape[0], _stream(stream), C.byref(t)))
        return t.value

    def wait(self, ticket: int, stream=None, host: bool = True):
        """prism_stack_wait: block the host (default) or make `stream` wait on the device."""
        check(self.lib, self.lib.prism_stack_wait(self.h, ticket, None if host else _stream(stream)))

    def status(self, stream=None):
        check(self.lib, self.lib.prism_stack_status(self.h, _stream(stream)))

    def inject_stall(self, stream=None):
        """Diagnostic (prism_stack_inject_stall): a device wait that nothing releases; the
        next status() raises PRISM_E_TIMEOUT after the library's wait limit."""
        check(self.lib, self.lib.prism_stack_inject_stall(self.h, _stream(stream)))

    def set_pair_attention(self, enable: bool):
        """PRISM_OPT_PAIR_ATTENTION: few-tile dim-256 attention on CTA pairs (default on)."""
        check(self.lib, self.lib.prism_stack_set_option(self.h, abi.OPT_PAIR_ATTENTION, int(enable)))

    def set_bucket_routing(self, enable: bool):
        """PRISM_OPT_BUCKET_ROUTING: router-filled expert buckets, no route kernel (default on)."""
        check(self.lib, self.lib.prism_stack_set_option(self.h, abi.OPT_BUCKET_ROUTING, int(enable)))

    def profile(self, enable: bool = True):
        check(self.lib, self.lib.prism_stack_profile(self.h, int(enable)))

    def profile_read(self):
        """{kernel kind: (total ms, launches)} since the last read (synchronises)."""
        n = len(abi.KERNEL_KINDS)
        ms, cnt = (C.c_double * n)(), (C.c_int64 * n)()
        check(self.lib, self.lib.prism_stack_profile_read(self.h, ms, cnt, n))
        return {k: (ms[i], cnt[i]) for i, k in enumerate(abi.KERNEL_KINDS) if cnt[i]}

    def launch_count(self, frames: int) -> int:
        return self.lib.prism_stack_launch_count(self.h, frames)

    def close(self):
        if self.h:
            self.lib.prism_stack_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

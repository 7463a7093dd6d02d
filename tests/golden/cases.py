"""Golden cases: small seeded inputs for every reference shader on the hot path.

Each case builds (shader, push constants, weight blob, feature arena, aux arena,
workgroup count) deterministically from numpy PCG64 seeds, so the inputs are rebuilt
at test time and only the outputs are stored (golden.npz, written by
make_golden.py from the reference's own shader sources run through
oracle/glsl_ref).  The frames are 16x12 tokens (2x2 windows, the bottom window row
half outside the frame, so phantom keys are exercised) except where noted.
"""
from __future__ import annotations

import hashlib

import numpy as np

from prism_inference_b200 import layout, synth

W, H = 16, 12
T = W * H


def _arena(n, x=None):
    f = np.zeros(n, np.float16)
    if x is not None:
        f[: x.size] = x.reshape(-1)
    return f


def _moe(n_experts, w=W, h=H, seed=synth.WEIGHT_SEED):
    L = layout.build_stack(256, 1, n_experts=n_experts, spatial_w=w, spatial_h=h)
    return L, synth.make_blob(L, seed=seed)


def build(name):
    """-> dict(shader, push, blob, feat, aux, groups, out=(array name, slice))"""
    if name == "attn_d256":
        L, blob = _moe(4)
        b = L.blocks[0]
        x = synth.make_frames(L, 1)[0]
        push = [T, 256, 8, 32, W, H, 8, b.qkv_w, b.qkv_b, b.out_w, b.out_b, 0, T * 256]
        return dict(shader="split2_qkv_attn_d256", push=push, blob=blob, feat=_arena(2 * T * 256, x), aux=None,
                    groups=4, out=("feat", slice(T * 256, 2 * T * 256)))
    if name == "attn_d256_16tok":
        # 4x4 frame: n_tokens = 16 < 64, so only the first 16 window slots are keys
        L, blob = _moe(4, w=4, h=4)
        b = L.blocks[0]
        t = 16
        x = synth.make_frames(L, 1)[0]
        push = [t, 256, 8, 32, 4, 4, 8, b.qkv_w, b.qkv_b, b.out_w, b.out_b, 0, t * 256]
        return dict(shader="split2_qkv_attn_d256", push=push, blob=blob, feat=_arena(2 * t * 256, x), aux=None,
                    groups=1, out=("feat", slice(t * 256, 2 * t * 256)))
    if name in ("router4", "expert_skip4"):
        L, blob = _moe(4)
        b = L.blocks[0]
        rng = np.random.Generator(np.random.PCG64(11))
        y = (rng.standard_normal(T * 256, dtype=np.float32)).astype(np.float16)
        feat = _arena(2 * T * 256, y)
        if name == "router4":
            push = [T, 256, 4, b.router_w, b.router_b, 0, 0, T]
            return dict(shader="moe_router", push=push, blob=blob, feat=feat, aux=np.zeros(T + 64, np.int32),
                        groups=(T + 255) // 256, out=("aux", slice(0, T + 4)))
        aux = np.zeros(T + 64, np.int32)
        aux[:T] = rng.integers(0, 4, T, dtype=np.int32)
        pushes = []
        for e in range(4):
            eo = e * b.expert_stride
            pushes.append([T, 256, e, b.expert_w1 + eo, b.expert_b1 + eo, b.expert_w2 + eo, b.expert_b2 + eo,
                           0, T * 256, 0])
        return dict(shader="moe_expert_skip", push=pushes, blob=blob, feat=feat, aux=aux,
                    groups=(T + 255) // 256, out=("feat", slice(T * 256, 2 * T * 256)))
    if name == "moe_ffn_16exp":
        L, blob = _moe(16)
        b = L.blocks[0]
        rng = np.random.Generator(np.random.PCG64(12))
        y = (rng.standard_normal(T * 256, dtype=np.float32)).astype(np.float16)
        push = [T, 256, b.router_w, b.router_b, b.expert_stride, b.expert_w1, b.expert_b1, b.expert_w2,
                b.expert_b2, 0, T * 256]
        return dict(shader="moe_ffn_16exp", push=push, blob=blob, feat=_arena(2 * T * 256, y), aux=None,
                    groups=(T + 255) // 256, out=("feat", slice(T * 256, 2 * T * 256)))
    if name == "dense_d256_h1024":
        L = layout.build_stack(256, 1, ffn_hidden=1024, ffn_chunk=256, spatial_w=W, spatial_h=H)
        blob = synth.make_blob(L)
        b = L.blocks[0]
        x = synth.make_frames(L, 1)[0]
        push = [T, 256, 8, 32, W, H, 8, b.qkv_w, b.qkv_b, b.out_w, b.out_b, b.ffn_w1, b.ffn_b1, b.ffn_w2,
                b.ffn_b2, 0, T * 256]
        return dict(shader="attention_windowed_d256", push=push, blob=blob, feat=_arena(2 * T * 256, x),
                    aux=None, groups=4, out=("feat", slice(T * 256, 2 * T * 256)))
    if name == "dense_d128_h512":
        L = layout.build_stack(128, 1, n_heads=4, ffn_hidden=512, ffn_chunk=512, spatial_w=W, spatial_h=H)
        blob = synth.make_blob(L)
        b = L.blocks[0]
        x = synth.make_frames(L, 1)[0]
        push = [T, 128, 4, 32, W, H, 8, b.qkv_w, b.qkv_b, b.out_w, b.out_b, b.ffn_w1, b.ffn_b1, b.ffn_w2,
                b.ffn_b2, 0, T * 128]
        return dict(shader="attention_windowed", push=push, blob=blob, feat=_arena(2 * T * 128, x), aux=None,
                    groups=4, out=("feat", slice(T * 128, 2 * T * 128)))
    if name in ("proj_up", "proj_down"):
        L = layout.build_stack(256, 0, up_adapter=True, down_adapter=True, spatial_w=W, spatial_h=H)
        blob = synth.make_blob(L)
        rng = np.random.Generator(np.random.PCG64(13))
        if name == "proj_up":
            x = rng.standard_normal(T * 128, dtype=np.float32).astype(np.float16)
            return dict(shader="pw_project_128to256", push=[T, L.up_w, L.up_b, 0, T * 128], blob=blob,
                        feat=_arena(T * (128 + 256), x), aux=None, groups=(T + 255) // 256,
                        out=("feat", slice(T * 128, T * 384)))
        x = rng.standard_normal(T * 256, dtype=np.float32).astype(np.float16)
        return dict(shader="pw_project_256to128", push=[T, L.down_w, L.down_b, 0, T * 256], blob=blob,
                    feat=_arena(T * (256 + 128), x), aux=None, groups=(T + 255) // 256,
                    out=("feat", slice(T * 256, T * 384)))
    raise KeyError(name)


CASES = ("attn_d256", "attn_d256_16tok", "router4", "expert_skip4", "moe_ffn_16exp", "dense_d256_h1024",
         "dense_d128_h512", "proj_up", "proj_down")


def input_digest(case) -> str:
    h = hashlib.sha256()
    h.update(np.ascontiguousarray(case["blob"]).view(np.uint16).tobytes())
    h.update(np.ascontiguousarray(case["feat"]).view(np.uint16).tobytes())
    if case["aux"] is not None:
        h.update(case["aux"].tobytes())
    return h.hexdigest()


def output_of(case):
    arr_name, sl = case["out"]
    return case[arr_name][sl].copy()

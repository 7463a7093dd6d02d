"""Golden cases: small seeded inputs for every reference shader on the hot path, and for
the encoder / decoder shaders around it (CODEC_CASES).

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
    if name in CODEC_CASES:
        return _codec(name)
    raise KeyError(name)


# ---- the encoder / decoder around the stack (prism_moe_bench.cpp:386-471), CHW feature maps.
# A 24x14 frame and its stride-2 pyramid 12x7, 6x4, 3x2 (odd heights round up, as 135 -> 68
# does in the reference).  Every case is one dispatch on its own seeded inputs.
R = ((24, 14), (12, 7), (6, 4), (3, 2))
P = tuple(w * h for w, h in R)


def _codec_weights(rows, cols, seed):
    """[rows][cols] row-major weights ~ N(0, 1/cols) followed by [rows] biases ~ N(0, 0.1)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    w = (rng.standard_normal(rows * cols, dtype=np.float32) / np.float32(np.sqrt(cols))).astype(np.float16)
    b = (rng.standard_normal(rows, dtype=np.float32) * np.float32(0.1)).astype(np.float16)
    return np.concatenate([w, b]), 0, rows * cols


def _codec_features(sizes, seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    return [rng.standard_normal(n, dtype=np.float32).astype(np.float16) for n in sizes]


def _codec(name):
    (w0, h0), (w1, h1), (w2, h2), (w3, h3) = R
    p0, p1, p2, p3 = P
    g = lambda n: (n + 255) // 256  # noqa: E731
    if name == "enc_ic":  # conv3x3_coopvec_9ch: 9 -> 32, ReLU
        blob, wo, bo = _codec_weights(32, 81, 21)
        (x,) = _codec_features([9 * p0], 31)
        return dict(shader="conv3x3_coopvec_9ch", push=[9, 32, w0, h0, wo, bo, 0, 9 * p0, 1], blob=blob,
                    feat=_arena(9 * p0 + 32 * p0, x), aux=None, groups=g(p0), out=("feat", slice(9 * p0, 41 * p0)))
    if name == "enc1":  # strided_conv_coopvec_32ch: 32 -> 64, stride 2
        blob, wo, bo = _codec_weights(64, 288, 22)
        (x,) = _codec_features([32 * p0], 32)
        return dict(shader="strided_conv_coopvec_32ch", push=[32, 64, w0, h0, w1, h1, wo, bo, 0, 32 * p0],
                    blob=blob, feat=_arena(32 * p0 + 64 * p1, x), aux=None, groups=g(p1),
                    out=("feat", slice(32 * p0, 32 * p0 + 64 * p1)))
    if name == "enc2":  # strided_conv_split_64ch: 64 -> 128, two 32-channel groups
        blob, wo, bo = _codec_weights(128, 576, 23)
        (x,) = _codec_features([64 * p1], 33)
        return dict(shader="strided_conv_split_64ch", push=[64, 128, w1, h1, w2, h2, wo, bo, 0, 64 * p1],
                    blob=blob, feat=_arena(64 * p1 + 128 * p2, x), aux=None, groups=g(p2),
                    out=("feat", slice(64 * p1, 64 * p1 + 128 * p2)))
    if name == "enc3":  # strided_conv_split_128ch: 128 -> 128, four groups, fp16 running sum
        blob, wo, bo = _codec_weights(128, 1152, 24)
        (x,) = _codec_features([128 * p2], 34)
        return dict(shader="strided_conv_split_128ch", push=[128, 128, w2, h2, w3, h3, wo, bo, 0, 128 * p2],
                    blob=blob, feat=_arena(128 * p2 + 128 * p3, x), aux=None, groups=g(p3),
                    out=("feat", slice(128 * p2, 128 * p2 + 128 * p3)))
    if name == "dec3":  # upsample 128 @ r3 + skip 128 @ r2 -> PW 256 -> 128, ReLU
        blob, wo, bo = _codec_weights(128, 256, 25)
        up, skip = _codec_features([128 * p3, 128 * p2], 35)
        o = 128 * p3 + 128 * p2
        return dict(shader="dec3_fused", push=[w2, h2, w3, h3, 128, wo, bo, 0, 128 * p3, o], blob=blob,
                    feat=_arena(o + 128 * p2, np.concatenate([up, skip])), aux=None, groups=g(p2),
                    out=("feat", slice(o, o + 128 * p2)))
    if name == "dec2":  # upsample 128 @ r2 + skip 64 @ r1 -> PW 192 -> 64, ReLU
        blob, wo, bo = _codec_weights(64, 192, 26)
        up, skip = _codec_features([128 * p2, 64 * p1], 36)
        o = 128 * p2 + 64 * p1
        return dict(shader="dec2_fused", push=[w1, h1, w2, h2, 128, 64, wo, bo, 0, 128 * p2, o], blob=blob,
                    feat=_arena(o + 64 * p1, np.concatenate([up, skip])), aux=None, groups=g(p1),
                    out=("feat", slice(o, o + 64 * p1)))
    if name == "dec1":  # upsample 64 @ r1 + skip 32 @ r0 -> PW 96 -> 32, ReLU
        blob, wo, bo = _codec_weights(32, 96, 27)
        up, skip = _codec_features([64 * p1, 32 * p0], 37)
        o = 64 * p1 + 32 * p0
        return dict(shader="dec1_fused", push=[w0, h0, w1, h1, 64, 32, wo, bo, 0, 64 * p1, o], blob=blob,
                    feat=_arena(o + 32 * p0, np.concatenate([up, skip])), aux=None, groups=g(p0),
                    out=("feat", slice(o, o + 32 * p0)))
    if name == "out12":  # pw_conv_coopvec_32to12, no activation
        blob, wo, bo = _codec_weights(12, 32, 28)
        (x,) = _codec_features([32 * p0], 38)
        return dict(shader="pw_conv_coopvec_32to12", push=[32, 12, w0, h0, wo, bo, 0, 32 * p0, 0], blob=blob,
                    feat=_arena(32 * p0 + 12 * p0, x), aux=None, groups=g(p0),
                    out=("feat", slice(32 * p0, 44 * p0)))
    if name == "pixelshuffle":  # 12 channels @ r0 -> RGB @ 2x, sigmoid; output in binding 2 (fp16)
        (x,) = _codec_features([12 * p0], 39)
        rgb = np.zeros(3 * 4 * p0, np.float16)
        return dict(shader="pixelshuffle_sigmoid", push=[w0, h0, 2 * w0, 2 * h0, 2, 0, 0],
                    blob=np.zeros(8, np.float16), feat=_arena(12 * p0, x), aux=rgb,
                    groups=((2 * w0 + 15) // 16, (2 * h0 + 15) // 16), out=("aux", slice(0, 12 * p0)))
    raise KeyError(name)


CODEC_CASES = ("enc_ic", "enc1", "enc2", "enc3", "dec3", "dec2", "dec1", "out12", "pixelshuffle")
# the transformer-stack passes (the hot path); the codec passes run through their own tests
HOT_CASES = ("attn_d256", "attn_d256_16tok", "router4", "expert_skip4", "moe_ffn_16exp", "dense_d256_h1024",
             "dense_d128_h512", "proj_up", "proj_down")
CASES = HOT_CASES + CODEC_CASES


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

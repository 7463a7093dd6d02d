"""The oracle restatement against the reference's own shader sources.

golden.npz holds the outputs of the unmodified reference GLSL (run on the host via
oracle/glsl_ref, see tests/golden/make_golden.py).  The restatement must match them
bit for bit; where the shader-source library itself is present, further random
shapes are compared directly.
"""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import CODEC_KINDS
from prism_inference_b200.abi import AttnParams, DenseParams, ExpertParams, ProjParams, RouterParams

GOLD = Path(__file__).resolve().parent / "golden"

import sys  # noqa: E402
sys.path.insert(0, str(GOLD))
from cases import CASES, build, input_digest, output_of  # noqa: E402


def run_oracle(o, c):
    sh, p, blob, feat, aux = c["shader"], c["push"], c["blob"], c["feat"], c["aux"]
    if sh == "split2_qkv_attn_d256":
        o.attn(AttnParams(*p), blob, feat)
    elif sh == "moe_router":
        o.router(RouterParams(*p), blob, feat, aux)
    elif sh == "moe_expert_skip":
        for q in p:
            o.expert(ExpertParams(*q), blob, feat, aux)
    elif sh == "moe_ffn_16exp":
        T, D, rw, rb, stride, w1, b1, w2, b2, inp, out = p
        a = np.zeros(T + 16, np.int32)
        o.router(RouterParams(T, D, 16, rw, rb, inp, 0, T), blob, feat, a)
        for e in range(16):
            eo = e * stride
            o.expert(ExpertParams(T, D, e, w1 + eo, b1 + eo, w2 + eo, b2 + eo, inp, out, 0), blob, feat, a)
    elif sh == "attention_windowed_d256":
        o.dense(DenseParams(*p), 1024, 256, blob, feat)
    elif sh == "attention_windowed":
        o.dense(DenseParams(*p), 512, 512, blob, feat)
    elif sh == "pw_project_128to256":
        o.proj_up(ProjParams(*p), blob, feat)
    elif sh == "pw_project_256to128":
        o.proj_down(ProjParams(*p), blob, feat)
    elif sh in CODEC_KINDS:  # the encoder / decoder passes around the stack
        o.codec_pass(sh, p, blob, feat, aux)
    else:
        raise KeyError(sh)


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLD / "golden.npz"), json.loads((GOLD / "golden_inputs.json").read_text())


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_golden(oracle, golden, name):
    gold, digests = golden
    c = build(name)
    assert input_digest(c) == digests[name], "seeded inputs drifted from the ones the golden outputs were made with"
    run_oracle(oracle, c)
    got = output_of(c)
    ref = gold[name]
    assert got.dtype == ref.dtype and got.shape == ref.shape
    if got.dtype == np.float16:
        diff = int((got.view(np.uint16) != ref.view(np.uint16)).sum())
    else:
        diff = int((got != ref).sum())
    assert diff == 0, f"{name}: {diff} elements differ from the reference shader output"


def _glsl_ref():
    from oracle import REF_LIB, GlslRef
    if not REF_LIB.exists():
        pytest.skip("oracle/_ref not built (needs the reference tree)")
    return GlslRef()


@pytest.mark.parametrize("w,h,seed", [(24, 20, 1), (8, 8, 2), (40, 9, 3)])
def test_oracle_matches_shader_source_random_shapes(oracle, w, h, seed):
    """Attention, router (N=4) and the expert dispatch loop on other frame shapes."""
    ref = _glsl_ref()
    from prism_inference_b200 import layout, synth
    T = w * h
    L = layout.build_stack(256, 1, n_experts=4, spatial_w=w, spatial_h=h)
    blob = synth.make_blob(L, seed=seed)
    b = L.blocks[0]
    feat = np.zeros(3 * T * 256, np.float16)
    feat[:T * 256] = synth.make_frames(L, 1, first=seed)[0].reshape(-1)
    f1, f2 = feat.copy(), feat.copy()
    pc = [T, 256, 8, 32, w, h, 8, b.qkv_w, b.qkv_b, b.out_w, b.out_b, 0, T * 256]
    ref.dispatch("split2_qkv_attn_d256", pc, blob, f1, None, ((w + 7) // 8) * ((h + 7) // 8))
    oracle.attn(AttnParams(*pc), blob, f2)
    a1, a2 = np.zeros(T + 8, np.int32), np.zeros(T + 8, np.int32)
    pr = [T, 256, 4, b.router_w, b.router_b, T * 256, 0, T]
    ref.dispatch("moe_router", pr, blob, f1, a1, (T + 255) // 256)
    oracle.router(RouterParams(*pr), blob, f2, a2)
    for e in range(4):
        eo = e * b.expert_stride
        pe = [T, 256, e, b.expert_w1 + eo, b.expert_b1 + eo, b.expert_w2 + eo, b.expert_b2 + eo, T * 256,
              2 * T * 256, 0]
        ref.dispatch("moe_expert_skip", pe, blob, f1, a1, (T + 255) // 256)
        oracle.expert(ExpertParams(*pe), blob, f2, a2)
    assert (a1 == a2).all()
    assert (f1.view(np.uint16) == f2.view(np.uint16)).all()


def test_oracle_stack_equals_pass_sequence(oracle):
    """oracle_stack_forward == the reference dispatch sequence of per-pass calls
    (prism_moe_bench.cpp:408-444: up, (attn, router, experts) x blocks, down)."""
    from prism_inference_b200 import layout, synth
    w, h = 16, 12
    T = w * h
    L = layout.build_stack(256, 2, n_experts=8, up_adapter=True, down_adapter=True, spatial_w=w, spatial_h=h)
    blob = synth.make_blob(L)
    x = synth.make_frames(L, 1)
    out, assign, stats = oracle.stack(L, blob, x)
    # pass sequence on an arena: [in128 | a256 | b256 | y256 | out128]
    f = np.zeros(T * (128 + 3 * 256 + 128), np.float16)
    f[:T * 128] = x.reshape(-1)
    A, B, Y, O = T * 128, T * 384, T * 640, T * 896
    oracle.proj_up(ProjParams(T, L.up_w, L.up_b, 0, A), blob, f)
    aux = np.zeros(T + 8, np.int32)
    ci, co = A, B
    for bi, b in enumerate(L.blocks):
        oracle.attn(AttnParams(T, 256, 8, 32, w, h, 8, b.qkv_w, b.qkv_b, b.out_w, b.out_b, ci, Y), blob, f)
        oracle.router(RouterParams(T, 256, 8, b.router_w, b.router_b, Y, 0, T), blob, f, aux)
        assert (aux[:T] == assign[bi]).all()
        for e in range(8):
            eo = e * b.expert_stride
            oracle.expert(ExpertParams(T, 256, e, b.expert_w1 + eo, b.expert_b1 + eo, b.expert_w2 + eo,
                                       b.expert_b2 + eo, Y, co, 0), blob, f, aux)
        ci, co = co, ci
    oracle.proj_down(ProjParams(T, L.down_w, L.down_b, ci, O), blob, f)
    assert (f[O:O + T * 128].view(np.uint16) == out.reshape(-1).view(np.uint16)).all()
    assert stats[0] == 2 * T and stats[2] == 0


def test_oracle_forced_routing_only_at_ties(oracle):
    """Forcing another routing is accepted only where the top-2 margin is below the threshold."""
    from prism_inference_b200 import layout, synth
    L = layout.build_stack(256, 1, n_experts=16, spatial_w=16, spatial_h=12)
    blob = synth.make_blob(L)
    x = synth.make_frames(L, 1)
    out, assign, stats = oracle.stack(L, blob, x)
    forced = (assign + 1) % 16
    _, a2, st2 = oracle.stack(L, blob, x, forced=forced, tie_thr=1e-3)
    assert st2[1] == st2[3]          # every tie token followed the forced choice
    assert st2[2] == assign.size - st2[3]  # every other difference counted as hard
    assert ((a2 == forced) == (np.arange(a2.size) >= 0)[None, :] & (a2 == forced)).all()


def test_gelu_rounding_points(oracle):
    for v in (-3.0, -0.5, 0.0, 0.1, 1.0, 2.5):
        x = float(np.float16(v))
        g = 0.5 * x * (1.0 + np.tanh(np.float32(0.7978846) * (np.float32(x) + np.float32(0.044715) * x * x * x)))
        assert abs(oracle.gelu_h(x) - float(np.float16(g))) <= 2 ** -10 * max(1.0, abs(g))



@pytest.mark.parametrize("w0,h0,seed", [(17, 9, 5), (40, 22, 6), (2, 1, 7)])
def test_codec_chain_matches_shader_source_random_shapes(oracle, w0, h0, seed):
    """The whole encoder / decoder chain of prism_moe_bench.cpp:386-471 (the stack itself
    left out: the bottleneck map goes straight to dec3) on other frame sizes, odd and
    degenerate ones included: the reference shader sources and the restatement give the same
    bits for every pass and the final RGB."""
    ref = _glsl_ref()
    rng = np.random.Generator(np.random.PCG64(seed))
    r = [(w0, h0)]
    for _ in range(3):
        r.append(((r[-1][0] + 1) // 2, (r[-1][1] + 1) // 2))
    p = [w * h for w, h in r]
    shapes = {"ic": (32, 81), "e1": (64, 288), "e2": (128, 576), "e3": (128, 1152), "d3": (128, 256),
              "d2": (64, 192), "d1": (32, 96), "o": (12, 32)}
    off, parts = {}, []
    n = 0
    for k, (rows, cols) in shapes.items():
        w = (rng.standard_normal(rows * cols, dtype=np.float32) / np.float32(np.sqrt(cols))).astype(np.float16)
        bias = (rng.standard_normal(rows, dtype=np.float32) * np.float32(0.1)).astype(np.float16)
        off[k] = (n, n + rows * cols)
        parts += [w, bias]
        n += rows * cols + rows
    blob = np.concatenate(parts)
    sizes = {"in": 9 * p[0], "e0": 32 * p[0], "e1": 64 * p[1], "e2": 128 * p[2], "e3": 128 * p[3],
             "d3": 128 * p[2], "d2": 64 * p[1], "d1": 32 * p[0], "o12": 12 * p[0]}
    fo, n = {}, 0
    for k, s in sizes.items():
        fo[k] = n
        n += s
    feat = np.zeros(n, np.float16)
    feat[:sizes["in"]] = rng.standard_normal(sizes["in"], dtype=np.float32).astype(np.float16)
    (w0_, h0_), (w1, h1), (w2, h2), (w3, h3) = r
    g = lambda m: (m + 255) // 256  # noqa: E731
    passes = [
        ("conv3x3_coopvec_9ch", [9, 32, w0_, h0_, *off["ic"], fo["in"], fo["e0"], 1], g(p[0])),
        ("strided_conv_coopvec_32ch", [32, 64, w0_, h0_, w1, h1, *off["e1"], fo["e0"], fo["e1"]], g(p[1])),
        ("strided_conv_split_64ch", [64, 128, w1, h1, w2, h2, *off["e2"], fo["e1"], fo["e2"]], g(p[2])),
        ("strided_conv_split_128ch", [128, 128, w2, h2, w3, h3, *off["e3"], fo["e2"], fo["e3"]], g(p[3])),
        ("dec3_fused", [w2, h2, w3, h3, 128, *off["d3"], fo["e3"], fo["e2"], fo["d3"]], g(p[2])),
        ("dec2_fused", [w1, h1, w2, h2, 128, 64, *off["d2"], fo["d3"], fo["e1"], fo["d2"]], g(p[1])),
        ("dec1_fused", [w0_, h0_, w1, h1, 64, 32, *off["d1"], fo["d2"], fo["e0"], fo["d1"]], g(p[0])),
        ("pw_conv_coopvec_32to12", [32, 12, w0_, h0_, *off["o"], fo["d1"], fo["o12"], 0], g(p[0])),
    ]
    f1, f2 = feat.copy(), feat.copy()
    for shader, push, groups in passes:
        ref.dispatch(shader, push, blob, f1, None, groups)
        oracle.codec_pass(shader, push, blob, f2)
        assert (f1.view(np.uint16) == f2.view(np.uint16)).all(), shader
    rgb1, rgb2 = np.zeros(12 * p[0], np.float16), np.zeros(12 * p[0], np.float16)
    ps = [w0_, h0_, 2 * w0_, 2 * h0_, 2, fo["o12"], 0]
    ref.dispatch("pixelshuffle_sigmoid", ps, blob, f1, rgb1, ((2 * w0_ + 15) // 16, (2 * h0_ + 15) // 16))
    oracle.codec_pass("pixelshuffle_sigmoid", ps, blob, f2, rgb2)
    assert (rgb1.view(np.uint16) == rgb2.view(np.uint16)).all()
    assert float(rgb2.astype(np.float32).min()) > 0.0

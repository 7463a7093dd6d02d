"""The encoder / decoder passes around the stack (prism_moe_bench.cpp:386-471) on the GPU,
through the C ABI's prism_codec_pass: against the reference shaders' own outputs (the golden
cases), pass by pass at the reference's 960x540 frame against the oracle, and as a whole chain."""
import sys
from pathlib import Path

import numpy as np
import pytest

from helpers import assert_close

GOLD = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLD))
from cases import CODEC_CASES, build, output_of  # noqa: E402

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16).copy()).cuda().view(torch.float16)


def _host(t):
    import torch
    torch.cuda.synchronize()
    return t.view(torch.int16).cpu().numpy().view(np.float16)


@pytest.mark.parametrize("name", CODEC_CASES)
def test_codec_pass_matches_reference_golden(prism_ctx, name):
    c = build(name)
    w, f = _dev(c["blob"]), _dev(c["feat"])
    rgb = _dev(c["aux"]) if c["aux"] is not None else None
    prism_ctx.codec_pass(c["shader"], c["push"], w, f, rgb)
    prism_ctx.status()
    c = dict(c)
    c["feat"] = _host(f)
    if rgb is not None:
        c["aux"] = _host(rgb)
    gold = np.load(GOLD / "golden.npz")[name]
    assert_close(output_of(c), gold, name)


def _pyramid(w0, h0):
    r = [(w0, h0)]
    for _ in range(3):
        r.append(((r[-1][0] + 1) // 2, (r[-1][1] + 1) // 2))
    return r


def _chain(w0, h0, seed):
    """Weights, a feature arena and the nine passes of prism_moe_bench.cpp:386-471 (the stack
    left out: the bottleneck map goes to dec3 directly) at a render size of w0 x h0."""
    rng = np.random.Generator(np.random.PCG64(seed))
    r = _pyramid(w0, h0)
    p = [w * h for w, h in r]
    shapes = {"ic": (32, 81), "e1": (64, 288), "e2": (128, 576), "e3": (128, 1152), "d3": (128, 256),
              "d2": (64, 192), "d1": (32, 96), "o": (12, 32)}
    off, parts, n = {}, [], 0
    for k, (rows, cols) in shapes.items():
        wt = (rng.standard_normal(rows * cols, dtype=np.float32) / np.float32(np.sqrt(cols))).astype(np.float16)
        b = (rng.standard_normal(rows, dtype=np.float32) * np.float32(0.1)).astype(np.float16)
        off[k] = (n + 3, n + 3 + rows * cols)  # odd element offsets: the blob is read at any alignment
        parts += [np.zeros(3, np.float16), wt, b]
        n += 3 + rows * cols + rows
    blob = np.concatenate(parts)
    sizes = {"in": 9 * p[0], "e0": 32 * p[0], "e1": 64 * p[1], "e2": 128 * p[2], "e3": 128 * p[3],
             "d3": 128 * p[2], "d2": 64 * p[1], "d1": 32 * p[0], "o12": 12 * p[0]}
    fo, n = {}, 1
    for k, s in sizes.items():
        fo[k] = n
        n += s
    feat = np.zeros(n, np.float16)
    feat[fo["in"]:fo["in"] + sizes["in"]] = rng.standard_normal(sizes["in"], dtype=np.float32).astype(np.float16)
    (w0_, h0_), (w1, h1), (w2, h2), (w3, h3) = r
    passes = [
        ("conv3x3_coopvec_9ch", [9, 32, w0_, h0_, *off["ic"], fo["in"], fo["e0"], 1], "e0"),
        ("strided_conv_coopvec_32ch", [32, 64, w0_, h0_, w1, h1, *off["e1"], fo["e0"], fo["e1"]], "e1"),
        ("strided_conv_split_64ch", [64, 128, w1, h1, w2, h2, *off["e2"], fo["e1"], fo["e2"]], "e2"),
        ("strided_conv_split_128ch", [128, 128, w2, h2, w3, h3, *off["e3"], fo["e2"], fo["e3"]], "e3"),
        ("dec3_fused", [w2, h2, w3, h3, 128, *off["d3"], fo["e3"], fo["e2"], fo["d3"]], "d3"),
        ("dec2_fused", [w1, h1, w2, h2, 128, 64, *off["d2"], fo["d3"], fo["e1"], fo["d2"]], "d2"),
        ("dec1_fused", [w0_, h0_, w1, h1, 64, 32, *off["d1"], fo["d2"], fo["e0"], fo["d1"]], "d1"),
        ("pw_conv_coopvec_32to12", [32, 12, w0_, h0_, *off["o"], fo["d1"], fo["o12"], 0], "o12"),
    ]
    ps = [w0_, h0_, 2 * w0_, 2 * h0_, 2, fo["o12"], 0]
    return blob, feat, passes, ps, fo, sizes, 12 * p[0]


def test_codec_passes_at_reference_frame_size(prism_ctx, oracle):
    """Each pass at the reference's sizes (960x540 render, 120x68 bottleneck), on the GPU's own
    inputs for that pass (the oracle is given the same arena), so each pass is checked alone."""
    blob, feat, passes, ps, fo, sizes, n_rgb = _chain(960, 540, 3)
    w, f = _dev(blob), _dev(feat)
    for shader, push, out in passes:
        cur = _host(f)
        prism_ctx.codec_pass(shader, push, w, f)
        got = _host(f)[fo[out]:fo[out] + sizes[out]]
        oracle.codec_pass(shader, push, blob, cur)
        assert_close(got, cur[fo[out]:fo[out] + sizes[out]], shader)
    prism_ctx.status()
    import torch
    rgb = torch.zeros(n_rgb, dtype=torch.float16, device="cuda")
    prism_ctx.codec_pass("pixelshuffle_sigmoid", ps, w, f, rgb)
    cur = _host(f)
    ref = np.zeros(n_rgb, np.float16)
    oracle.codec_pass("pixelshuffle_sigmoid", ps, blob, cur, ref)
    assert_close(_host(rgb), ref, "pixelshuffle_sigmoid")


@pytest.mark.parametrize("w0,h0,seed", [(40, 22, 6), (17, 9, 5), (2, 1, 7), (130, 70, 8)])
def test_codec_chain_matches_oracle(prism_ctx, oracle, w0, h0, seed):
    """The whole chain run independently on the GPU and by the oracle, odd and degenerate frame
    sizes included (partial 128-pixel tiles, maps of one pixel): the final RGB agrees."""
    import torch
    blob, feat, passes, ps, fo, sizes, n_rgb = _chain(w0, h0, seed)
    w, f = _dev(blob), _dev(feat)
    rgb = torch.zeros(n_rgb, dtype=torch.float16, device="cuda")
    for shader, push, _ in passes:
        prism_ctx.codec_pass(shader, push, w, f)
        oracle.codec_pass(shader, push, blob, feat)
    prism_ctx.codec_pass("pixelshuffle_sigmoid", ps, w, f, rgb)
    ref = np.zeros(n_rgb, np.float16)
    oracle.codec_pass("pixelshuffle_sigmoid", ps, blob, feat, ref)
    prism_ctx.status()
    assert_close(_host(rgb), ref, f"chain {w0}x{h0}")
    g = _host(f)
    for k in ("e3", "d1"):
        assert_close(g[fo[k]:fo[k] + sizes[k]], feat[fo[k]:fo[k] + sizes[k]], f"chain {w0}x{h0} {k}")


def test_codec_pass_argument_errors(prism_ctx):
    import torch
    from prism_inference_b200.abi import PrismError
    w = torch.zeros(40000, dtype=torch.float16, device="cuda")
    f = torch.zeros(1000, dtype=torch.float16, device="cuda")
    with pytest.raises(PrismError, match="ARG"):
        prism_ctx.codec_pass("conv3x3_coopvec_9ch", [9, 32, 4, 4, 0, 2592, 0, 144], w, f)  # 8 of 9 constants
    with pytest.raises(PrismError, match="RANGE"):  # 32 x 16 output values do not fit
        prism_ctx.codec_pass("conv3x3_coopvec_9ch", [9, 32, 4, 4, 0, 2592, 0, 600, 1], w, f)
    with pytest.raises(PrismError, match="ARG"):  # output overlaps the input
        prism_ctx.codec_pass("conv3x3_coopvec_9ch", [9, 32, 4, 4, 0, 2592, 0, 100, 1], w, f)

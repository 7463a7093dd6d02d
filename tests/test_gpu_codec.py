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


def _chain(w0, h0, seed, feat_pad=1):
    """Weights, feature arena and dispatch list of one frame's encoder / decoder path at a
    render size of w0 x h0, with weights at odd element offsets and the maps at odd offsets
    (feat_pad=1: every pass gathers with plain loads) or 16-byte aligned ones (feat_pad=0: the
    passes whose map rows are 16-byte multiples stage their input rows by TMA)."""
    from prism_inference_b200 import codec
    fc = codec.frame_chain(w0, h0, weight_pad=3, feat_pad=feat_pad)
    blob, feat = codec.synthetic(fc, seed)
    return blob, feat, fc.passes, fc.pixelshuffle, fc.feat_off, fc.feat_size, fc.rgb_elems


@pytest.mark.parametrize("feat_pad", [1, 0], ids=["plain-gather", "tma-staged"])
def test_codec_passes_at_reference_frame_size(prism_ctx, oracle, feat_pad):
    """Each pass at the reference's sizes (960x540 render, 120x68 bottleneck), on the GPU's own
    inputs for that pass (the oracle is given the same arena), so each pass is checked alone."""
    blob, feat, passes, ps, fo, sizes, n_rgb = _chain(960, 540, 3, feat_pad)
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


@pytest.mark.parametrize("w0,h0,seed,feat_pad", [(40, 22, 6, 1), (17, 9, 5, 1), (2, 1, 7, 1), (130, 70, 8, 1),
                                                 (192, 100, 9, 0), (64, 3, 10, 0), (136, 72, 11, 0)])
def test_codec_chain_matches_oracle(prism_ctx, oracle, w0, h0, seed, feat_pad):
    """The whole chain run independently on the GPU and by the oracle, odd and degenerate frame
    sizes included (partial 128-pixel tiles, maps of one pixel): the final RGB agrees.  The
    aligned cases run the TMA-staged passes on rows with a partial last tile (192 = 128 + 64),
    maps narrower than a tile and one row high, and a mix (136 wide: 68-pixel rows fall back)."""
    import torch
    blob, feat, passes, ps, fo, sizes, n_rgb = _chain(w0, h0, seed, feat_pad)
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

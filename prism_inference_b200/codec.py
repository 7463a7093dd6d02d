"""The encoder / decoder around the transformer stack: buffer layout and dispatch list of one
frame, as prism_moe_bench.cpp:386-471 records them (the stack itself left out: the bottleneck
map of the encoder goes to dec3).

A render frame of w0 x h0 pixels, 9 input channels (CHW fp16), goes through
    conv3x3_coopvec_9ch (9 -> 32) -> strided_conv_coopvec_32ch (32 -> 64, /2)
    -> strided_conv_split_64ch (64 -> 128, /2) -> strided_conv_split_128ch (128 -> 128, /2)
    -> dec3_fused (2x up + skip e2 -> 128) -> dec2_fused (-> 64, skip e1) -> dec1_fused (-> 32, skip e0)
    -> pw_conv_coopvec_32to12 -> pixelshuffle_sigmoid (12 channels -> RGB at 2x)
with each level's size rounded up ((w + 1) / 2, as 135 -> 68 in the reference).  Every pass is one
prism_codec_pass call (Prism.codec_pass) with these push constants.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Tuple

import numpy as np

# (rows, cols) of each pass's weight matrix, row-major [out][in], in the blob order below
WEIGHTS = {"ic": (32, 81), "e1": (64, 288), "e2": (128, 576), "e3": (128, 1152), "d3": (128, 256),
           "d2": (64, 192), "d1": (32, 96), "o": (12, 32)}


@dataclass
class FrameChain:
    render: Tuple[int, int]
    levels: List[Tuple[int, int]]              # (w, h) of the render size and its three halvings
    weight_off: Dict[str, Tuple[int, int]]     # pass -> (weight, bias) element offsets in the blob
    blob_elems: int
    feat_off: Dict[str, int]                   # map -> element offset in the feature arena
    feat_size: Dict[str, int]
    feat_elems: int
    passes: List[Tuple[str, List[int], str]] = field(default_factory=list)  # (shader, push, output map)
    pixelshuffle: List[int] = field(default_factory=list)
    rgb_elems: int = 0

    def pass_bytes_flops(self, shader: str) -> Tuple[int, float]:
        """Algorithmic DRAM bytes (each input map read once, the output written once, the weights
        read once, fp16) and FLOPs (2 per MAC) of one pass."""
        (w0, h0), (w1, h1), (w2, h2), (w3, h3) = self.levels
        p0, p1, p2, p3 = w0 * h0, w1 * h1, w2 * h2, w3 * h3
        io = {"conv3x3_coopvec_9ch": ((9 * p0, 32 * p0), "ic", p0),
              "strided_conv_coopvec_32ch": ((32 * p0, 64 * p1), "e1", p1),
              "strided_conv_split_64ch": ((64 * p1, 128 * p2), "e2", p2),
              "strided_conv_split_128ch": ((128 * p2, 128 * p3), "e3", p3),
              "dec3_fused": ((128 * p3 + 128 * p2, 128 * p2), "d3", p2),
              "dec2_fused": ((128 * p2 + 64 * p1, 64 * p1), "d2", p1),
              "dec1_fused": ((64 * p1 + 32 * p0, 32 * p0), "d1", p0),
              "pw_conv_coopvec_32to12": ((32 * p0, 12 * p0), "o", p0)}
        if shader == "pixelshuffle_sigmoid":
            return 2 * (12 * p0 + 12 * p0), 0.0
        (rd, wr), k, px = io[shader]
        rows, cols = WEIGHTS[k]
        return 2 * (rd + wr + rows * cols + rows), 2.0 * rows * cols * px


def frame_chain(w0: int, h0: int, weight_pad: int = 0, feat_pad: int = 0) -> FrameChain:
    """Layout of one frame's path at render size w0 x h0.  weight_pad / feat_pad put that many
    elements before every weight matrix / the arena (odd values exercise unaligned offsets)."""
    levels = [(w0, h0)]
    for _ in range(3):
        levels.append(((levels[-1][0] + 1) // 2, (levels[-1][1] + 1) // 2))
    p = [w * h for w, h in levels]
    off, n = {}, 0
    for k, (rows, cols) in WEIGHTS.items():
        n += weight_pad
        off[k] = (n, n + rows * cols)
        n += rows * cols + rows
    sizes = {"in": 9 * p[0], "e0": 32 * p[0], "e1": 64 * p[1], "e2": 128 * p[2], "e3": 128 * p[3],
             "d3": 128 * p[2], "d2": 64 * p[1], "d1": 32 * p[0], "o12": 12 * p[0]}
    fo, m = {}, feat_pad
    for k, s in sizes.items():
        fo[k] = m
        m += s
    (w0_, h0_), (w1, h1), (w2, h2), (w3, h3) = levels
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
    return FrameChain(render=(w0, h0), levels=levels, weight_off=off, blob_elems=n, feat_off=fo, feat_size=sizes,
                      feat_elems=m, passes=passes, pixelshuffle=[w0_, h0_, 2 * w0_, 2 * h0_, 2, fo["o12"], 0],
                      rgb_elems=12 * p[0])


def synthetic(fc: FrameChain, seed: int) -> Tuple[np.ndarray, np.ndarray]:
    """Seeded weights ~ N(0, 1/fan_in), biases ~ N(0, 0.1) and a frame ~ N(0, 1) (the reference
    ships no trained encoder / decoder); returns (blob, feature arena)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    blob = np.zeros(fc.blob_elems, np.float16)
    for k, (rows, cols) in WEIGHTS.items():
        wo, bo = fc.weight_off[k]
        blob[wo:wo + rows * cols] = (rng.standard_normal(rows * cols, dtype=np.float32)
                                     / np.float32(np.sqrt(cols))).astype(np.float16)
        blob[bo:bo + rows] = (rng.standard_normal(rows, dtype=np.float32) * np.float32(0.1)).astype(np.float16)
    feat = np.zeros(fc.feat_elems, np.float16)
    o, n = fc.feat_off["in"], fc.feat_size["in"]
    feat[o:o + n] = rng.standard_normal(n, dtype=np.float32).astype(np.float16)
    return blob, feat

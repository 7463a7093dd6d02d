"""Seeded synthetic weights and frames for the benchmark configurations.

The reference ships no trained model and no frames (README.md:117-125) and its
benches never upload data (prism_moe_bench.cpp:141-152), so every run here uses
seeded synthetic data with the shapes and distributions BASELINE.json names:
weights fp16 ~ N(0, 0.02), input frames fp16 HWC ~ N(0, 1).

Generator: numpy PCG64.  Weights use seed `seed`; frame f of an input batch uses
seed 0x5EED + f, so frame f is identical whatever the batch size.
"""
from __future__ import annotations

import numpy as np

from .layout import StackLayout

FRAME_SEED = 0x5EED
WEIGHT_SEED = 0x5EED0000


def make_blob(layout: StackLayout, seed: int = WEIGHT_SEED, std: float = 0.02,
              router_skew: int = 0, skew_bias=0.0) -> np.ndarray:
    """Flat fp16 blob (as np.float16) for `layout`.  router_skew > 0 adds skew_bias
    (a number, or one number per MoE block) to the router bias of experts
    0..router_skew-1 in every MoE block (the load-imbalance stress configuration)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    blob = np.empty(layout.total, dtype=np.float16)
    chunk = 1 << 24
    for s in range(0, layout.total, chunk):
        n = min(chunk, layout.total - s)
        blob[s:s + n] = (rng.standard_normal(n, dtype=np.float32) * np.float32(std)).astype(np.float16)
    if router_skew > 0:
        moe = [b for b in layout.blocks if b.kind == "moe"]
        for i, b in enumerate(moe):
            sb = skew_bias[i % len(skew_bias)] if isinstance(skew_bias, (tuple, list)) else skew_bias
            rb = b.router_b
            blob[rb:rb + router_skew] = (blob[rb:rb + router_skew].astype(np.float32)
                                         + np.float32(sb)).astype(np.float16)
    return blob


def make_frames(layout: StackLayout, frames: int, first: int = 0, std: float = 1.0) -> np.ndarray:
    """[frames][T][in_dim] fp16 frames ~ N(0, std^2); frame i uses seed 0x5EED + first + i."""
    T, C = layout.tokens, layout.in_dim
    out = np.empty((frames, T, C), dtype=np.float16)
    for i in range(frames):
        rng = np.random.Generator(np.random.PCG64(FRAME_SEED + first + i))
        out[i] = (rng.standard_normal(T * C, dtype=np.float32) * np.float32(std)).astype(np.float16).reshape(T, C)
    return out

"""The five benchmark configurations of BASELINE.json, as stack layouts.

Where BASELINE.json and the reference shaders disagree, both are available:
  * dense FFN width: BASELINE.json states 128->128->128 (dim 128) and 256->256->256
    (dim 256); the reference shaders use 512 (attention_windowed.comp.glsl:151-170)
    and 1024 in four fp16-accumulated 256-wide chunks
    (attention_windowed_d256.comp.glsl:143-177).  `reference_widths=True` selects
    the shader widths.
  * LayerNorm: BASELINE.json says "pre-norm ... LN/activation as in reference
    shaders"; no reference shader normalises, so no block has a LayerNorm.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Tuple

from .layout import StackLayout, build_stack

# Router bias added to experts 0..3 of each block in config 5 so that half of the
# tokens of every block route there.  Calibrated per block (bisection on the CPU
# oracle, one frame, the seeded synthetic weights), because the logit spread grows
# with depth.
SKEW_BIAS = (0.0777, 0.0483, 0.0288, 0.0324, 0.0414, 0.0504, 0.0521, 0.0762, 0.0524, 0.0083, 0.0784,
             0.0732, 0.0614, 0.0054, 0.0919, 0.1032, 0.0414, 0.0485, 0.1208, 0.0787, 0.1102, 0.0976)


@dataclass
class Config:
    key: str
    layout: StackLayout
    frames: Tuple[int, ...]
    router_skew: int = 0
    skew_bias: float = 0.0
    description: str = ""


def get(key: str, reference_widths: bool = False, n_blocks: int | None = None) -> Config:
    """key: 'moe16x1' (config 1), 'dense128x4' (2), 'dense256x12' (3),
    'moe64x16' (4, the headline), 'moe32x22skew' (5).  n_blocks overrides the depth
    (used only by small tests)."""
    if key == "moe16x1":
        L = build_stack(256, n_blocks or 1, n_experts=16)
        return Config(key, L, (1,), description="1 MoE block, dim 256, 8x32 heads, 16 experts")
    if key == "dense128x4":
        h = 512 if reference_widths else 128
        L = build_stack(128, n_blocks or 4, n_heads=4, ffn_hidden=h, ffn_chunk=h)
        return Config(key, L, (1, 16), description=f"dense d128 x4, 4x32 heads, FFN {h}")
    if key == "dense256x12":
        h = 1024 if reference_widths else 256
        L = build_stack(256, n_blocks or 12, ffn_hidden=h, ffn_chunk=256, up_adapter=True,
                        down_adapter=True)
        return Config(key, L, (1, 16, 64), description=f"dense d256 x12 + adapters, FFN {h}")
    if key == "moe64x16":
        L = build_stack(256, n_blocks or 16, n_experts=64, up_adapter=True, down_adapter=True)
        return Config(key, L, (1, 64), description="MoE 64 experts x16 blocks + adapters")
    if key == "moe32x22skew":
        L = build_stack(256, n_blocks or 22, n_experts=32, up_adapter=True, down_adapter=True)
        return Config(key, L, (8, 32, 128, 512), router_skew=4, skew_bias=SKEW_BIAS,
                      description="MoE 32 experts x22 blocks, router skewed to 4 experts")
    raise KeyError(key)


ALL = ("moe16x1", "dense128x4", "dense256x12", "moe64x16", "moe32x22skew")


def flops_per_frame(L: StackLayout, valid_only: bool = True) -> float:
    """Algorithmic FLOPs (2 per MAC) per frame, valid tokens only: QKV, attention
    (QK^T and PV over 64 keys), out-projection, router, one expert FFN (or the dense
    FFN) per token, plus adapters."""
    T = L.tokens
    D = L.dim
    f = 0.0
    if L.up_w >= 0:
        f += 2.0 * T * 128 * 256
    if L.down_w >= 0:
        f += 2.0 * T * 256 * 128
    for b in L.blocks:
        per = 2.0 * (3 * D * D + D * D) + 2.0 * 2 * 64 * D
        if b.kind == "moe":
            per += 2.0 * b.n_experts * D + 2.0 * 2 * D * D
        else:
            per += 2.0 * 2 * D * b.ffn_hidden
        f += per * T
    return f

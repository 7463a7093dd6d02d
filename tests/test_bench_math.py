"""bench.py's roofline arithmetic, on CPU: the per-kernel FLOP attribution adds up to the
layout's algorithmic FLOPs per frame for every configuration (each kernel kind counted once
per launch it makes per frame), and the batch-1 byte count of a frame that touches every
expert is the whole weight blob plus the frame in and out."""
import sys
from pathlib import Path

import pytest

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402
from prism_inference_b200 import configs  # noqa: E402


def _mixed_layout():
    """Dense and MoE blocks at dim 256 in one stack (no configuration mixes them, the FLOP
    attribution must still add up)."""
    from prism_inference_b200 import layout
    L = layout.build_stack(256, 3, n_experts=32, up_adapter=True, down_adapter=True)
    D = layout.build_stack(256, 2, ffn_hidden=1024, ffn_chunk=256)
    L.blocks = [L.blocks[0], D.blocks[0], L.blocks[1], D.blocks[1], L.blocks[2]]
    return L


@pytest.mark.parametrize("key", configs.ALL + ("mixed",))
def test_kernel_flops_add_up_to_the_layout(key):
    L = _mixed_layout() if key == "mixed" else configs.get(key).layout
    moe = sum(b.kind == "moe" for b in L.blocks)
    dense = len(L.blocks) - moe
    launches = {"attn": len(L.blocks), "router": moe, "expert": moe, "dense_ffn": dense,
                "proj_up": int(L.up_w >= 0), "proj_down": int(L.down_w >= 0)}
    total = sum(bench.kind_flops_per_frame(L, k) * n for k, n in launches.items())
    assert total == pytest.approx(configs.flops_per_frame(L), rel=1e-12)


def test_headline_flops_and_batch1_bytes():
    L = configs.get("moe64x16").layout
    assert configs.flops_per_frame(L) == pytest.approx(116.58e9, rel=1e-3)  # 115.51 + 1.07 GFLOP
    every = bench.batch1_bytes(L, [64] * L.n_moe_blocks)
    assert every == 2 * (L.total + L.tokens * (L.in_dim + L.out_dim))
    assert bench.batch1_bytes(L, [32] * L.n_moe_blocks) < every

"""Blob layout, configuration sizes and FLOP counts."""
import json

import numpy as np

from prism_inference_b200 import configs, layout, synth


def test_param_counts_match_readme():
    # README.md:11-15 (139M / 98M / 37M / 9M) and prism_moe_bench.cpp:170 stride
    assert configs.get("moe64x16").layout.total - 2 * (256 * 128) - 256 - 128 == 139_215_872
    assert layout.build_stack(256, 22, n_experts=32).total == 98_605_760
    assert layout.build_stack(256, 16, n_experts=16).total == 37_961_984
    assert layout.build_stack(256, 12, ffn_hidden=1024, ffn_chunk=256).total == 9_464_832
    L = configs.get("moe64x16").layout
    assert L.blocks[0].expert_stride == 131_584


def test_flops_per_frame():
    L = configs.get("moe64x16").layout
    f = configs.flops_per_frame(L)
    assert abs(f - (115.51e9 + 1.07e9)) / f < 1e-3


def test_export_weights_json_schema_roundtrip():
    L = layout.build_stack(256, 2, n_experts=4, up_adapter=True, down_adapter=True)
    js = json.loads(L.to_json())
    assert js["total_fp16_values"] == L.total and js["total_bytes"] == 2 * L.total
    for l in js["layers"]:
        assert set(l) == {"name", "type", "weight_count", "bias_count", "total_fp32", "weight_offset_fp16",
                          "bias_offset_fp16"}
        assert l["bias_offset_fp16"] == l["weight_offset_fp16"] + l["weight_count"]
    L2 = layout.stack_from_json(js, 256, 8, 4, 2)
    for a, b in zip(L.blocks, L2.blocks):
        assert a == b
    assert (L2.up_w, L2.down_w, L2.in_dim, L2.out_dim) == (L.up_w, L.down_w, 128, 128)


def test_synthetic_data_is_seeded_per_frame():
    L = layout.build_stack(256, 1, n_experts=4, spatial_w=16, spatial_h=8)
    a = synth.make_frames(L, 3)
    b = synth.make_frames(L, 1, first=2)
    assert (a[2].view(np.uint16) == b[0].view(np.uint16)).all()
    assert abs(float(a.astype(np.float32).std()) - 1.0) < 0.05
    w = synth.make_blob(L)
    assert abs(float(w.astype(np.float32).std()) - 0.02) < 0.002

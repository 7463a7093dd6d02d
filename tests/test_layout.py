"""Blob layout, configuration sizes and FLOP counts."""
import json

import numpy as np
import pytest

from helpers import checkpoint_of
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


def test_pack_write_read_weights(tmp_path):
    """Named (weight, bias) arrays -> flat blob at the layout's offsets -> .weights/.json pair
    -> the same blob and a table that rebuilds the same layout."""
    L = layout.build_stack(256, 2, n_experts=3, up_adapter=True, down_adapter=True)
    rng = np.random.default_rng(7)
    shapes = {"proj_up": (256, 128), "proj_down": (128, 256)}
    for i in range(2):
        shapes[f"blk{i}.qkv"] = (768, 256)
        shapes[f"blk{i}.out"] = (256, 256)
        shapes[f"blk{i}.router"] = (3, 256)
        for e in range(3):
            shapes[f"blk{i}.expert{e}.w1"] = (256, 256)
            shapes[f"blk{i}.expert{e}.w2"] = (256, 256)
    tensors = {n: (rng.standard_normal(s).astype(np.float32), rng.standard_normal(s[0]).astype(np.float32))
               for n, s in shapes.items()}
    blob = layout.pack_weights(L, tensors)
    b = L.blocks[1]
    w, bias = tensors["blk1.qkv"]
    assert np.array_equal(blob[b.qkv_w:b.qkv_w + w.size], w.astype(np.float16).reshape(-1))
    assert np.array_equal(blob[b.qkv_b:b.qkv_b + 768], bias.astype(np.float16))
    e2 = b.expert_w1 + 2 * b.expert_stride  # expert 2 of block 1 through the stride
    assert np.array_equal(blob[e2:e2 + 65536], tensors["blk1.expert2.w1"][0].astype(np.float16).reshape(-1))
    path = str(tmp_path / "stack.weights")
    js_path = layout.write_weights(path, L, blob)
    blob2, table = layout.read_weights(path)
    assert js_path.endswith("stack.json") and np.array_equal(blob, blob2)
    L2 = layout.stack_from_json(table, 256, 8, 3, 2)
    assert L2.blocks == L.blocks
    bad = dict(tensors)
    bad["blk0.out"] = (np.zeros((256, 255), np.float32), tensors["blk0.out"][1])
    with pytest.raises(ValueError):
        layout.pack_weights(L, bad)
    with pytest.raises(KeyError):
        layout.pack_weights(L, {k: v for k, v in tensors.items() if k != "proj_up"})


def test_synthetic_data_is_seeded_per_frame():
    L = layout.build_stack(256, 1, n_experts=4, spatial_w=16, spatial_h=8)
    a = synth.make_frames(L, 3)
    b = synth.make_frames(L, 1, first=2)
    assert (a[2].view(np.uint16) == b[0].view(np.uint16)).all()
    assert abs(float(a.astype(np.float32).std()) - 1.0) < 0.05
    w = synth.make_blob(L)
    assert abs(float(w.astype(np.float32).std()) - 0.02) < 0.002


@pytest.mark.parametrize("key,split", [("moe16x1", False), ("dense256x12", True), ("dense128x4", False)])
def test_export_checkpoint_roundtrip(tmp_path, key, split):
    """A checkpoint named after export.py's convention (q, k, v as one tensor or three) exports
    to the .weights / .json pair of the layout, bit-identical to the packed blob."""
    from prism_inference_b200 import export
    cfg = configs.get(key, n_blocks=2)
    L = cfg.layout
    blob = synth.make_blob(L, seed=11)
    ck = checkpoint_of(L, blob, split_qkv=split)
    np.savez(tmp_path / "ck.npz", **ck)
    out = str(tmp_path / "m.weights")
    assert export.main([str(tmp_path / "ck.npz"), out, "--config", key, "--n-blocks", "2"]) == 0
    blob2, table = layout.read_weights(out)
    assert blob2.view(np.uint16).tobytes() == blob.view(np.uint16).tobytes()
    assert table["layers"] == L.layers


def test_export_custom_names_and_missing_tensors(tmp_path):
    from prism_inference_b200 import export
    L = layout.build_stack(256, 1, n_experts=2)
    blob = synth.make_blob(L, seed=3)
    ck = checkpoint_of(L, blob)
    ck["encoder.layer0.mha.out_proj.weight"] = ck.pop("blocks.0.attn.proj.weight")
    ck["encoder.layer0.mha.out_proj.bias"] = ck.pop("blocks.0.attn.proj.bias")
    with pytest.raises(KeyError, match="blocks.0.attn.proj.weight"):
        export.export(L, ck, str(tmp_path / "a.weights"))
    export.export(L, ck, str(tmp_path / "a.weights"), names={"blk0.out": "encoder.layer0.mha.out_proj"})
    assert layout.read_weights(str(tmp_path / "a.weights"))[0].view(np.uint16).tobytes() == blob.view(np.uint16).tobytes()
    del ck["blocks.0.moe.router.bias"]
    with pytest.raises(KeyError, match="router.bias"):
        export.export(L, ck, str(tmp_path / "b.weights"), names={"blk0.out": "encoder.layer0.mha.out_proj"})


def test_reference_frame_layout_allows_the_staged_codec_passes():
    """The 960x540 frame path laid out with an aligned arena (as bench.py --codec does) meets what
    prism_codec_pass needs for its TMA-staged form (conv3x3_9ch, dec2, dec1, pointwise): every map
    starts 16-byte aligned and every level's row is a multiple of 8 pixels (16 bytes of fp16), and
    each decoder's output is at most twice its deeper map's width."""
    from prism_inference_b200 import codec
    fc = codec.frame_chain(960, 540)
    for name, off in fc.feat_off.items():
        assert (off * 2) % 16 == 0, f"map {name} at element {off} is not 16-byte aligned"
    for w, h in fc.levels:
        assert (w * 2) % 16 == 0, f"row of {w} pixels is not a multiple of 16 bytes"
    for shader, push, _ in fc.passes:
        if shader.startswith("dec"):
            out_w, in_w = push[0], push[2]
            assert out_w <= 2 * in_w, shader
    # an odd arena offset (the other tests' unaligned layout) takes the plain form instead
    odd = codec.frame_chain(960, 540, feat_pad=1)
    assert any((off * 2) % 16 for off in odd.feat_off.values())

"""Flat fp16 weight-blob layout for the transformer stack.

The reference addresses every weight by an fp16-ELEMENT offset into one flat blob
(push constants, e.g. split2_qkv_attn_d256.comp.glsl:36 multiplies by 2 for bytes).
Offsets come from bump allocators in the bench drivers: prism_moe_bench.cpp:164-172
(MoE block: qkv, out, router, experts with stride 131,584) and
prism_scaling_bench.cpp:538-548 (one set of dense weights per block).  The on-disk
format is export_weights.py:95-121: a raw fp16 file plus a JSON table
{"total_fp16_values", "total_bytes", "layers": [{"name", "type", "weight_count",
"bias_count", "total_fp32", "weight_offset_fp16", "bias_offset_fp16"}]}.

This module lays out a whole stack (optional 128->256 adapter, per-block weights,
optional 256->128 adapter) with the same bump allocation and emits both the
prism_stack_desc fields and that JSON table.
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from typing import List, Optional


@dataclass
class BlockLayout:
    kind: str  # "moe" | "dense"
    qkv_w: int = -1
    qkv_b: int = -1
    out_w: int = -1
    out_b: int = -1
    n_experts: int = 0
    router_w: int = -1
    router_b: int = -1
    expert_w1: int = -1
    expert_b1: int = -1
    expert_w2: int = -1
    expert_b2: int = -1
    expert_stride: int = 0
    ffn_hidden: int = 0
    ffn_chunk: int = 0
    ffn_w1: int = -1
    ffn_b1: int = -1
    ffn_w2: int = -1
    ffn_b2: int = -1


@dataclass
class StackLayout:
    dim: int
    n_heads: int
    head_dim: int = 32
    spatial_w: int = 120
    spatial_h: int = 68
    window_size: int = 8
    in_dim: int = 0
    out_dim: int = 0
    up_w: int = -1
    up_b: int = -1
    down_w: int = -1
    down_b: int = -1
    blocks: List[BlockLayout] = field(default_factory=list)
    total: int = 0
    layers: list = field(default_factory=list)

    @property
    def tokens(self) -> int:
        return self.spatial_w * self.spatial_h

    @property
    def n_moe_blocks(self) -> int:
        return sum(1 for b in self.blocks if b.kind == "moe")

    def _alloc(self, name: str, kind: str, w: int, b: int):
        wo = self.total
        self.total += w
        bo = self.total
        self.total += b
        self.layers.append(dict(name=name, type=kind, weight_count=w, bias_count=b,
                                total_fp32=w + b, weight_offset_fp16=wo, bias_offset_fp16=bo))
        return wo, bo

    def to_json(self) -> str:
        return json.dumps(dict(total_fp16_values=self.total, total_bytes=2 * self.total,
                               layers=self.layers), indent=2)

    def param_count(self) -> int:
        return self.total


def build_stack(dim: int, n_blocks: int, *, n_heads: Optional[int] = None, n_experts: int = 0,
                ffn_hidden: int = 0, ffn_chunk: int = 0, up_adapter: bool = False,
                down_adapter: bool = False, spatial_w: int = 120, spatial_h: int = 68,
                window_size: int = 8) -> StackLayout:
    """Bump-allocate a stack.  n_experts > 0 -> MoE blocks (router + experts),
    else dense blocks with FFN width ffn_hidden accumulated in ffn_chunk pieces."""
    if n_heads is None:
        n_heads = dim // 32
    L = StackLayout(dim=dim, n_heads=n_heads, spatial_w=spatial_w, spatial_h=spatial_h,
                    window_size=window_size)
    D = dim
    L.in_dim = 128 if up_adapter else D
    L.out_dim = 128 if down_adapter else D
    if up_adapter:
        L.up_w, L.up_b = L._alloc("proj_up", "linear", 256 * 128, 256)
    for i in range(n_blocks):
        if n_experts > 0:
            b = BlockLayout(kind="moe", n_experts=n_experts)
        else:
            b = BlockLayout(kind="dense", ffn_hidden=ffn_hidden, ffn_chunk=ffn_chunk or ffn_hidden)
        b.qkv_w, b.qkv_b = L._alloc(f"blk{i}.qkv", "linear", 3 * D * D, 3 * D)
        b.out_w, b.out_b = L._alloc(f"blk{i}.out", "linear", D * D, D)
        if n_experts > 0:
            b.router_w, b.router_b = L._alloc(f"blk{i}.router", "linear", n_experts * D, n_experts)
            b.expert_stride = D * D + D + D * D + D  # 131,584 at D=256 (prism_moe_bench.cpp:170)
            for e in range(n_experts):
                w1, b1 = L._alloc(f"blk{i}.expert{e}.w1", "linear", D * D, D)
                w2, b2 = L._alloc(f"blk{i}.expert{e}.w2", "linear", D * D, D)
                if e == 0:
                    b.expert_w1, b.expert_b1, b.expert_w2, b.expert_b2 = w1, b1, w2, b2
        else:
            h = ffn_hidden
            b.ffn_w1, b.ffn_b1 = L._alloc(f"blk{i}.ffn_w1", "linear", h * D, h)
            b.ffn_w2, b.ffn_b2 = L._alloc(f"blk{i}.ffn_w2", "linear", D * h, D)
        L.blocks.append(b)
    if down_adapter:
        L.down_w, L.down_b = L._alloc("proj_down", "linear", 128 * 256, 128)
    return L


def stack_from_json(js: dict, dim: int, n_heads: int, n_experts: int, n_blocks: int,
                    ffn_hidden: int = 0, ffn_chunk: int = 0, spatial_w: int = 120,
                    spatial_h: int = 68, window_size: int = 8) -> StackLayout:
    """Rebuild a StackLayout from an export_weights.py-style JSON table whose layer
    names follow build_stack's naming (proj_up, blk{i}.qkv, blk{i}.expert{e}.w1, ...)."""
    by = {l["name"]: l for l in js["layers"]}
    L = StackLayout(dim=dim, n_heads=n_heads, spatial_w=spatial_w, spatial_h=spatial_h,
                    window_size=window_size)
    L.total = js["total_fp16_values"]
    L.layers = js["layers"]
    up = by.get("proj_up")
    dn = by.get("proj_down")
    L.in_dim = 128 if up else dim
    L.out_dim = 128 if dn else dim
    if up:
        L.up_w, L.up_b = up["weight_offset_fp16"], up["bias_offset_fp16"]
    if dn:
        L.down_w, L.down_b = dn["weight_offset_fp16"], dn["bias_offset_fp16"]
    for i in range(n_blocks):
        q, o = by[f"blk{i}.qkv"], by[f"blk{i}.out"]
        if n_experts > 0:
            b = BlockLayout(kind="moe", n_experts=n_experts)
            r = by[f"blk{i}.router"]
            b.router_w, b.router_b = r["weight_offset_fp16"], r["bias_offset_fp16"]
            e0w1, e0w2 = by[f"blk{i}.expert0.w1"], by[f"blk{i}.expert0.w2"]
            b.expert_w1, b.expert_b1 = e0w1["weight_offset_fp16"], e0w1["bias_offset_fp16"]
            b.expert_w2, b.expert_b2 = e0w2["weight_offset_fp16"], e0w2["bias_offset_fp16"]
            if n_experts > 1:
                b.expert_stride = by[f"blk{i}.expert1.w1"]["weight_offset_fp16"] - b.expert_w1
        else:
            b = BlockLayout(kind="dense", ffn_hidden=ffn_hidden, ffn_chunk=ffn_chunk or ffn_hidden)
            f1, f2 = by[f"blk{i}.ffn_w1"], by[f"blk{i}.ffn_w2"]
            b.ffn_w1, b.ffn_b1 = f1["weight_offset_fp16"], f1["bias_offset_fp16"]
            b.ffn_w2, b.ffn_b2 = f2["weight_offset_fp16"], f2["bias_offset_fp16"]
        b.qkv_w, b.qkv_b = q["weight_offset_fp16"], q["bias_offset_fp16"]
        b.out_w, b.out_b = o["weight_offset_fp16"], o["bias_offset_fp16"]
        L.blocks.append(b)
    return L


# ---- weight files ------------------------------------------------------------------------
# Shapes of the named layers, in the reference's row-major [out][in] convention (each output
# row contiguous, as the shaders index W[row * dim + k]): blk{i}.qkv is [3*D][D] with the q, k
# and v matrices stacked, blk{i}.out [D][D], blk{i}.router [N][D], blk{i}.expert{e}.w1 / .w2
# [D][D], blk{i}.ffn_w1 [H][D], blk{i}.ffn_w2 [D][H], proj_up [256][128], proj_down [128][256].


def pack_weights(L: StackLayout, tensors) -> "np.ndarray":
    """The flat fp16 blob of layout L from named (weight, bias) arrays.

    tensors maps every layer name of L.layers to (weight, bias); each array is converted to
    fp16 and must hold exactly weight_count / bias_count values (the shapes above, or flat).
    Raises KeyError for a missing layer and ValueError for a size mismatch."""
    import numpy as np

    blob = np.zeros(L.total, dtype=np.float16)
    for l in L.layers:
        w, b = tensors[l["name"]]
        w = np.asarray(w, dtype=np.float16).reshape(-1)
        b = np.asarray(b, dtype=np.float16).reshape(-1)
        if w.size != l["weight_count"] or b.size != l["bias_count"]:
            raise ValueError(f"{l['name']}: {w.size} weights / {b.size} biases, the layout wants "
                             f"{l['weight_count']} / {l['bias_count']}")
        wo, bo = l["weight_offset_fp16"], l["bias_offset_fp16"]
        blob[wo:wo + w.size] = w
        blob[bo:bo + b.size] = b
    return blob


def unpack_weights(L: StackLayout, blob) -> dict:
    """The inverse of pack_weights: {layer name: (flat weight, flat bias)} fp16 views of blob."""
    import numpy as np

    blob = np.asarray(blob, dtype=np.float16)
    out = {}
    for l in L.layers:
        wo, bo = l["weight_offset_fp16"], l["bias_offset_fp16"]
        out[l["name"]] = (blob[wo:wo + l["weight_count"]], blob[bo:bo + l["bias_count"]])
    return out


def write_weights(path: str, L: StackLayout, blob) -> str:
    """Write blob as a raw fp16 .weights file and L's table as the .json beside it (the pair
    export_weights.py writes); returns the .json path."""
    import numpy as np

    if not path.endswith(".weights"):
        raise ValueError("the weight file name must end in .weights")
    blob = np.asarray(blob, dtype=np.float16)
    if blob.size != L.total:
        raise ValueError(f"blob holds {blob.size} values, the layout {L.total}")
    blob.tofile(path)
    js = path[: -len(".weights")] + ".json"
    with open(js, "w") as f:
        f.write(L.to_json())
    return js


def read_weights(path: str):
    """(blob, table) from a .weights / .json pair; the blob is checked against the table's
    total_fp16_values."""
    import numpy as np

    with open(path[: -len(".weights")] + ".json") as f:
        table = json.load(f)
    blob = np.fromfile(path, dtype=np.float16)
    if blob.size != table["total_fp16_values"]:
        raise ValueError(f"{path}: {blob.size} fp16 values, the table says {table['total_fp16_values']}")
    return blob, table

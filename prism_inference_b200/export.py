"""Checkpoint -> the flat fp16 weight file of the transformer stack.

The file pair is the one the reference's exporter writes (vulkan_engine/export_weights.py:76-121):
a raw fp16 `.weights` file and a `.json` table {"total_fp16_values", "total_bytes", "layers":
[{"name", "type", "weight_count", "bias_count", "total_fp32", "weight_offset_fp16",
"bias_offset_fp16"}]}, weights then bias per layer, offsets in fp16 elements.  The reference
exporter converts the ncnn Convolution layers of its convolutional model; the transformer benches
lay their weights out with bump allocators (prism_moe_bench.cpp:164-172) and no trained transformer
checkpoint or model definition ships with the reference.  This module maps the named tensors of a
checkpoint onto the stack layout of layout.build_stack, so a trained model can be loaded by
prism_stack_create (Python: Stack, C++: prism_bench --weights).

    python -m prism_inference_b200.export CHECKPOINT OUT.weights --config moe64x16 [--names MAP.json]

CHECKPOINT is a .npz archive or a torch state_dict (.pt / .pth).  Default tensor names, a
PyTorch-style module tree (nn.Linear weights are [out][in], the shaders' row-major layout):

    proj_in.{weight,bias}                        -> proj_up          [256][128]
    blocks.{i}.attn.qkv.{weight,bias}            -> blk{i}.qkv       [3D][D], q, k, v stacked
      (or blocks.{i}.attn.q / .k / .v, concatenated in that order)
    blocks.{i}.attn.proj.{weight,bias}           -> blk{i}.out       [D][D]
    blocks.{i}.moe.router.{weight,bias}          -> blk{i}.router    [N][D]
    blocks.{i}.moe.experts.{e}.fc1.{weight,bias} -> blk{i}.expert{e}.w1   [D][D]
    blocks.{i}.moe.experts.{e}.fc2.{weight,bias} -> blk{i}.expert{e}.w2   [D][D]
    blocks.{i}.ffn.fc1.{weight,bias}             -> blk{i}.ffn_w1    [H][D]
    blocks.{i}.ffn.fc2.{weight,bias}             -> blk{i}.ffn_w2    [D][H]
    proj_out.{weight,bias}                       -> proj_down        [128][256]

--names takes a JSON object {layout layer name: checkpoint tensor prefix} for other naming
schemes; layers it does not list keep the default prefix.
"""
from __future__ import annotations

import argparse
import json
import re
import sys
from typing import Dict, Mapping, Optional, Tuple

import numpy as np

from . import configs, layout


def default_names(L: layout.StackLayout) -> Dict[str, str]:
    """{layout layer name: checkpoint tensor prefix} of the default convention."""
    names = {}
    for l in L.layers:
        n = l["name"]
        if n == "proj_up":
            names[n] = "proj_in"
        elif n == "proj_down":
            names[n] = "proj_out"
        else:
            m = re.fullmatch(r"blk(\d+)\.(.+)", n)
            i, rest = m.group(1), m.group(2)
            if rest == "qkv":
                names[n] = f"blocks.{i}.attn.qkv"
            elif rest == "out":
                names[n] = f"blocks.{i}.attn.proj"
            elif rest == "router":
                names[n] = f"blocks.{i}.moe.router"
            elif rest.startswith("expert"):
                e, w = re.fullmatch(r"expert(\d+)\.w([12])", rest).groups()
                names[n] = f"blocks.{i}.moe.experts.{e}.fc{w}"
            else:  # ffn_w1 / ffn_w2
                names[n] = f"blocks.{i}.ffn.fc{rest[-1]}"
    return names


def collect(L: layout.StackLayout, tensors: Mapping[str, np.ndarray],
            names: Optional[Mapping[str, str]] = None) -> Dict[str, Tuple[np.ndarray, np.ndarray]]:
    """{layout layer name: (weight, bias)} from a checkpoint's named tensors.  Raises KeyError
    naming the missing tensor."""
    prefix = default_names(L)
    if names:
        unknown = set(names) - set(prefix)
        if unknown:
            raise KeyError(f"--names lists layers the layout does not have: {sorted(unknown)}")
        prefix.update(names)
    out = {}
    for l in L.layers:
        p = prefix[l["name"]]
        if f"{p}.weight" in tensors:
            w, b = tensors[f"{p}.weight"], tensors.get(f"{p}.bias")
        elif l["name"].endswith(".qkv") and f"{p[:-4]}.q.weight" in tensors:
            base = p[:-4]
            w = np.concatenate([np.asarray(tensors[f"{base}.{x}.weight"]) for x in "qkv"], axis=0)
            bs = [tensors.get(f"{base}.{x}.bias") for x in "qkv"]
            b = None if any(v is None for v in bs) else np.concatenate([np.asarray(v) for v in bs])
        else:
            raise KeyError(f"checkpoint has no tensor {p}.weight (layer {l['name']})")
        if b is None:
            raise KeyError(f"checkpoint has no tensor {p}.bias (layer {l['name']}); the shaders add a bias "
                           "to every product")
        out[l["name"]] = (np.asarray(w, dtype=np.float32), np.asarray(b, dtype=np.float32))
    return out


def export(L: layout.StackLayout, tensors: Mapping[str, np.ndarray], out_path: str,
           names: Optional[Mapping[str, str]] = None) -> str:
    """Write the .weights / .json pair of layout L from a checkpoint's tensors; returns the .json
    path."""
    blob = layout.pack_weights(L, collect(L, tensors, names))
    return layout.write_weights(out_path, L, blob)


def load_checkpoint(path: str) -> Dict[str, np.ndarray]:
    if path.endswith(".npz"):
        with np.load(path) as z:
            return {k: z[k] for k in z.files}
    import torch
    sd = torch.load(path, map_location="cpu", weights_only=True)
    if isinstance(sd, dict) and "state_dict" in sd and isinstance(sd["state_dict"], dict):
        sd = sd["state_dict"]
    return {k: v.detach().float().numpy() for k, v in sd.items() if hasattr(v, "detach")}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("checkpoint")
    ap.add_argument("out", help="output .weights file (the .json table is written beside it)")
    ap.add_argument("--config", default="moe64x16", choices=configs.ALL)
    ap.add_argument("--n-blocks", type=int, default=None)
    ap.add_argument("--reference-widths", action="store_true", help="the shaders' dense FFN widths")
    ap.add_argument("--names", default=None, help="JSON {layout layer name: checkpoint tensor prefix}")
    a = ap.parse_args(argv)
    L = configs.get(a.config, reference_widths=a.reference_widths, n_blocks=a.n_blocks).layout
    names = json.load(open(a.names)) if a.names else None
    js = export(L, load_checkpoint(a.checkpoint), a.out, names)
    print(f"wrote {a.out} ({L.total} fp16 values) and {js}")
    return 0


if __name__ == "__main__":
    sys.exit(main())

"""prism_bench, the C++ caller of the C ABI (csrc/prism_bench.cpp): its blob layout is the
Python builder's, field for field, for every configuration (so a .weights file written by
layout.write_weights loads into it unchanged); on a GPU it runs the reference's timing
protocol end to end, with its own bit-equality check of the host-buffer output."""
import json
import subprocess

import numpy as np
import pytest

from prism_inference_b200 import abi, configs, layout, synth
from prism_inference_b200.build import BENCH

FIELDS = ("kind", "qkv_w", "qkv_b", "out_w", "out_b", "n_experts", "router_w", "router_b", "expert_w1",
          "expert_b1", "expert_w2", "expert_b2", "expert_stride", "ffn_hidden", "ffn_chunk", "ffn_w1",
          "ffn_b1", "ffn_w2", "ffn_b2")


@pytest.fixture(scope="module")
def exe():
    if not BENCH.exists():
        from prism_inference_b200 import build
        build.build()
    return str(BENCH)


@pytest.mark.parametrize("key", configs.ALL)
def test_layout_matches_python_builder(exe, key):
    r = subprocess.run([exe, "--config", key, "--layout"], capture_output=True, text=True, check=True)
    js = json.loads(r.stdout)
    L = configs.get(key).layout
    desc, blocks = abi.stack_desc(L)
    assert js["total"] == L.total
    assert (js["in_dim"], js["out_dim"]) == (L.in_dim, L.out_dim)
    assert js["up"] == [desc.up_w, desc.up_b] and js["down"] == [desc.down_w, desc.down_b]
    assert len(js["blocks"]) == len(L.blocks)
    for i, row in enumerate(js["blocks"]):
        assert row == [getattr(blocks[i], f) for f in FIELDS], f"block {i}"


def test_usage_and_no_gpu_exit_codes(exe):
    assert subprocess.run([exe, "--help"], capture_output=True).returncode == 0
    assert subprocess.run([exe, "--config", "nope"], capture_output=True).returncode == 2
    import torch
    if not torch.cuda.is_available():
        r = subprocess.run([exe, "--frames", "1"], capture_output=True, text=True)
        assert r.returncode == 3 and "no usable CUDA device" in r.stderr


@pytest.mark.gpu
def test_cpp_bench_runs_the_protocol(exe, tmp_path):
    """A short run of the C++ bench on a weights file written by the Python tooling (the
    skewed configuration's blob): device buffers, prism_stack_infer, submit/wait, batch-1
    graph; the bench itself fails unless the host-buffer outputs equal the device output."""
    cfg = configs.get("moe32x22skew")
    blob = synth.make_blob(cfg.layout, router_skew=cfg.router_skew, skew_bias=cfg.skew_bias)
    layout.write_weights(str(tmp_path / "skew.weights"), cfg.layout, blob)
    r = subprocess.run([exe, "--config", "moe32x22skew", "--frames", "4", "--warmup", "2", "--iters", "5",
                        "--weights", str(tmp_path / "skew.weights")], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    js = json.loads(r.stdout.strip().splitlines()[-1])
    assert js["weights"] == "file" and js["frames"] == 4
    assert js["device_tokens_per_s"] > 0 and js["pipelined_tokens_per_s"] > 0 and js["batch1_ms"]["mean"] > 0
    print(r.stdout)

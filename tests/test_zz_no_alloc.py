"""prism_expert_all_static - all experts of one MoE pass without any device
allocation - against the reference-style loop of one prism_expert call per expert,
through the C ABI, and against the CPU oracle of moe_expert_skip.comp.glsl.

This entry point exists for callers that cannot allocate device memory when the pass
runs, such as a post-process hook inside a game's frame loop (the setting Prism is
built for): there, cudaMalloc can synchronize the device and stall the frame, and
the host may not allow device allocation after start-up at all.  Its routing scratch
lives in a fixed per-device array that every call reuses, so the test makes two
calls in a row with different routings (the second must not see the first one's
counts) and checks the size limit.

The file is named to run last in a full `pytest -x` run, and it also passes alone.
"""
import numpy as np
import pytest

from helpers import assert_close
from prism_inference_b200 import layout, synth
from prism_inference_b200.abi import STATIC_MAX_TOKENS, ExpertParams, PrismError

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    if a.dtype == np.float16:
        return torch.from_numpy(a.view(np.int16).copy()).cuda().view(torch.float16)
    return torch.from_numpy(a.copy()).cuda()


def _host(t):
    import torch
    torch.cuda.synchronize()
    return t.view(torch.int16).cpu().numpy().view(np.float16)


def _case(seed, n_experts, frames):
    """Feature arena [y | out], assignments with some tokens owned by no expert of the call."""
    L = layout.build_stack(256, 1, n_experts=n_experts)
    blob = synth.make_blob(L, seed=synth.WEIGHT_SEED + seed)
    T = L.tokens * frames
    rng = np.random.Generator(np.random.PCG64(seed))
    feat = np.empty(2 * T * 256, np.float16)
    feat[:T * 256] = rng.standard_normal(T * 256, dtype=np.float32).astype(np.float16)
    feat[T * 256:] = np.float16(7.0)  # sentinel: rows no expert owns must keep it
    aux = rng.integers(0, n_experts, T, dtype=np.int32)
    aux[::97] = n_experts + 3  # owned by no expert of this call
    aux[::89] = -1
    b = L.blocks[0]
    p = ExpertParams(T, 256, 0, b.expert_w1, b.expert_b1, b.expert_w2, b.expert_b2, 0, T * 256, 0)
    return blob, feat, aux, p, b.expert_stride, T


def _per_expert_loop(ctx, blob, feat, aux, p, n_experts, stride):
    w, f, a = _dev(blob), _dev(feat), _dev(aux)
    for e in range(n_experts):
        o = e * stride
        q = ExpertParams(p.n_tokens, p.dim, e, p.w1_offset + o, p.b1_offset + o, p.w2_offset + o, p.b2_offset + o,
                         p.input_offset, p.output_offset, p.assignment_offset)
        ctx.expert(q, w, f, a)
    return _host(f)


def _oracle_loop(oracle, blob, feat, aux, p, n_experts, stride):
    """The CPU restatement of moe_expert_skip.comp.glsl, one dispatch per expert."""
    f = feat.copy()
    for e in range(n_experts):
        o = e * stride
        q = ExpertParams(p.n_tokens, p.dim, e, p.w1_offset + o, p.b1_offset + o, p.w2_offset + o, p.b2_offset + o,
                         p.input_offset, p.output_offset, p.assignment_offset)
        oracle.expert(q, blob, f, aux)
    return f


def test_static_expert_pass_matches_per_expert_calls(prism_ctx, oracle):
    # two calls in a row on the shared scratch: a 64-expert frame, then 16 experts
    # over 8 frames (65,280 tokens, just under the limit); each checked against the
    # per-expert entry point and against the CPU oracle
    for seed, n_experts, frames in ((1, 64, 1), (2, 16, 8)):
        blob, feat, aux, p, stride, T = _case(seed, n_experts, frames)
        ref = _per_expert_loop(prism_ctx, blob, feat, aux, p, n_experts, stride)
        w, f, a = _dev(blob), _dev(feat), _dev(aux)
        prism_ctx.expert_all_static(p, n_experts, stride, w, f, a)
        got = _host(f)
        what = f"static expert pass, {n_experts} experts x {frames} frames"
        assert_close(got[T * 256:], ref[T * 256:], what + " vs prism_expert")
        cpu = _oracle_loop(oracle, blob, feat, aux, p, n_experts, stride)
        assert_close(got[T * 256:], cpu[T * 256:], what + " vs oracle")
        unowned = (aux < 0) | (aux >= n_experts)
        out = got[T * 256:].reshape(T, 256)
        assert (out[unowned] == np.float16(7.0)).all()


def test_static_expert_pass_rejects_passes_beyond_its_scratch(prism_ctx):
    import torch
    T = STATIC_MAX_TOKENS + 1
    w = torch.zeros(300_000, dtype=torch.float16, device="cuda")
    f = torch.zeros(2 * T * 256, dtype=torch.float16, device="cuda")
    a = torch.zeros(T, dtype=torch.int32, device="cuda")
    p = ExpertParams(T, 256, 0, 0, 65536, 65792, 131328, 0, T * 256, 0)
    with pytest.raises(PrismError, match="RANGE"):
        prism_ctx.expert_all_static(p, 1, 0, w, f, a)

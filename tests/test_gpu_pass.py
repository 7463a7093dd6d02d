"""Per-pass drop-ins on the GPU (through the C ABI) against the reference's shader
outputs (golden vectors) and the oracle, including full 120x68 frames."""
import sys
from pathlib import Path

import numpy as np
import pytest

from helpers import assert_close, routing_agreement
from prism_inference_b200.abi import AttnParams, DenseParams, ExpertParams, PrismError, ProjParams, RouterParams

GOLD = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLD))
from cases import HOT_CASES, build, output_of  # noqa: E402

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    if a is None:
        return torch.zeros(1, dtype=torch.int32, device="cuda")
    if a.dtype == np.float16:
        return torch.from_numpy(a.view(np.int16).copy()).cuda().view(torch.float16)
    return torch.from_numpy(a.copy()).cuda()


def _host(t, like):
    import torch
    torch.cuda.synchronize()
    if t.dtype == torch.float16:
        return t.view(torch.int16).cpu().numpy().view(np.float16)
    return t.cpu().numpy()


def run_gpu(ctx, c):
    sh, p = c["shader"], c["push"]
    w, f, a = _dev(c["blob"]), _dev(c["feat"]), _dev(c["aux"])
    if sh == "split2_qkv_attn_d256":
        ctx.attn_window(AttnParams(*p), w, f)
    elif sh == "moe_router":
        ctx.router(RouterParams(*p), w, f, a)
    elif sh == "moe_expert_skip":
        for q in p:
            ctx.expert(ExpertParams(*q), w, f, a)
    elif sh == "moe_ffn_16exp":
        T, D, rw, rb, stride, w1, b1, w2, b2, inp, out = p
        import torch
        aux = torch.zeros(T + 16, dtype=torch.int32, device="cuda")
        ctx.router(RouterParams(T, D, 16, rw, rb, inp, 0, T), w, f, aux)
        for e in range(16):
            eo = e * stride
            ctx.expert(ExpertParams(T, D, e, w1 + eo, b1 + eo, w2 + eo, b2 + eo, inp, out, 0), w, f, aux)
    elif sh == "attention_windowed_d256":
        ctx.dense_block(DenseParams(*p), 1024, 256, w, f)
    elif sh == "attention_windowed":
        ctx.dense_block(DenseParams(*p), 512, 512, w, f)
    elif sh == "pw_project_128to256":
        ctx.proj_up(ProjParams(*p), w, f)
    elif sh == "pw_project_256to128":
        ctx.proj_down(ProjParams(*p), w, f)
    c = dict(c)
    c["feat"] = _host(f, c["feat"])
    if c["aux"] is not None:
        c["aux"] = _host(a, c["aux"])
    return output_of(c)


@pytest.mark.parametrize("name", HOT_CASES)
def test_pass_matches_reference_golden(prism_ctx, name):
    gold = np.load(GOLD / "golden.npz")[name]
    got = run_gpu(prism_ctx, build(name))
    if got.dtype == np.float16:
        assert_close(got, gold, name)
    else:  # router: assignment + counts; the golden inputs have no near-ties
        assert (got == gold).all()


def _moe_frame(n_experts, seed=0, w=120, h=68):
    from prism_inference_b200 import layout, synth
    L = layout.build_stack(256, 1, n_experts=n_experts, spatial_w=w, spatial_h=h)
    return L, synth.make_blob(L, seed=synth.WEIGHT_SEED + seed), synth.make_frames(L, 1, first=seed)[0]


def test_full_frame_moe_block_passes(prism_ctx, oracle):
    """attention -> router (N=64) -> 64 expert dispatches on a 120x68 frame, as
    prism_moe_bench.cpp:416-437 records them, against the oracle."""
    import torch
    L, blob, x = _moe_frame(64)
    T, D = L.tokens, 256
    b = L.blocks[0]
    feat = np.zeros(3 * T * D, np.float16)
    feat[:T * D] = x.reshape(-1)
    aux = np.zeros(T + 64, np.int32)
    wd, fd, ad = _dev(blob), _dev(feat), _dev(aux)
    pa = AttnParams(T, D, 8, 32, 120, 68, 8, b.qkv_w, b.qkv_b, b.out_w, b.out_b, 0, T * D)
    pr = RouterParams(T, D, 64, b.router_w, b.router_b, T * D, 0, T)
    prism_ctx.attn_window(pa, wd, fd)
    prism_ctx.router(pr, wd, fd, ad)
    oracle.attn(pa, blob, feat)
    g_feat = _host(fd, feat)
    assert_close(g_feat[T * D:2 * T * D], feat[T * D:2 * T * D], "attention")
    # router on the GPU's attention output in both (isolates the router)
    feat[T * D:2 * T * D] = g_feat[T * D:2 * T * D]
    margin = oracle.router(pr, blob, feat, aux, want_margin=True)
    g_aux = _host(ad, aux)
    hard, ties = routing_agreement(g_aux[:T], aux[:T], margin)
    assert hard == 0, f"{hard} tokens routed differently at margin >= 1e-3 ({ties} at ties)"
    assert g_aux[T:T + 64].sum() == T
    # experts with the GPU's routing in both
    ad2 = _dev(g_aux)
    for e in range(64):
        eo = e * b.expert_stride
        pe = ExpertParams(T, D, e, b.expert_w1 + eo, b.expert_b1 + eo, b.expert_w2 + eo, b.expert_b2 + eo, T * D,
                          2 * T * D, 0)
        prism_ctx.expert(pe, wd, fd, ad2)
        oracle.expert(pe, blob, feat, g_aux)
    assert_close(_host(fd, feat)[2 * T * D:], feat[2 * T * D:], "experts")


def test_reference_bump_layout_unaligned_experts(prism_ctx, oracle):
    """The reference's own bump layout (prism_moe_bench.cpp:164-172: qkv, out, an unused
    dense FFN slot, a 4-row router, experts) puts expert weights at 8-byte boundaries;
    the per-pass kernels read the blob at any 2-byte alignment."""
    rng = np.random.Generator(np.random.PCG64(5))
    off = 0

    def wa(n):
        nonlocal off
        o = off
        off += n
        return o
    qkv_w, qkv_b, out_w, out_b = wa(3 * 65536), wa(768), wa(65536), wa(256)
    wa(1024 * 256), wa(1024), wa(256 * 1024), wa(256)
    rtr_w, rtr_b = wa(4 * 256), wa(4)
    e0 = [wa(65536), wa(256), wa(65536), wa(256)]
    for _ in range(3):
        wa(65536), wa(256), wa(65536), wa(256)
    assert (e0[0] * 2) % 16 == 8
    blob = (rng.standard_normal(off, dtype=np.float32) * 0.02).astype(np.float16)
    T = 120 * 68
    feat = np.zeros(3 * T * 256, np.float16)
    feat[:T * 256] = rng.standard_normal(T * 256, dtype=np.float32).astype(np.float16)
    aux = np.zeros(T + 64, np.int32)
    wd, fd, ad = _dev(blob), _dev(feat), _dev(aux)
    pa = AttnParams(T, 256, 8, 32, 120, 68, 8, qkv_w, qkv_b, out_w, out_b, 0, T * 256)
    prism_ctx.attn_window(pa, wd, fd)
    oracle.attn(pa, blob, feat)
    pr = RouterParams(T, 256, 4, rtr_w, rtr_b, T * 256, 0, T)
    feat[T * 256:2 * T * 256] = _host(fd, feat)[T * 256:2 * T * 256]
    prism_ctx.router(pr, wd, fd, ad)
    g_aux = _host(ad, aux)
    for e in range(4):
        eo = e * 131584
        pe = ExpertParams(T, 256, e, e0[0] + eo, e0[1] + eo, e0[2] + eo, e0[3] + eo, T * 256, 2 * T * 256, 0)
        prism_ctx.expert(pe, wd, fd, ad)
        oracle.expert(pe, blob, feat, g_aux)
    assert_close(_host(fd, feat)[2 * T * 256:], feat[2 * T * 256:], "unaligned experts")


def test_out_of_range_offsets_are_rejected(prism_ctx):
    import torch
    w = torch.zeros(1000, dtype=torch.float16, device="cuda")
    f = torch.zeros(1000, dtype=torch.float16, device="cuda")
    with pytest.raises(PrismError, match="RANGE"):
        prism_ctx.attn_window(AttnParams(64, 256, 8, 32, 8, 8, 8, 0, 0, 0, 0, 0, 0), w, f)
    with pytest.raises(PrismError, match="UNSUPPORTED"):
        prism_ctx.attn_window(AttnParams(64, 192, 6, 32, 8, 8, 8, 0, 0, 0, 0, 0, 0), w, f)
    a = torch.zeros(10, dtype=torch.int32, device="cuda")
    with pytest.raises(PrismError, match="UNSUPPORTED"):
        prism_ctx.router(RouterParams(1, 256, 300, 0, 0, 0, 0, 0), w, f, a)

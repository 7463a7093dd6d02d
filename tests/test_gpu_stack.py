"""The fast path (prism_stack_forward: tcgen05 adapters, route + grouped expert
GEMM) against the oracle stack.

Routing: the oracle follows the GPU's choice only where its own top-2 margin is
below 1e-3 (a tie); any other difference is a hard mismatch and fails the test.
Ties are reported."""
import numpy as np
import pytest

from helpers import TIE_MARGIN, assert_close
from prism_inference_b200 import Prism, Stack, configs, layout, synth

pytestmark = pytest.mark.gpu


def _run(ctx, L, blob, x, max_frames=None, pair=True, buckets=True):
    import torch
    F = x.shape[0]
    st = Stack(ctx, L, blob, max_frames or F)
    st.set_pair_attention(pair)
    st.set_bucket_routing(buckets)
    xd = torch.from_numpy(x.view(np.int16)).cuda().view(torch.float16)
    out = torch.empty((F, L.tokens, L.out_dim), dtype=torch.float16, device="cuda")
    asg = torch.full((max(1, L.n_moe_blocks), F * L.tokens), -1, dtype=torch.int32, device="cuda")
    st.forward(xd, out, asg)
    torch.cuda.synchronize()
    st.status()
    o = out.view(torch.int16).cpu().numpy().view(np.float16)
    a = asg.cpu().numpy()
    st.close()
    return o, a


def _check(ctx, oracle, L, blob, x, what):
    o, a = _run(ctx, L, blob, x)
    ref, ra, stats = oracle.stack(L, blob, x, forced=a if L.n_moe_blocks else None, tie_thr=TIE_MARGIN)
    assert stats[2] == 0, f"{what}: {stats[2]} hard routing mismatches"
    m = assert_close(o, ref, what)
    print(f"{what}: max_abs {m[0]:.3g} rel_l2 {m[1]:.3g}; routed {stats[0]}, followed at ties {stats[1]}, "
          f"near-ties {stats[3]}")
    return o, a


def test_stack_adapters_only(prism_ctx, oracle):
    """The two tcgen05 adapter GEMMs alone (no blocks): 128->256 ReLU, 256->128."""
    L = layout.build_stack(256, 0, up_adapter=True, down_adapter=True)
    blob = synth.make_blob(L)
    x = synth.make_frames(L, 2)
    o, _ = _run(prism_ctx, L, blob, x)
    ref, _, _ = oracle.stack(L, blob, x)
    assert_close(o, ref, "adapters")


@pytest.mark.parametrize("key,n_blocks,frames", [("moe16x1", 1, 1), ("moe64x16", 2, 2), ("moe32x22skew", 2, 1),
                                                 ("dense256x12", 2, 1), ("dense128x4", 2, 2)])
def test_stack_matches_oracle(prism_ctx, oracle, key, n_blocks, frames):
    cfg = configs.get(key, n_blocks=n_blocks)
    blob = synth.make_blob(cfg.layout, router_skew=cfg.router_skew, skew_bias=cfg.skew_bias)
    x = synth.make_frames(cfg.layout, frames)
    _check(prism_ctx, oracle, cfg.layout, blob, x, key)


@pytest.mark.parametrize("n_experts", [1, 100, 256])
def test_stack_expert_counts(prism_ctx, oracle, n_experts):
    """Router widths at the edges: one expert (16 padded logits), 100 (two router weight
    stages of 96 + 16 rows), 256 (three stages, logits up to the last TMEM column); the
    route plan's tile list with many partial tiles."""
    L = layout.build_stack(256, 1, n_experts=n_experts, up_adapter=True, down_adapter=True)
    blob = synth.make_blob(L, seed=synth.WEIGHT_SEED + n_experts)
    x = synth.make_frames(L, 2)
    _, a = _check(prism_ctx, oracle, L, blob, x, f"{n_experts} experts")
    assert a.min() >= 0 and a.max() < n_experts


@pytest.mark.parametrize("w,h,frames", [(4, 4, 2), (20, 12, 3), (8, 8, 1), (40, 9, 2)])
def test_stack_odd_frame_shapes(prism_ctx, oracle, w, h, frames):
    """Partial windows in x and y, frames of fewer than 64 tokens (keys = n_tokens),
    odd window counts (a tile with one window)."""
    L = layout.build_stack(256, 2, n_experts=8, up_adapter=True, down_adapter=True, spatial_w=w, spatial_h=h)
    blob = synth.make_blob(L)
    x = synth.make_frames(L, frames)
    _check(prism_ctx, oracle, L, blob, x, f"{w}x{h}x{frames}")


@pytest.mark.parametrize("what,dim_blocks,kw,frames", [
    ("moe64 68x120", 2, dict(n_experts=64), 1),
    ("moe100 68x120", 1, dict(n_experts=100), 1),
    ("moe256 68x120", 1, dict(n_experts=256), 1),
    ("dense256 68x120", 2, dict(ffn_hidden=1024, ffn_chunk=256), 1),
    ("moe8 20x12", 2, dict(n_experts=8, spatial_w=20, spatial_h=12), 3),
    ("moe8 4x4", 2, dict(n_experts=8, spatial_w=4, spatial_h=4), 1),
    ("moe8 40x9", 1, dict(n_experts=8, spatial_w=40, spatial_h=9), 2),
])
def test_pair_attention_is_bit_identical(prism_ctx, oracle, what, dim_blocks, kw, frames):
    """The latency paths against the plain ones: attention with each tile split over a CTA pair
    (taken when a forward has at most sm_count / 2 attention tiles) against one CTA per tile, and
    bucket routing (router-filled expert buckets, no route kernel) against the route kernel's
    compact permutation: all four combinations give the same output and routing bit for bit, and
    the default one matches the oracle within tolerance.  Covers one 68x120 frame, router widths
    of 1-3 weight stages, a dense block, partial windows, a tile with one window and frames of
    fewer than 64 tokens."""
    L = layout.build_stack(256, dim_blocks, up_adapter=True, down_adapter=True, **kw)
    blob = synth.make_blob(L)
    x = synth.make_frames(L, frames)
    o1, a1 = _check(prism_ctx, oracle, L, blob, x, what)
    for pair, buckets in ((False, True), (True, False), (False, False)):
        o0, a0 = _run(prism_ctx, L, blob, x, pair=pair, buckets=buckets)
        how = f"{what} (pair {pair}, buckets {buckets})"
        assert np.array_equal(a0, a1), f"{how}: routing differs from the default path"
        assert np.array_equal(o0.view(np.int16), o1.view(np.int16)), f"{how}: outputs differ"


@pytest.mark.parametrize("key", ["dense256x12", "dense128x4"])
def test_stack_reference_ffn_widths(prism_ctx, oracle, key):
    """The shader widths: FFN 1024 in four fp16-accumulated chunks (d256) and 512
    unsplit (d128)."""
    cfg = configs.get(key, reference_widths=True, n_blocks=2)
    blob = synth.make_blob(cfg.layout)
    x = synth.make_frames(cfg.layout, 1)
    _check(prism_ctx, oracle, cfg.layout, blob, x, key + "-ref-widths")


@pytest.mark.parametrize("hidden,chunk", [(128, 128), (256, 256), (512, 512), (512, 128), (512, 256)])
def test_dense128_ffn_shapes(prism_ctx, oracle, hidden, chunk):
    """The dim-128 block on tensor cores for every FFN shape its kernels take: one product of
    width 128, 256 or 512 (the d128 shader's unsplit FFN, attention_windowed.comp.glsl:151-170;
    256 and 512 accumulate GEMM2 over 256-wide pieces of the hidden layer in fp32), and 128- or
    256-wide chunks summed in fp16 (the d256 shader's rule)."""
    L = layout.build_stack(128, 2, n_heads=4, ffn_hidden=hidden, ffn_chunk=chunk, spatial_w=40, spatial_h=20)
    blob = synth.make_blob(L, seed=synth.WEIGHT_SEED + hidden + chunk)
    x = synth.make_frames(L, 3)
    _check(prism_ctx, oracle, L, blob, x, f"d128 ffn {hidden}/{chunk}")


def test_dense128_unsupported_ffn_is_rejected(prism_ctx):
    from prism_inference_b200.abi import PrismError
    L = layout.build_stack(128, 1, n_heads=4, ffn_hidden=384, ffn_chunk=384)
    with pytest.raises(PrismError, match="UNSUPPORTED"):
        Stack(prism_ctx, L, synth.make_blob(L), 1)


def test_stack_from_exported_weight_file(prism_ctx, oracle, tmp_path):
    """The trained-model path end to end: named checkpoint tensors -> export.py -> the
    .weights / .json pair -> the layout rebuilt from the JSON table alone -> prism_stack_create
    from the file's blob -> GPU forward, against the oracle run on the same file."""
    from helpers import checkpoint_of
    from prism_inference_b200 import export
    L = configs.get("moe64x16", n_blocks=2).layout
    ck = checkpoint_of(L, synth.make_blob(L, seed=synth.WEIGHT_SEED + 77), split_qkv=True)
    np.savez(tmp_path / "ck.npz", **ck)
    path = str(tmp_path / "prism.weights")
    assert export.main([str(tmp_path / "ck.npz"), path, "--config", "moe64x16", "--n-blocks", "2"]) == 0
    blob, table = layout.read_weights(path)
    L2 = layout.stack_from_json(table, 256, 8, 64, 2)
    x = synth.make_frames(L2, 2)
    _check(prism_ctx, oracle, L2, blob, x, "moe64x16 from an exported weight file")


def test_headline_stack_full_depth(prism_ctx, oracle):
    """Config 4 as benchmarked: 64 experts x 16 blocks + adapters, one frame."""
    cfg = configs.get("moe64x16")
    blob = synth.make_blob(cfg.layout)
    x = synth.make_frames(cfg.layout, 1)
    _check(prism_ctx, oracle, cfg.layout, blob, x, "moe64x16-full")


def _truncated(L, k):
    """The first k blocks of L over the same blob, without the down adapter (dim-256 output):
    the stack's state after block k."""
    import copy
    T = copy.deepcopy(L)
    T.blocks = T.blocks[:k]
    T.down_w, T.down_b, T.out_dim = -1, -1, T.dim
    return T


@pytest.mark.parametrize("seed", [1, 2, 3, 4])
def test_headline_stack_seeds_and_depth(prism_ctx, oracle, seed):
    """Config 4 at full depth on four more weight and input seeds, with the error after
    blocks 1, 2, 4, 8 and 16 reported (each a truncated stack over the same blob, checked
    against the oracle with its own routing): the margin to the tolerance at every depth."""
    cfg = configs.get("moe64x16")
    L = cfg.layout
    blob = synth.make_blob(L, seed=synth.WEIGHT_SEED + 7919 * seed)
    x = synth.make_frames(L, 1, first=101 * seed)
    rows = []
    for k in (1, 2, 4, 8, 16):
        o, a = _run(prism_ctx, _truncated(L, k), blob, x)
        ref, _, stats = oracle.stack(_truncated(L, k), blob, x, forced=a, tie_thr=TIE_MARGIN)
        assert stats[2] == 0, f"seed {seed}, {k} blocks: {stats[2]} hard routing mismatches"
        m = assert_close(o, ref, f"seed {seed}, after block {k}")
        rows.append(f"{k}:{m[0]:.2g}/{m[1]:.2g}")
    _check(prism_ctx, oracle, L, blob, x, f"moe64x16-full seed {seed}")
    print(f"seed {seed} max_abs/rel_l2 by depth: " + " ".join(rows))


def test_skewed_config_full_depth(prism_ctx, oracle):
    """Config 5 at its full depth: 32 experts x 22 blocks + adapters, about half of the
    tokens routed to 4 experts (long expert segments, many full tiles of one expert)."""
    cfg = configs.get("moe32x22skew")
    blob = synth.make_blob(cfg.layout, router_skew=cfg.router_skew, skew_bias=cfg.skew_bias)
    x = synth.make_frames(cfg.layout, 2)
    _check(prism_ctx, oracle, cfg.layout, blob, x, "moe32x22skew-full")


def test_bench_workload_frames(prism_ctx, oracle):
    """The benchmarked workload itself (config 4, 64 frames, 16 blocks): sampled frames of
    the batch equal single-frame runs bit for bit (tiles and expert segments mix frames and
    hold up to 64x a single frame's rows), and the last frame matches the oracle."""
    import torch
    cfg = configs.get("moe64x16")
    L = cfg.layout
    T = L.tokens
    blob = synth.make_blob(L)
    x = synth.make_frames(L, 64)
    st = Stack(prism_ctx, L, blob, 64)
    xd = torch.from_numpy(x.view(np.int16)).cuda().view(torch.float16)
    out = torch.empty((64, T, L.out_dim), dtype=torch.float16, device="cuda")
    asg = torch.empty((L.n_moe_blocks, 64 * T), dtype=torch.int32, device="cuda")
    st.forward(xd, out, asg)
    one = torch.empty((1, T, L.out_dim), dtype=torch.float16, device="cuda")
    asg1 = torch.empty((L.n_moe_blocks, T), dtype=torch.int32, device="cuda")
    for f in (0, 37, 63):
        st.forward(xd[f:f + 1], one, asg1)
        assert torch.equal(one[0].view(torch.int16), out[f].view(torch.int16)), f
        assert torch.equal(asg1, asg[:, f * T:(f + 1) * T]), f
    torch.cuda.synchronize()
    st.status()
    o = out[63:].view(torch.int16).cpu().numpy().view(np.float16)
    a = asg[:, 63 * T:].cpu().numpy()
    st.close()
    ref, _, stats = oracle.stack(L, blob, x[63:], forced=a, tie_thr=TIE_MARGIN)
    assert stats[2] == 0, f"{stats[2]} hard routing mismatches"
    m = assert_close(o, ref, "moe64x16 frame 63 of 64")
    print(f"frame 63 of 64: max_abs {m[0]:.3g} rel_l2 {m[1]:.3g}; followed at ties {stats[1]}")


def test_frames_are_independent_and_deterministic(prism_ctx):
    """Frame f gives the same bits alone and inside a batch (tiles mix frames), and
    two runs give the same bits."""
    cfg = configs.get("moe64x16", n_blocks=3)
    blob = synth.make_blob(cfg.layout)
    x = synth.make_frames(cfg.layout, 4)
    o4, a4 = _run(prism_ctx, cfg.layout, blob, x)
    o4b, _ = _run(prism_ctx, cfg.layout, blob, x)
    o1, a1 = _run(prism_ctx, cfg.layout, blob, x[2:3], max_frames=4)
    assert (o4.view(np.uint16) == o4b.view(np.uint16)).all()
    assert (o4[2].view(np.uint16) == o1[0].view(np.uint16)).all()
    T = cfg.layout.tokens
    assert (a4[:, 2 * T:3 * T] == a1).all()


def test_stack_graph_replay_matches_eager(prism_ctx):
    """prism_stack_forward captured in a CUDA graph (its kernels chained by programmatic
    dependent launch) gives the eager call's bits on every replay, also for routing."""
    import torch
    cfg = configs.get("moe64x16", n_blocks=3)
    L = cfg.layout
    blob = synth.make_blob(L)
    x = synth.make_frames(L, 2)
    st = Stack(prism_ctx, L, blob, 2)
    xd = torch.from_numpy(x.view(np.int16)).cuda().view(torch.float16)
    eager = torch.empty((2, L.tokens, L.out_dim), dtype=torch.float16, device="cuda")
    asg_e = torch.empty((L.n_moe_blocks, 2 * L.tokens), dtype=torch.int32, device="cuda")
    st.forward(xd, eager, asg_e)
    torch.cuda.synchronize()
    out = torch.empty_like(eager)
    asg = torch.empty_like(asg_e)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # warm the capture stream, as torch recommends
        st.forward(xd, out, asg)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        st.forward(xd, out, asg)
    for _ in range(2):
        out.zero_()
        asg.fill_(-1)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), eager.view(torch.int16))
        assert torch.equal(asg, asg_e)
    st.status()
    del g
    st.close()


def test_routing_histogram_and_skew(prism_ctx):
    cfg = configs.get("moe32x22skew", n_blocks=2)
    blob = synth.make_blob(cfg.layout, router_skew=cfg.router_skew, skew_bias=cfg.skew_bias)
    x = synth.make_frames(cfg.layout, 2)
    _, a = _run(prism_ctx, cfg.layout, blob, x)
    for blk in a:
        h = np.bincount(blk, minlength=32)
        assert h.sum() == blk.size and blk.min() >= 0 and blk.max() < 32
        frac = h[:4].sum() / blk.size
        assert 0.3 < frac < 0.7, f"skewed experts take {frac:.2f} of the tokens"


def test_stack_zero_frames_is_a_no_op(prism_ctx):
    """An empty batch launches nothing and leaves the output untouched; the next full call
    is unaffected (routing counters stay clean)."""
    import torch
    cfg = configs.get("moe16x1")
    blob = synth.make_blob(cfg.layout)
    st = Stack(prism_ctx, cfg.layout, blob, 1)
    x = torch.zeros((1, cfg.layout.tokens, cfg.layout.in_dim), dtype=torch.float16, device="cuda")
    out = torch.full((1, cfg.layout.tokens, cfg.layout.out_dim), 7.0, dtype=torch.float16, device="cuda")
    st.forward(x[:0], out[:0])  # frames = 0 (valid pointers)
    torch.cuda.synchronize()
    st.status()
    assert bool((out == 7.0).all())
    st.close()
    o1, a1 = _run(prism_ctx, cfg.layout, blob, synth.make_frames(cfg.layout, 1))
    o2, a2 = _run(prism_ctx, cfg.layout, blob, synth.make_frames(cfg.layout, 1))
    assert (o1.view(np.uint16) == o2.view(np.uint16)).all() and (a1 == a2).all()


def test_moe_block_on_caller_arenas(prism_ctx, oracle):
    """prism_moe_block on views into one feature arena and one aux arena at the reference's
    pass offsets (input, output, assignments, counts): the block's output matches the oracle,
    the counts are the histogram of the assignments, and the arena outside the output is
    untouched.  A handle with adapters or more blocks is refused."""
    import torch
    from prism_inference_b200.abi import PrismError
    cfg = configs.get("moe16x1")
    L = cfg.layout
    T = L.tokens
    blob = synth.make_blob(L)
    x = synth.make_frames(L, 1)
    blk = Stack(prism_ctx, L, blob, 1)
    arena = torch.full((3 * T * 256,), 5.0, dtype=torch.float16, device="cuda")
    arena[:T * 256] = torch.from_numpy(x.reshape(-1).view(np.int16)).cuda().view(torch.float16)
    aux = torch.full((T + 64,), -7, dtype=torch.int32, device="cuda")
    xin = arena[:T * 256].view(1, T, 256)
    xout = arena[2 * T * 256:].view(1, T, 256)
    blk.moe_block(xin, xout, aux[:T], aux[T:T + 16])
    torch.cuda.synchronize()
    blk.status()
    a = aux[:T].cpu().numpy()
    counts = aux[T:T + 16].cpu().numpy()
    assert (counts == np.bincount(a, minlength=16)).all()
    assert (aux[T + 16:] == -7).all() and (arena[T * 256:2 * T * 256] == 5.0).all()
    o = xout.view(torch.int16).cpu().numpy().view(np.float16)
    ref, _, stats = oracle.stack(L, blob, x, forced=a[None], tie_thr=TIE_MARGIN)
    assert stats[2] == 0
    assert_close(o, ref, "prism_moe_block")
    blk.close()
    L2 = layout.build_stack(256, 1, n_experts=16, up_adapter=True, down_adapter=True)
    st = Stack(prism_ctx, L2, synth.make_blob(L2), 1)
    with pytest.raises(PrismError, match="ARG"):
        st.moe_block(xin, xout)
    st.close()


def test_host_buffer_infer_and_pipelined_submit(prism_ctx):
    """prism_stack_infer (the reference's Infer: host in, host out, GPU ms) and the pipelined
    prism_stack_submit / prism_stack_wait give prism_stack_forward's bits: pageable numpy and
    page-locked tensor buffers, five submissions of different sizes through the two staging
    slots (one empty), a submission without download, host and device-side waits."""
    import torch
    from prism_inference_b200.abi import PrismError
    cfg = configs.get("moe64x16", n_blocks=2)
    L = cfg.layout
    T = L.tokens
    blob = synth.make_blob(L)
    x = synth.make_frames(L, 3)
    st = Stack(prism_ctx, L, blob, 3)
    xd = torch.from_numpy(x.view(np.int16)).cuda().view(torch.float16)
    ref = torch.empty((3, T, L.out_dim), dtype=torch.float16, device="cuda")
    st.forward(xd, ref)
    torch.cuda.synchronize()
    st.status()
    ref_h = ref.view(torch.int16).cpu().numpy()

    out_np = np.zeros((3, T, L.out_dim), np.float16)
    ms = st.infer(x, out_np)
    assert ms > 0.0
    assert (out_np.view(np.int16) == ref_h).all()

    xin = torch.from_numpy(x.view(np.int16)).pin_memory()
    sizes = [3, 1, 2, 0, 3]
    outs = [torch.zeros((3, T, L.out_dim), dtype=torch.int16).pin_memory() for _ in sizes]
    tickets = [st.submit(xin[:n], outs[i][:n]) for i, n in enumerate(sizes)]
    assert tickets == list(range(tickets[0], tickets[0] + len(sizes)))
    st.wait(tickets[-1])  # covers every earlier ticket
    for i, n in enumerate(sizes):
        assert (outs[i][:n].numpy() == ref_h[:n]).all(), i
        assert not outs[i][n:].any(), i  # nothing written past the submitted frames

    t = st.submit(xin, None)  # forward without download
    outs[0].zero_()
    t = st.submit(xin, outs[0])
    st.wait(t, host=False)  # the current stream waits on the device for the download
    ev = torch.cuda.Event()
    ev.record()
    ev.synchronize()  # the current stream only: done once the download has landed
    assert (outs[0].numpy() == ref_h).all()
    st.status()
    with pytest.raises(PrismError, match="RANGE"):
        st.wait(t + 1)
    st.close()


def test_infer_gpu_on_caller_buffers_with_byte_offsets(prism_ctx):
    """prism_stack_infer_gpu (InferGPU, prism_vulkan.cpp:922-1004): frames read from and written
    to the caller's device buffers at byte offsets.  16-byte aligned offsets run in place, a
    2-byte offset goes through the staging slot; both give prism_stack_forward's bits and leave
    the buffers outside the output untouched.  Overlapping ranges and host memory are refused."""
    import torch
    from prism_inference_b200.abi import PrismError
    cfg = configs.get("moe64x16", n_blocks=2)
    L = cfg.layout
    T = L.tokens
    blob = synth.make_blob(L)
    x = synth.make_frames(L, 2)
    st = Stack(prism_ctx, L, blob, 2)
    xd = torch.from_numpy(x.view(np.int16)).cuda().view(torch.float16)
    ref = torch.empty((2, T, L.out_dim), dtype=torch.float16, device="cuda")
    st.forward(xd, ref)
    torch.cuda.synchronize()
    st.status()
    nin, nout = x.nbytes, ref.numel() * 2
    for off_in, off_out in ((256, 4096), (2, 6)):
        src = torch.full((off_in + nin + 64,), 0x5A, dtype=torch.uint8, device="cuda")
        src[off_in:off_in + nin] = xd.view(torch.uint8).reshape(-1)
        dst = torch.full((off_out + nout + 64,), 0x33, dtype=torch.uint8, device="cuda")
        ms = st.infer_gpu(src, dst, 2, off_in, off_out)
        assert ms > 0.0
        got = dst[off_out:off_out + nout].view(torch.int16).view(2, T, L.out_dim)
        assert torch.equal(got, ref.view(torch.int16)), (off_in, off_out)
        assert bool((dst[:off_out] == 0x33).all()) and bool((dst[off_out + nout:] == 0x33).all())
    arena = torch.zeros(nin + nout, dtype=torch.uint8, device="cuda")
    with pytest.raises(PrismError, match="ARG"):
        st.infer_gpu(arena, arena, 2, 0, nin - 16)  # output overlaps the input
    with pytest.raises(PrismError, match="ARG"):
        st.infer_gpu(torch.zeros(nin, dtype=torch.uint8), arena, 2)  # host memory
    st.close()


def test_device_wait_timeout_is_reported_and_recovered(prism_ctx):
    """A device wait that nothing releases gives up after the library's wait limit (2 s)
    instead of hanging: prism_stack_status raises PRISM_E_TIMEOUT once, resets the routing
    state the stalled kernel left behind, and the next forward gives a clean run's bits.  A
    forward issued between the stall and the status call finds the routing counts
    inconsistent, plans no expert work, and is reported through the same status call."""
    import time

    import torch
    from prism_inference_b200.abi import PrismError
    cfg = configs.get("moe64x16", n_blocks=2)
    L = cfg.layout
    blob = synth.make_blob(L)
    x = synth.make_frames(L, 2)
    st = Stack(prism_ctx, L, blob, 2)
    xd = torch.from_numpy(x.view(np.int16)).cuda().view(torch.float16)
    ref = torch.empty((2, L.tokens, L.out_dim), dtype=torch.float16, device="cuda")
    st.forward(xd, ref)
    torch.cuda.synchronize()
    st.status()
    out = torch.empty_like(ref)

    t0 = time.perf_counter()
    st.inject_stall()
    with pytest.raises(PrismError, match="TIMEOUT"):
        st.status()
    waited = time.perf_counter() - t0
    assert 1.5 < waited < 60, f"the stalled wait ended after {waited:.2f} s"
    st.status()  # the error word was cleared
    out.zero_()
    st.forward(xd, out)
    torch.cuda.synchronize()
    st.status()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))

    st.inject_stall()
    st.forward(xd, out)  # counts one token high: routing must refuse, not scatter out of range
    with pytest.raises(PrismError, match="TIMEOUT"):
        st.status()
    out.zero_()
    st.forward(xd, out)
    torch.cuda.synchronize()
    st.status()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    st.close()


def test_stack_argument_errors(prism_ctx):
    import torch
    from prism_inference_b200.abi import PrismError
    cfg = configs.get("moe16x1")
    blob = synth.make_blob(cfg.layout)
    st = Stack(prism_ctx, cfg.layout, blob, 1)
    x = torch.zeros((2, cfg.layout.tokens, 256), dtype=torch.float16, device="cuda")
    out = torch.zeros_like(x)
    with pytest.raises(PrismError, match="RANGE"):
        st.forward(x, out)  # 2 frames > max_frames 1
    with pytest.raises(PrismError, match="ARG"):
        st.forward(x[:1], x[:1])  # out aliases in
    L = layout.build_stack(256, 1, n_experts=16)
    with pytest.raises(PrismError, match="RANGE"):
        Stack(prism_ctx, L, blob[:1000], 1)
    from prism_inference_b200 import abi
    assert st.lib.prism_stack_set_option(st.h, 99, 1) == abi.PRISM_E_ARG  # unknown option
    assert st.lib.prism_stack_set_option(st.h, abi.OPT_BUCKET_ROUTING, 0) == 0
    st.close()

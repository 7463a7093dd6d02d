#!/usr/bin/env python3
"""Benchmark of the MoE transformer stack (BASELINE.json metric: tokens/s and
frames/s at 68x120 tokens on 1/2/4/8 B200, plus batch-1 latency).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config moe64x16] [--frames B]

Workload (N=1 and per rank): BASELINE.json config 4, the 64-expert x 16-block dim-256
stack with the 128->256 / 256->128 adapters, B = 64 frames of 68x120 tokens per GPU
(weak scaling: every rank runs its own B frames with replicated weights; there is no
collective on the data path).  A step is one prism_stack_forward over the B frames.
Data: seeded synthetic frames ~N(0,1) and weights ~N(0,0.02) (the reference ships
neither).  The activations (267 MB per buffer) are larger than the 126 MB L2.

value: tokens/s over all ranks, inputs resident in HBM, device time (CUDA events,
max over ranks).  e2e: the same metric through the C ABI's host-buffer call
(prism_stack_submit / prism_stack_wait) from page-locked host memory: the host->device copy
of every step's frames and the device->host copy of every step's output are inside the timed
region, overlapped across neighbouring steps by the library's two staging slots as a serving
loop runs.  roofline: the kernel kind with the largest share of the
timed region, its algorithmic FLOPs per launch (the attention kernel's include the router GEMM
fused into it) / its mean event-timed duration,
against the sustained cuBLAS bf16 figure of MEASURED_PEAKS.json.

--impl reference: the reference's own implementation of the path on the host cores:
its GLSL shader sources compiled as C++ (oracle/_ref, see oracle/glsl_ref), dispatched
in the order of prism_moe_bench.cpp:408-444 with all host threads.  The reference
Vulkan path cannot run on this box (no Vulkan driver, Win32 host code).

Other measurements (not the driver's line):
    python bench.py --codec    the nine encoder / decoder passes at 960x540 (prism_codec_pass),
                               frames/s, e2e through page-locked host memory
    python bench.py --dropin   one MoE block through the per-pass drop-ins (the reference's
                               per-dispatch loop) against prism_moe_block on the same arenas
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from prism_inference_b200 import configs, synth  # noqa: E402
from prism_inference_b200.abi import KERNEL_KINDS  # noqa: E402

METRIC = "MoE-stack tokens/s at 68x120 tokens (64 experts x 16 blocks, dim 256)"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--config", default="moe64x16", choices=configs.ALL)
    p.add_argument("--frames", type=int, default=64, help="frames per GPU per step")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--codec", action="store_true",
                   help="the encoder / decoder passes around the stack at the reference's 960x540 render size "
                        "(prism_codec_pass) instead of the stack")
    p.add_argument("--dropin", action="store_true",
                   help="one MoE block through the per-pass drop-ins (the reference's per-dispatch loop) "
                        "against prism_moe_block on the same arenas")
    return p.parse_args()


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ---------------------------------------------------------------- clocks ----
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms; the figures reported are
    the samples taken between mark() and stop() (the timed regions)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def wait_first(self, timeout=15.0):
        """Block until the first sample has arrived (nvidia-smi can take a while to start)."""
        t0 = time.time()
        while self.proc and not self.rows and time.time() - t0 < timeout:
            time.sleep(0.05)

    def mark(self) -> int:
        return len(self.rows)

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) == 9:
                self.rows.append(parts)

    def stop(self, first: int = 0):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        sm = []
        smax = None
        rows = self.rows[first:]
        in_region = len(rows)
        if not rows:  # a region shorter than the sampling period: the nearest sample after it
            rows = self.rows[-1:]
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
            except ValueError:
                continue
            for i, n in enumerate(names):
                if r[5 + i].lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": in_region}


# ---------------------------------------------------------------- flops ------
def kind_flops_per_frame(L, kind):
    """Algorithmic FLOPs of one kernel kind for one frame (valid tokens only)."""
    T, D = L.tokens, L.dim
    moe = [b for b in L.blocks if b.kind == "moe"]
    dense = [b for b in L.blocks if b.kind == "dense"]
    if kind == "attn":
        # QKV, QK^T and PV over 64 keys, out-projection; on the tensor-core path (dim 256) the
        # MoE router GEMM runs inside the attention launch of each MoE block, so the mean
        # launch carries the router FLOPs of the MoE blocks spread over all attention launches
        f = T * (2.0 * 4 * D * D + 2.0 * 2 * 64 * D)
        if moe and D == 256:
            f += T * 2.0 * sum(b.n_experts for b in moe) * D / len(L.blocks)
        return f
    if kind == "router":  # the separate CUDA-core router (dim 128 only)
        return T * 2.0 * moe[0].n_experts * D if moe and D != 256 else 0.0
    if kind == "expert":
        return T * 2.0 * 2 * D * D
    if kind == "dense_ffn":
        return T * 2.0 * 2 * D * dense[0].ffn_hidden if dense else 0.0
    if kind in ("proj_up", "proj_down"):
        return T * 2.0 * 128 * 256
    return 0.0


def batch1_bytes(L, experts_touched):
    """Algorithmic DRAM bytes of one frame through the stack: every weight and bias the frame
    touches once (attention, router and adapter weights; of the experts, those that received
    at least one token, per MoE block) plus the frame in and the result out, fp16."""
    D, T = L.dim, L.tokens
    n = 0
    if L.up_w >= 0:
        n += 256 * 128 + 256
    if L.down_w >= 0:
        n += 128 * 256 + 128
    moe = iter(experts_touched)
    for b in L.blocks:
        n += 3 * D * D + 3 * D + D * D + D
        if b.kind == "moe":
            n += b.n_experts * D + b.n_experts + next(moe) * (2 * D * D + 2 * D)
        else:
            n += 2 * D * b.ffn_hidden + b.ffn_hidden + D
    return 2 * (n + T * L.in_dim + T * L.out_dim)


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("bf16_tflops_sustained", 1401.2), d.get("hbm_gbs", 6450.0), "measured"
    return 1400.0, 6650.0, "fallback"


def load_traffic(kind, frames):
    """DRAM bytes (read + write) per launch of a kernel kind: the committed ncu capture's
    bytes per frame times the frames one launch processes, or None without a capture."""
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        e = json.loads(p.read_text()).get(kind)
        if e:
            return e["dram_bytes_per_frame"] * frames
    return None


# ---------------------------------------------------------------- cpu -------
def reference_cpu_forward(L, blob, x, n_blocks=None):
    """The reference's own shader sources (oracle/_ref) over frames x, dispatched in the
    order of prism_moe_bench.cpp:408-444.  The router shader computes 4 logits
    (moe_router.comp.glsl:33-37), so it is dispatched with n_experts = min(N, 4) as the
    bench effectively runs it; the N expert dispatches each scan every token."""
    from oracle import GlslRef
    ref = GlslRef()
    T = L.tokens
    blocks = L.blocks[: n_blocks or len(L.blocks)]
    F = x.shape[0]
    feat = np.zeros(T * (128 + 3 * 256 + 128), np.float16)
    aux = np.zeros(T + 256, np.int32)
    A, B, Y, O = T * 128, T * 384, T * 640, T * 896
    n_wg = (T + 255) // 256
    n_win = ((L.spatial_w + 7) // 8) * ((L.spatial_h + 7) // 8)
    t0 = time.perf_counter()
    for f in range(F):
        feat[:T * 128] = x[f].reshape(-1)
        ref.dispatch("pw_project_128to256", [T, L.up_w, L.up_b, 0, A], blob, feat, None, n_wg)
        ci, co = A, B
        for b in blocks:
            ref.dispatch("split2_qkv_attn_d256", [T, 256, 8, 32, L.spatial_w, L.spatial_h, 8, b.qkv_w, b.qkv_b,
                                                  b.out_w, b.out_b, ci, Y], blob, feat, None, n_win)
            ref.dispatch("moe_router", [T, 256, min(4, b.n_experts), b.router_w, b.router_b, Y, 0, T], blob, feat,
                         aux, n_wg)
            for e in range(b.n_experts):
                eo = e * b.expert_stride
                ref.dispatch("moe_expert_skip", [T, 256, e, b.expert_w1 + eo, b.expert_b1 + eo, b.expert_w2 + eo,
                                                 b.expert_b2 + eo, Y, co, 0], blob, feat, aux, n_wg)
            ci, co = co, ci
        ref.dispatch("pw_project_256to128", [T, L.down_w, L.down_b, ci, O], blob, feat, None, n_wg)
    return time.perf_counter() - t0


def cpu_baseline(cfg, blob, min_seconds=10.0):
    """Whole frames of the full stack through the reference shader sources on all host
    cores, one frame at a time until at least min_seconds of CPU work were timed."""
    from oracle import REF_LIB, use_host_threads
    L = cfg.layout
    threads = use_host_threads()
    total, frames = 0.0, 0
    while total < min_seconds and frames < 16:
        x = synth.make_frames(L, 1, first=frames)
        if REF_LIB.exists():
            total += reference_cpu_forward(L, blob, x)
            kind = "reference"
        else:
            from oracle import Oracle
            o = Oracle()
            t0 = time.perf_counter()
            o.stack(L, blob, x)
            total += time.perf_counter() - t0
            kind = "port"
        frames += 1
    return {"value": frames * L.tokens / total, "unit": "tokens/s", "cores": threads, "kind": kind,
            "sample": f"{frames} frames x {len(L.blocks)} blocks of {cfg.key} ({total:.1f} s)"}


def run_reference(args):
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    cfg = configs.get(args.config)
    L = cfg.layout
    from oracle import REF_LIB, use_host_threads
    if not REF_LIB.exists():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref (the reference shader sources "
                          "compiled for the host) is not built"}))
        return
    threads = use_host_threads()  # all host cores, also under torchrun (OMP_NUM_THREADS=1)
    blob = synth.make_blob(L, router_skew=cfg.router_skew, skew_bias=cfg.skew_bias)
    x = synth.make_frames(L, 1)
    # a step is one whole frame through the whole stack (~3.3 s for config 4 on 16 host cores), so
    # the timed region is what the line reports, with nothing extrapolated
    nb = len(L.blocks)
    for _ in range(args.warmup):
        reference_cpu_forward(L, blob, x, nb)
    times = [reference_cpu_forward(L, blob, x, nb) for _ in range(args.steps)]
    dt = sum(times) / len(times)
    value = L.tokens / dt
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": f"{cfg.key}: {cfg.description}, 1 frame per step",
                       "frames_per_step": 1},
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "reference",
                             "sample": f"1 frame x all {nb} blocks (+ adapters) per step"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


# ---------------------------------------------------------------- ours ------
def run_ours(args):
    import torch
    import torch.distributed as dist
    from prism_inference_b200 import Prism, Stack

    ws, rank, local = dist_env()
    if ws > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta
        # NCCL may print a version banner on stdout while the communicator comes up; send it to
        # stderr so that stdout carries only the JSON line
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
            dist.barrier()
            torch.cuda.synchronize()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    dev = torch.cuda.current_device()
    cfg = configs.get(args.config)
    L = cfg.layout
    B = args.frames
    T = L.tokens
    blob = synth.make_blob(L, router_skew=cfg.router_skew, skew_bias=cfg.skew_bias)
    ctx = Prism(dev)
    st = Stack(ctx, L, blob, B)
    # each rank runs its own frames (seeded by global frame index)
    x_host = synth.make_frames(L, B, first=rank * B)
    x = torch.from_numpy(x_host.view(np.int16)).cuda().view(torch.float16)
    out = torch.empty((B, T, L.out_dim), dtype=torch.float16, device="cuda")
    stream = torch.cuda.current_stream()

    def barrier():
        if ws > 1:
            dist.barrier()

    def max_over_ranks(v):
        if ws == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- warm-up
    for _ in range(args.warmup):
        st.forward(x, out)
    torch.cuda.synchronize()
    st.status()

    # ---- timed region (device-resident inputs); per-kernel events on the same stream
    clocks = ClockSampler(dev)
    clocks.start()
    clocks.wait_first()
    st.profile(True)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clock_mark = clocks.mark()
    e0.record(stream)
    for _ in range(args.steps):
        st.forward(x, out)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = e0.elapsed_time(e1) / args.steps
    prof = st.profile_read()
    st.profile(False)
    ms = max_over_ranks(ms)
    st.status()
    launches = st.launch_count(B) * args.steps

    # ---- end to end through the C ABI with host buffers: every step, prism_stack_submit
    # uploads the step's frames from page-locked host memory, runs the stack on `stream` and
    # downloads the output into host memory.  The library's two staging slots overlap step i's
    # upload and step i-1's download with the forward in between, as a serving loop runs;
    # prism_stack_wait makes `stream` wait on the device for the last download.
    ref_out = out.cpu()  # the device-resident result of the same frames
    xh = torch.from_numpy(x_host.view(np.int16)).view(torch.float16).pin_memory()
    oh = [torch.empty((B, T, L.out_dim), dtype=torch.float16).pin_memory() for _ in range(2)]

    def e2e_steps(n):
        t = None
        for i in range(n):
            t = st.submit(xh, oh[i & 1], stream)
        st.wait(t, stream, host=False)

    e2e_steps(2)
    torch.cuda.synchronize()
    barrier()
    e0.record(stream)
    e0.synchronize()  # the start is stamped before the first upload is queued
    e2e_steps(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms_e2e = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    clk = clocks.stop(clock_mark)  # samples over both timed regions
    st.status()
    oh = oh[(args.steps - 1) & 1]
    if not torch.equal(oh.view(torch.int16), ref_out.view(torch.int16)):
        raise SystemExit("bench: the end-to-end output differs from the device-resident output")
    del ref_out

    # ---- batch-1 latency (one frame through the whole stack)
    x1, o1 = x[:1], out[:1]
    for _ in range(3):
        st.forward(x1, o1)
    torch.cuda.synchronize()
    e0.record(stream)
    n1 = max(10, args.steps)
    for _ in range(n1):
        st.forward(x1, o1)
    e1.record(stream)
    torch.cuda.synchronize()
    ms_b1 = max_over_ranks(e0.elapsed_time(e1) / n1)
    st.status()

    # ---- the same frame, the whole stack replayed as one CUDA graph (prism_stack_forward
    # is stream-ordered without host synchronisation, so it can be captured)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        st.forward(x1, o1)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(n1):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms_b1_graph = max_over_ranks(e0.elapsed_time(e1) / n1)
    del g
    st.status()
    # the same graph with the attention tiles on one CTA each (PRISM_OPT_PAIR_ATTENTION off):
    # what the CTA-pair latency path gains at batch 1
    st.set_pair_attention(False)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        st.forward(x1, o1)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(n1):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms_b1_graph_one_cta = max_over_ranks(e0.elapsed_time(e1) / n1)
    del g
    st.set_pair_attention(True)
    st.status()
    # batch 1 is bound by streaming the weights the frame touches from HBM
    asg1 = torch.empty((max(1, L.n_moe_blocks), T), dtype=torch.int32, device="cuda")
    st.forward(x1, o1, asg1 if L.n_moe_blocks else None)
    torch.cuda.synchronize()
    touched = [int(np.unique(a).size) for a in asg1.cpu().numpy()[:L.n_moe_blocks]]
    b1_bytes = batch1_bytes(L, touched)
    b1_gbs = b1_bytes / (ms_b1_graph / 1e3) / 1e9

    # ---- N > 1: the sharded output collected on rank 0 (NCCL over NVLink), timed apart
    # from the compute (the frames are independent: this is the only exchange)
    gather = None
    if ws > 1:
        recv = [torch.empty_like(out) for _ in range(ws)] if rank == 0 else None
        for _ in range(2):
            dist.gather(out, recv, dst=0)
        torch.cuda.synchronize()
        barrier()
        e0.record(stream)
        dist.gather(out, recv, dst=0)
        e1.record(stream)
        torch.cuda.synchronize()
        gms = max_over_ranks(e0.elapsed_time(e1))
        nbytes = out.numel() * out.element_size() * (ws - 1)
        gather = {"ms": gms, "bytes_to_rank0": nbytes, "GB_per_s": nbytes / (gms / 1e3) / 1e9}
        del recv

    tokens_per_step = B * T * ws
    value = tokens_per_step / (ms / 1e3)
    e2e = tokens_per_step / (ms_e2e / 1e3)

    # ---- roofline of the dominant kernel kind
    peak_tf, peak_gbs, peak_src = load_peaks()
    b1_roof = {"bound": "hbm", "achieved": b1_gbs, "peak": peak_gbs, "unit": "GB/s", "frac": b1_gbs / peak_gbs,
               "peak_source": f"{peak_src} hbm_gbs", "bytes_per_frame": b1_bytes,
               "experts_touched_per_block": statistics.mean(touched) if touched else 0,
               "time": "batch1_graph_ms"}
    roof = None
    if prof:
        kind = max(prof, key=lambda k: prof[k][0])
        tot_ms, n = prof[kind]
        per_launch_ms = tot_ms / n
        fl = kind_flops_per_frame(L, kind) * B
        achieved = fl / (per_launch_ms / 1e3) / 1e12
        roof = {"kernel": kind, "bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                "frac": achieved / peak_tf, "peak_source": f"{peak_src} bf16_tflops_sustained",
                "traffic": load_traffic(kind, B), "traffic_source": "profiles/traffic.json (ncu, scaled by frames)",
                "ms_per_launch": per_launch_ms,
                "share": tot_ms / (ms * args.steps)}
    kernel_ms = {k: round(v[0] / args.steps, 4) for k, v in prof.items()}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(cfg, blob)

    if rank == 0:
        flops_step = configs.flops_per_frame(L) * B * ws
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f16", "data": "synthetic",
                "config": {"workload": f"{cfg.key}: {cfg.description}", "frames_per_gpu": B,
                           "tokens_per_frame": T, "seq_len": T, "global_batch": B * ws,
                           "parallelism": f"frame-sharded x{ws}, weights replicated",
                           "l2": "inputs/activations larger than L2 (134 MB in, 267 MB per activation buffer)",
                           "frames_per_s": B * ws / (ms / 1e3), "batch1_ms": ms_b1, "batch1_graph_ms": ms_b1_graph,
                           "batch1_graph_ms_one_cta_attention": ms_b1_graph_one_cta,
                           "batch1_roofline": b1_roof,
                           "output_gather": gather,
                           "tflops_effective": flops_step / (ms / 1e3) / 1e12,
                           "kernel_ms_per_step": kernel_ms},
                "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": int(xh.numel() * 2),
                        "d2h_bytes_per_step": int(oh.numel() * 2), "ms_per_step": ms_e2e,
                        "api": "prism_stack_submit / prism_stack_wait (C ABI, host buffers)",
                        "overlap": "upload, forward and download of neighbouring steps on three streams, "
                                   "two device staging slots inside the library"},
                "gpu_launches": launches, "roofline": roof, "cpu_baseline": cpu, "clocks": clk}
        print(json.dumps(line))
    st.close()
    ctx.close()
    if ws > 1:
        dist.destroy_process_group()


# ---------------------------------------------------------------- codec -----
def codec_cpu_baseline(fc, blob, feat, min_seconds=5.0):
    """The reference's own encoder / decoder shader sources (oracle/_ref) for whole frames on all
    host cores, until at least min_seconds of CPU work were timed."""
    from oracle import REF_LIB, GlslRef, use_host_threads
    if not REF_LIB.exists():
        return None
    ref = GlslRef()
    threads = use_host_threads()
    total, frames = 0.0, 0
    f = feat.copy()
    rgb = np.zeros(fc.rgb_elems, np.float16)
    while total < min_seconds and frames < 8:
        t0 = time.perf_counter()
        for shader, push, _ in fc.passes:
            if shader.startswith("strided"):
                px = push[4] * push[5]
            elif shader.startswith("dec"):
                px = push[0] * push[1]
            else:
                px = push[2] * push[3]
            ref.dispatch(shader, push, blob, f, None, (px + 255) // 256)
        ps = fc.pixelshuffle
        ref.dispatch("pixelshuffle_sigmoid", ps, blob, f, rgb, ((ps[2] + 15) // 16, (ps[3] + 15) // 16))
        total += time.perf_counter() - t0
        frames += 1
    return {"value": frames / total, "unit": "frames/s", "cores": threads, "kind": "reference",
            "sample": f"{frames} frames of the 9 encoder / decoder shaders at {fc.render[0]}x{fc.render[1]} ({total:.1f} s)"}


def run_codec(args):
    """One step = one frame through the nine encoder / decoder passes (prism_codec_pass each) at
    the reference's 960x540 render size; every rank runs its own frame (weak scaling).  value: the
    chain replayed as one CUDA graph (device time); per-pass times: CUDA events around each
    eager call."""
    import torch
    import torch.distributed as dist
    from prism_inference_b200 import Prism, codec
    ws, rank, local = dist_env()
    if ws > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.cuda.current_device()
    fc = codec.frame_chain(960, 540)
    blob, feat = codec.synthetic(fc, seed=0x5EED + rank)
    ctx = Prism(dev)
    w = torch.from_numpy(blob.view(np.int16)).cuda().view(torch.float16)
    f = torch.from_numpy(feat.view(np.int16)).cuda().view(torch.float16)
    rgb = torch.zeros(fc.rgb_elems, dtype=torch.float16, device="cuda")
    names = [p[0] for p in fc.passes] + ["pixelshuffle_sigmoid"]
    pushes = [p[1] for p in fc.passes] + [fc.pixelshuffle]
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)]

    def frame(timed=False, fb=None, rb=None):
        stream = torch.cuda.current_stream()
        fb = f if fb is None else fb
        rb = rgb if rb is None else rb
        for i, (sh, pc) in enumerate(zip(names, pushes)):
            if timed:
                ev[i].record(stream)
            ctx.codec_pass(sh, pc, w, fb, rb if sh == "pixelshuffle_sigmoid" else None, stream)
        if timed:
            ev[-1].record(stream)

    for _ in range(args.warmup):
        frame()
    torch.cuda.synchronize()
    ctx.status()
    stream = torch.cuda.current_stream()
    per = np.zeros(len(names))
    for _ in range(args.steps):
        torch.cuda.synchronize()
        frame(timed=True)
        torch.cuda.synchronize()
        per += np.array([ev[i].elapsed_time(ev[i + 1]) for i in range(len(names))])
    per /= args.steps
    # the whole frame as one CUDA graph (no host work between the launches)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        frame()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        frame()
    for _ in range(3):
        g.replay()
    clocks = ClockSampler(dev)
    clocks.start()
    clocks.wait_first()
    mark = clocks.mark()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    # end to end, as a serving loop runs it: every step uploads its frame from page-locked host
    # memory into one of two device frame slots, replays the chain there and downloads its RGB,
    # with the upload of the next frame and the download of the previous one on their own
    # streams (the copies cross PCIe in both directions while the chain runs)
    o, n = fc.feat_off["in"], fc.feat_size["in"]
    xin = torch.from_numpy(feat[o:o + n].view(np.int16)).view(torch.float16).pin_memory()
    rgb_h = [torch.empty(fc.rgb_elems, dtype=torch.float16).pin_memory() for _ in range(2)]
    slots = [(f, rgb), (f.clone(), torch.zeros_like(rgb))]
    graphs = [g]
    with torch.cuda.stream(side):
        frame(fb=slots[1][0], rb=slots[1][1])
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g1 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g1):
        frame(fb=slots[1][0], rb=slots[1][1])
    graphs.append(g1)
    up, comp, down = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    uploaded = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]
    downloaded = [torch.cuda.Event() for _ in range(2)]
    steps_e2e = max(args.steps, 20)
    torch.cuda.synchronize()
    e0.record(stream)
    for st_ in (up, comp, down):
        st_.wait_stream(stream)
    for i in range(steps_e2e):
        sl = i % 2
        fb, rb = slots[sl]
        with torch.cuda.stream(up):
            if i >= 2:
                up.wait_event(computed[sl])  # the chain of two steps ago has read this slot's input
            fb[o:o + n].copy_(xin, non_blocking=True)
            uploaded[sl].record(up)
        with torch.cuda.stream(comp):
            comp.wait_event(uploaded[sl])
            if i >= 2:
                comp.wait_event(downloaded[sl])  # this slot's RGB of two steps ago is home
            graphs[sl].replay()
            computed[sl].record(comp)
        with torch.cuda.stream(down):
            down.wait_event(computed[sl])
            rgb_h[sl].copy_(rb, non_blocking=True)
            downloaded[sl].record(down)
    for st_ in (up, comp, down):
        stream.wait_stream(st_)
    e1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1) / steps_e2e
    if not torch.equal(rgb_h[(steps_e2e - 1) % 2].view(torch.int16), rgb.cpu().view(torch.int16)):
        raise RuntimeError("codec e2e: the downloaded RGB differs from the device-resident chain's")
    clk = clocks.stop(mark)
    del g, g1, graphs
    ctx.status()
    if ws > 1:
        t = torch.tensor([ms, ms_e2e], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_e2e = float(t[0]), float(t[1])
    peak_tf, peak_gbs, src = load_peaks()
    rows = {}
    for i, sh in enumerate(names):
        b, fl = fc.pass_bytes_flops(sh)
        rows[sh] = {"ms_eager": round(float(per[i]), 5), "GB_per_s": round(b / (per[i] / 1e3) / 1e9, 1),
                    "TFLOP_per_s": round(fl / (per[i] / 1e3) / 1e12, 1)}
    total_bytes = sum(fc.pass_bytes_flops(s)[0] for s in names)
    achieved = total_bytes / (ms / 1e3) / 1e9
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = codec_cpu_baseline(fc, blob, feat)
    if rank == 0:
        line = {"metric": "encoder/decoder frames/s at 960x540 render (9 passes, 1080p RGB out)",
                "value": ws * 1e3 / ms, "unit": "frames/s", "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f16", "data": "synthetic",
                "config": {"workload": "encoder/decoder of prism_moe_bench.cpp:386-471 at 960x540 (the stack left out)",
                           "frames_per_gpu": 1, "passes_eager": rows, "algorithmic_bytes_per_frame": total_bytes,
                           "l2": "maps of one frame total 140 MB; a pass reads the previous pass's output"},
                "e2e": {"value": ws * 1e3 / ms_e2e, "unit": "frames/s", "h2d_bytes_per_step": int(xin.numel() * 2),
                        "d2h_bytes_per_step": int(rgb_h[0].numel() * 2), "ms_per_step": ms_e2e, "steps": steps_e2e,
                        "api": "prism_codec_pass per pass (graph replay); frame in / RGB out through page-locked host memory",
                        "overlap": "upload, chain and download of neighbouring steps on three streams, two device frame slots"},
                # a pass kernel each, a weight repack before each pass whose matrix streams (over
                # 64 KB: the two split convolutions), the pixel shuffle
                "gpu_launches": len(fc.passes) + sum(p[0].startswith("strided_conv_split") for p in fc.passes) + 1,
                "roofline": {"kernel": "whole chain", "bound": "hbm", "achieved": achieved, "peak": peak_gbs,
                             "unit": "GB/s", "frac": achieved / peak_gbs, "peak_source": f"{src} hbm_gbs",
                             "traffic": None},
                "cpu_baseline": cpu, "clocks": clk}
        print(json.dumps(line))
    ctx.close()
    if ws > 1:
        dist.destroy_process_group()


def run_dropin(args):
    """One MoE block of the headline configuration (dim 256, 64 experts) on one 120x68 frame, as a
    host keeping the reference's per-dispatch loop runs it (prism_moe_bench.cpp:416-437: attention,
    the router, one expert dispatch per expert, through prism_attn_window / prism_router /
    prism_expert on the reference's arenas), against prism_moe_block on the same arenas (the tcgen05
    path).  Both as replayed CUDA graphs (device time, no host launch cost); the outputs are
    compared.  1 GPU; not part of the driver's contract."""
    import torch
    from prism_inference_b200 import Prism, Stack, layout, synth
    from prism_inference_b200.abi import AttnParams, ExpertParams, RouterParams
    ctx = Prism(0)
    L = layout.build_stack(256, 1, n_experts=64)
    T, D, E = L.tokens, 256, 64
    b = L.blocks[0]
    blob = synth.make_blob(L)
    x = synth.make_frames(L, 1)[0]
    w = torch.from_numpy(blob.view(np.int16)).cuda().view(torch.float16)
    feat = torch.zeros(3 * T * D, dtype=torch.float16, device="cuda")
    feat[:T * D] = torch.from_numpy(x.reshape(-1).view(np.int16)).cuda().view(torch.float16)
    aux = torch.zeros(T + E, dtype=torch.int32, device="cuda")
    pa = AttnParams(T, D, 8, 32, L.spatial_w, L.spatial_h, 8, b.qkv_w, b.qkv_b, b.out_w, b.out_b, 0, T * D)
    pr = RouterParams(T, D, E, b.router_w, b.router_b, T * D, 0, T)
    pe = [ExpertParams(T, D, e, b.expert_w1 + e * b.expert_stride, b.expert_b1 + e * b.expert_stride,
                       b.expert_w2 + e * b.expert_stride, b.expert_b2 + e * b.expert_stride, T * D, 2 * T * D, 0)
          for e in range(E)]
    blk = Stack(ctx, L, blob, 1)
    fast_out = torch.zeros(T * D, dtype=torch.float16, device="cuda")
    fast_aux = torch.zeros(T + E, dtype=torch.int32, device="cuda")

    def dropin():
        ctx.attn_window(pa, w, feat)
        ctx.router(pr, w, feat, aux)
        for p_ in pe:
            ctx.expert(p_, w, feat, aux)

    def dropin_static():  # the experts as one allocation-free call (prism_expert_all_static)
        ctx.attn_window(pa, w, feat)
        ctx.router(pr, w, feat, aux)
        ctx.expert_all_static(pe[0], E, b.expert_stride, w, feat, aux)

    def fast():
        blk.moe_block(feat[:T * D].view(1, T, D), fast_out.view(1, T, D), fast_aux[:T], fast_aux[T:])

    def timed(fn):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        for _ in range(max(args.warmup, 3)):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        del g
        return e0.elapsed_time(e1) / args.steps

    ms_static = timed(dropin_static)
    ms_dropin = timed(dropin)
    ms_fast = timed(fast)
    ctx.status()
    blk.status()
    a = feat[2 * T * D:].float()
    f = fast_out.float()
    diff = (a - f).abs().max().item()
    rel = ((a - f).norm() / f.norm()).item()
    same_route = float((aux[:T] == fast_aux[:T]).float().mean().item())
    print(json.dumps({"metric": "one MoE block (dim 256, 64 experts) on one 120x68 frame: per-pass drop-ins vs "
                                "prism_moe_block", "unit": "ms",
                      "dropin_ms": ms_dropin, "dropin_launches": 2 + E, "dropin_static_experts_ms": ms_static,
                      "moe_block_ms": ms_fast,
                      "speedup": ms_dropin / ms_fast, "max_abs_diff": diff, "rel_l2_diff": rel,
                      "routing_agreement": same_route, "steps": args.steps, "data": "synthetic"}))
    blk.close()
    ctx.close()


def main():
    args = parse()
    if args.dropin:
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "--dropin measures this library only"}))
            return
        run_dropin(args)
        return
    if args.codec:
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "--codec measures this library only"}))
            return
        run_codec(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

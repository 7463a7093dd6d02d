"""Frame sharding (the multi-GPU data path) on CPU: the plan, and world-size-2 gloo
ranks that each run the oracle on their own frames and gather - the result must equal
a single-process run; a rank that fails must surface as an error on the other rank."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from prism_inference_b200 import shard


def test_plan_covers_every_frame_once():
    for total in (0, 1, 7, 64, 65, 512):
        for ws in (1, 2, 3, 4, 8):
            p = shard.plan(total, ws)
            assert sum(n for _, n in p) == total
            assert [s for s, _ in p] == list(np.cumsum([0] + [n for _, n in p])[:-1])
            assert max(n for _, n in p) - min(n for _, n in p) <= 1
    with pytest.raises(ValueError):
        shard.plan(4, 0)
    with pytest.raises(ValueError):
        shard.my_frames(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, ws, port, total, out_path, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=timedelta(seconds=20))
    try:
        from oracle import Oracle
        from prism_inference_b200 import layout, synth
        L = layout.build_stack(256, 1, n_experts=4, spatial_w=16, spatial_h=8)
        blob = synth.make_blob(L)
        first, n = shard.my_frames(total, ws, rank)
        if rank == fail_rank:
            raise RuntimeError("rank failure injected on the host")
        x = synth.make_frames(L, n, first=first)
        out, _, _ = Oracle().stack(L, blob, x)
        full = shard.gather_frames(torch.from_numpy(out.view(np.int16)), total, ws)
        if rank == 0:
            np.save(out_path, full.numpy())
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_two_rank_frame_shard_equals_single_process(tmp_path):
    from oracle import Oracle
    from prism_inference_b200 import layout, synth
    total = 5
    out_path = str(tmp_path / "gathered.npy")
    mp.start_processes(_worker, args=(2, _free_port(), total, out_path, -1), nprocs=2, join=True,
                       start_method="spawn")
    got = np.load(out_path).view(np.float16)
    L = layout.build_stack(256, 1, n_experts=4, spatial_w=16, spatial_h=8)
    ref, _, _ = Oracle().stack(L, synth.make_blob(L), synth.make_frames(L, total))
    assert (got.view(np.uint16) == ref.view(np.uint16)).all()


def test_failed_rank_is_reported(tmp_path):
    out_path = str(tmp_path / "never.npy")
    with pytest.raises(Exception):
        mp.start_processes(_worker, args=(2, _free_port(), 4, out_path, 1), nprocs=2, join=True,
                           start_method="spawn")
    assert not os.path.exists(out_path)

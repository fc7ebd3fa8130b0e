"""Multi-process path on CPU (gloo, world size 2): each rank solves its shard of
utterances (here with the CPU oracle standing in for the engine), shards are
gathered in rank order and equal the single-process result exactly; the timer
reduction is a max over ranks."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import shard


def test_shard_ranges_cover_and_balance():
    for n in (0, 1, 7, 64, 2048):
        for world in (1, 2, 3, 4, 8):
            rs = [shard.shard_range(n, world, r) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == n
            assert all(rs[i][1] == rs[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in rs]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard.shard_range(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path.insert(0, os.path.join(root, "dots.tts.cpp_b200"))
    sys.path.insert(0, os.path.join(root, "oracle"))
    import torch
    import torch.distributed as dist
    import oracle as O
    import synth
    import shard as S
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    orc = O.Oracle()
    orc.set_threads(1)
    w = synth.dit_weights(3, n_layers=1)
    n_total = 5
    fc, fu = synth.fm_history(3, n_total, 4, w)
    z0 = synth.normal(3, "z0", (n_total, 4, 128), 1.0)
    a, b = S.shard_range(n_total, world, rank)
    z = orc.euler_solve(w, 1, fc[a:b], fu[a:b], z0[a:b], nfe=2, cfg_scale=2.0)
    parts = [None] * world
    dist.all_gather_object(parts, z)
    t = S.max_over_ranks(float(rank + 1), dist)
    if rank == 0:
        np.save(os.path.join(out_dir, "gathered.npy"), np.concatenate(parts))
        np.save(os.path.join(out_dir, "tmax.npy"), np.array([t]))
    dist.barrier()
    dist.destroy_process_group()


def test_gloo_two_ranks_equal_single_process(tmp_path, orc):
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    import synth
    w = synth.dit_weights(3, n_layers=1)
    fc, fu = synth.fm_history(3, 5, 4, w)
    z0 = synth.normal(3, "z0", (5, 4, 128), 1.0)
    full = orc.euler_solve(w, 1, fc, fu, z0, nfe=2, cfg_scale=2.0)
    got = np.load(tmp_path / "gathered.npy")
    assert np.array_equal(got, full)
    assert float(np.load(tmp_path / "tmax.npy")[0]) == 2.0

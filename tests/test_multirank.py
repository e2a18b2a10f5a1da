"""Window sharding across ranks (the N>1 path), on CPU with gloo ranks.

Each rank takes its LPT share of a layer's windows (s2b200.shard_windows),
computes those windows with the oracle, and the ranks all-reduce their text
partial sums -- the one exchange of the sharded path. The result must equal
the single-rank layer: video rows exactly (every token has one owner), text
within fp32 summation-order rounding.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import s2b200
from s2b200 import synth

GRID, HEADS, LT = (3, 12, 20), 2, 7


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, shifted, out_dir):
    import oracle  # spawned process: import here
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        vid, txt, gam, fr = synth.layer_inputs(GRID, heads=HEADS, text_len=LT, seed=21)
        wins = s2b200.make_windows(*GRID, shifted)
        ids = s2b200.shard_windows(wins, LT, world)[rank]
        mask = np.zeros(len(wins), np.uint8)
        mask[ids] = 1
        vo, to, _ = oracle.port().window_attention(vid, txt, GRID, HEADS, list(gam), fr, shifted,
                                                   window_mask=mask, threads=1)
        v = torch.from_numpy(vo)
        t = torch.from_numpy(to)
        dist.all_reduce(v)   # disjoint rows: the sum is the union
        dist.all_reduce(t)   # text partials, each already scaled by 1/total windows
        if rank == 0:
            np.save(os.path.join(out_dir, f"vid_{shifted}.npy"), v.numpy())
            np.save(os.path.join(out_dir, f"txt_{shifted}.npy"), t.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shifted", [0, 1])
def test_two_gloo_ranks_reproduce_the_single_rank_layer(tmp_path, port, shifted):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), shifted, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    vid, txt, gam, fr = synth.layer_inputs(GRID, heads=HEADS, text_len=LT, seed=21)
    ref_v, ref_t, _ = port.window_attention(vid, txt, GRID, HEADS, list(gam), fr, shifted, threads=1)
    got_v = np.load(tmp_path / f"vid_{shifted}.npy")
    got_t = np.load(tmp_path / f"txt_{shifted}.npy")
    assert np.array_equal(got_v, ref_v)
    np.testing.assert_allclose(got_t, ref_t, rtol=0, atol=1e-6)


@pytest.mark.parametrize("grid,shifted,n", [((6, 45, 80), 0, 8), ((6, 45, 80), 1, 8), ((12, 67, 120), 1, 4),
                                            ((2, 16, 30), 1, 2)])
def test_shard_windows_partitions_and_balances(grid, shifted, n):
    wins = s2b200.make_windows(*grid, shifted)
    parts = s2b200.shard_windows(wins, 58, n)
    allids = np.sort(np.concatenate(parts))
    assert np.array_equal(allids, np.arange(len(wins)))
    cost = s2b200.window_costs(wins, 58)
    loads = np.array([cost[p].sum() for p in parts])
    # LPT bound: no rank exceeds the mean by more than the largest single window
    assert loads.max() <= loads.mean() + cost.max() + 1e-9
    assert s2b200.shard_windows(wins, 58, n)[0].tolist() == parts[0].tolist()  # deterministic


@pytest.mark.parametrize("grid,shifted,n", [((6, 45, 80), 0, 2), ((6, 45, 80), 1, 8), ((12, 67, 120), 1, 4),
                                            ((2, 16, 30), 0, 3)])
def test_library_sharding_matches_python_lpt(grid, shifted, n):
    """The library's ownership (used by the sharded DiT step) is the same LPT
    assignment as the Python helper used by the layer-level sharding."""
    wins = s2b200.make_windows(*grid, shifted)
    owner = s2b200.shard_owners(wins, 58, n)
    parts = s2b200.shard_windows(wins, 58, n)
    for r in range(n):
        assert np.nonzero(owner == r)[0].tolist() == parts[r].tolist()

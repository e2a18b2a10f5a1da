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


# ---- the sharded DiT step's row exchange (plain <-> shifted ownership) -------------

def _exchange_rank_main(rank, world, port, grid, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    ok = True
    try:
        for kind in (0, 1):
            m = s2b200.shard_exchange(grid, 58, world, rank, kind)
            nxt = s2b200.shard_exchange(grid, 58, world, rank, 1 - kind)
            # every local row carries its token id; exchange them exactly as the step exchanges hidden rows
            x = torch.from_numpy(m["local_tokens"].astype(np.float64))
            send = x[torch.from_numpy(m["send_rows"]).long()]
            recv = torch.empty(int(m["recv_counts"].sum()), dtype=torch.float64)
            dist.all_to_all_single(recv, send, output_split_sizes=m["recv_counts"].tolist(),
                                   input_split_sizes=m["send_counts"].tolist())
            y = torch.full((len(nxt["local_tokens"]),), -1.0, dtype=torch.float64)
            y[torch.from_numpy(m["recv_rows"]).long()] = recv
            ok &= bool(torch.equal(y, torch.from_numpy(nxt["local_tokens"].astype(np.float64))))
        np.save(os.path.join(out_dir, f"ok_{rank}.npy"), np.array([ok]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_row_exchange_maps_on_gloo_ranks(tmp_path, world):
    """The maps of the sharded Euler step (s2_shard_exchange, the host function
    the GPU path uploads): each gloo rank holds its local rows of one window
    kind (values = token ids), exchanges them with all_to_all_single as the step
    does with hidden rows, and must end with exactly its local rows of the other
    kind in their order -- both directions, 720p grid."""
    grid = (6, 45, 80)
    mp.start_processes(_exchange_rank_main, args=(world, _free_port(), grid, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    for r in range(world):
        assert bool(np.load(tmp_path / f"ok_{r}.npy")[0]), f"rank {r}"


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("grid", [(6, 45, 80), (12, 67, 120), (2, 16, 30)])
def test_shard_local_rows_follow_the_single_rank_order(grid, world):
    """Every rank's local rows are the single-rank packed order (s2_build_varlen:
    window by window, (t, y, x) inside a window) restricted to its windows; the
    ranks' rows partition the grid; the joint ownership keeps every layer kind's
    load within the stated bounds and moves fewer rows than per-kind LPT."""
    T, H, W = grid
    L = T * H * W
    for kind in (0, 1):
        wins = s2b200.make_windows(T, H, W, kind)
        cu, rows = s2b200.build_varlen(T, H, W, wins, 0)
        seen = np.zeros(L, np.int64)
        for r in range(world):
            m = s2b200.shard_exchange(grid, 58, world, r, kind)
            want = np.concatenate([rows[cu[i]:cu[i + 1], 0] for i in m["window_ids"]]) if len(m["window_ids"]) \
                else np.zeros(0, np.int32)
            assert np.array_equal(m["local_tokens"], want), (kind, r)
            seen[m["local_tokens"]] += 1
        assert np.all(seen == 1), "the ranks' rows must partition the grid"
    if world > 1:
        moved = s2b200.shard_exchange(grid, 58, world, 0, 0)["moved_rows"]
        lpt = [s2b200.shard_owners(s2b200.make_windows(T, H, W, k), 58, world) for k in (0, 1)]
        tok = [np.zeros(L, np.int64) for _ in range(2)]
        for k in (0, 1):
            for i, w in enumerate(s2b200.make_windows(T, H, W, k)):
                t = np.arange(w[0], w[1])[:, None, None]
                y = np.arange(w[2], w[3])[None, :, None]
                x = np.arange(w[4], w[5])[None, None, :]
                tok[k][((t * H + y) * W + x).ravel()] = lpt[k][i]
        assert moved <= int((tok[0] != tok[1]).sum()), (moved, int((tok[0] != tok[1]).sum()))
        # the shifted layers' load (video rows + 1e-4 * S_w^2: a block's work) stays within the
        # 2 % cap whenever a rank can take each window
        w1 = s2b200.make_windows(T, H, W, 1)
        rows1 = ((w1[:, 1] - w1[:, 0]) * (w1[:, 3] - w1[:, 2]) * (w1[:, 5] - w1[:, 4])).astype(np.float64)
        cost = rows1 + 1e-4 * (rows1 + 58.0) ** 2
        load = np.array([cost[s2b200.shard_exchange(grid, 58, world, r, 1)["window_ids"]].sum() for r in range(world)])
        assert load.max() <= max(1.02 * cost.sum() / world, cost.max()) * 1.0001


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("grid", [(6, 45, 80), (2, 16, 30)])
def test_row_destinations_cover_every_rank_once(grid, world):
    """The peer-store exchange's per-row destinations (s2_shard_row_destinations):
    every rank's kind-k row goes to the rank holding its token under the other
    kind, at that token's place in that rank's local order, and together the
    ranks fill every destination row exactly once; the rows that leave their
    rank are the grid's moved rows."""
    for kind in (0, 1):
        other = [s2b200.shard_exchange(grid, 58, world, r, 1 - kind)["local_tokens"] for r in range(world)]
        filled = [np.zeros(len(o), np.int64) for o in other]
        moved = 0
        for r in range(world):
            tok = s2b200.shard_exchange(grid, 58, world, r, kind)["local_tokens"]
            dr, dw = s2b200.shard_row_destinations(grid, 58, world, r, kind)
            assert len(dr) == len(tok)
            for i in range(len(tok)):
                assert other[dr[i]][dw[i]] == tok[i], (kind, r, i)
                filled[dr[i]][dw[i]] += 1
            moved += int((dr != r).sum())
        assert all(np.all(f == 1) for f in filled), kind
        assert moved == s2b200.shard_exchange(grid, 58, world, 0, kind)["moved_rows"]

"""The sharded DiT Euler step on 2 and 4 GPUs (one process per GPU, the
library's NCCL communicator): each rank keeps only its windows' video rows,
all-reduces every block's text attention mean, and at every plain <-> shifted
boundary the block's last GEMM stores each row into its next owner's input
buffer (peer memory over NVLink). The result must match the same step on one
GPU (and, on 2 GPUs, the reference). Skipped where the box has too few GPUs.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

import parity
import s2b200
from s2b200 import synth

pytestmark = pytest.mark.gpu

CASE = dict(n_blocks=4, dim=256, heads=2, mlp=256, tc=256, lat=(2, 12, 20), Lt=9)


def _case():
    c = CASE
    flags = [dict(shared=False, shifted=False, last=False), dict(shared=True, shifted=True, last=False),
             dict(shared=False, shifted=False, last=False), dict(shared=True, shifted=True, last=True)]
    wi = synth.dit_input_weights(c["dim"], 33, c["tc"], 256)
    wo = synth.dit_output_weights(c["dim"])
    bws = [synth.block_weights(c["dim"], c["heads"], c["mlp"], flags[i]["shared"], seed=100 + i)
           for i in range(c["n_blocks"])]
    noise, cond, text = synth.dit_latents(c["lat"], 16, c["Lt"], c["tc"])
    return flags, wi, wo, bws, noise, cond, text


def _model(device, flags, wi, wo, bws, windows=(0, 0, 0)):
    c = CASE
    m = s2b200.SeedVR2DiT(device=device, n_blocks=c["n_blocks"], dim=c["dim"], heads=c["heads"],
                          mlp_hidden=c["mlp"], text_channels=c["tc"], window_override=windows)
    m.load_input(wi)
    m.load_output(wo)
    for i, f in enumerate(flags):
        m.load_block(i, bws[i], **f)
    return m


def _rank(rank, world, port, out_dir, windows=(0, 0, 0)):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.cuda.set_device(rank)
    comm = s2b200.Comm.create(rank, rank, world)
    flags, wi, wo, bws, noise, cond, text = _case()
    m = _model(rank, flags, wi, wo, bws, windows)
    m.set_comm(comm)
    args = [torch.from_numpy(a).cuda(rank) for a in (noise, cond, text)]
    x0 = m.euler_step(*args)        # eager
    for _ in range(3):              # captured once (NCCL calls inside the graph), then replayed
        x0b = m.euler_step(*args, x0=torch.empty_like(x0))
    torch.cuda.synchronize()
    assert m.device_error() == 0
    np.save(os.path.join(out_dir, f"x0_{rank}.npy"), x0.cpu().numpy())
    np.save(os.path.join(out_dir, f"x0b_{rank}.npy"), x0b.cpu().numpy())
    m.close()
    comm.close()
    dist.barrier()
    dist.destroy_process_group()


def _rank_mismatch(rank, world, port, out_dir):
    """Each rank steps a grid of its own width: every rank must refuse the step."""
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.cuda.set_device(rank)
    comm = s2b200.Comm.create(rank, rank, world)
    comm.set_timeout(60000)
    flags, wi, wo, bws, _, _, text = _case()
    m = _model(rank, flags, wi, wo, bws)
    m.set_comm(comm)
    T, H, W = CASE["lat"]
    noise, cond, _ = synth.dit_latents((T, H, W + 4 * rank), 16, CASE["Lt"], CASE["tc"])
    status, msg = 0, ""
    try:
        m.euler_step(*(torch.from_numpy(a).cuda(rank) for a in (noise, cond, text)))
    except s2b200.S2Error as e:
        status, msg = e.status, str(e)
    with open(os.path.join(out_dir, f"mismatch_{rank}.txt"), "w") as f:
        f.write(f"{status}\n{msg}\n")
    m.close()
    comm.close()
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_step_refuses_different_grids(tmp_path):
    """Ranks called with different grids would derive different exchange maps:
    the shard set-up gathers every rank's grid and all ranks return
    S2_INVALID_ARGUMENT instead of storing rows where no peer expects them."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    port = 29500 + (os.getpid() + 250) % 1000
    mp.start_processes(_rank_mismatch, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        status, msg = (tmp_path / f"mismatch_{r}.txt").read_text().split("\n", 1)
        assert int(status) == s2b200.S2_INVALID_ARGUMENT, (r, status, msg)
        assert "all ranks must run the same step" in msg, msg


def test_sharded_euler_step_two_gpus(tmp_path, ref):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    port = 29500 + os.getpid() % 1000
    mp.start_processes(_rank, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    flags, wi, wo, bws, noise, cond, text = _case()
    single = _model(0, flags, wi, wo, bws).euler_step_host(noise, cond, text)
    hp = dict(dim=CASE["dim"], text_channels=CASE["tc"], sinusoidal_dim=256, embedding_dim=6 * CASE["dim"],
              out_channels=16, eps=1e-5)
    bps = [dict(block_index=i, dim=CASE["dim"], heads=CASE["heads"], head_dim=128, mlp_hidden=CASE["mlp"], eps=1e-5,
                **f) for i, f in enumerate(flags)]
    ex0, _ = ref.euler_step(hp, wi, bps, bws, wo, noise, cond, text, 1000.0)
    outs = [np.load(tmp_path / f"x0_{r}.npy") for r in range(2)]
    assert np.array_equal(outs[0], outs[1])                  # every rank ends with the full output
    assert np.array_equal(outs[0], np.load(tmp_path / "x0b_0.npy"))
    m = parity.metrics(outs[0], single)
    assert m["max_abs"] <= 1e-4, m                           # only the text sums change order
    p = parity.metrics(noise - outs[0], noise - ex0)
    assert p["nrmse"] <= 0.02 and p["cosine"] >= 0.9998, p


def test_sharded_euler_step_four_gpus(tmp_path):
    """Four ranks, each writing rows to three peers at every boundary: explicit 1x3x4
    windows on the 2x6x10 token grid (12 plain windows), so every rank owns windows
    of both kinds; checked against the same model on one GPU."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 4:
        pytest.skip("needs 4 GPUs")
    windows = (1, 3, 4)
    port = 29500 + (os.getpid() + 500) % 1000
    mp.start_processes(_rank, args=(4, port, str(tmp_path), windows), nprocs=4, join=True, start_method="spawn")
    flags, wi, wo, bws, noise, cond, text = _case()
    single = _model(0, flags, wi, wo, bws, windows).euler_step_host(noise, cond, text)
    outs = [np.load(tmp_path / f"x0_{r}.npy") for r in range(4)]
    for r in range(1, 4):
        assert np.array_equal(outs[0], outs[r]), r
    assert np.array_equal(outs[0], np.load(tmp_path / "x0b_0.npy"))
    m = parity.metrics(outs[0], single)
    assert m["max_abs"] <= 1e-4, m

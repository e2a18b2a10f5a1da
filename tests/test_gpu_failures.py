"""Failure handling, exercised without faulting the GPU: every failure is made on
the host and every device wait is bounded.

* A bounded wait that runs out: a one-shot test hook makes the attention
  kernel's load producer leave out one K tile in its first CTA, with a 20 ms
  wait limit. The tensor-core role's wait for that tile gives up, the kernel
  drains its in-flight copies and MMAs, frees TMEM and ends with an error code
  in the error word (one of the kernel's wait codes: whichever of the stalled
  waits gives up first); the layer's device-error query returns
  S2_INFERENCE_FAILED, and the same layer object's next forward is clean and
  equal to a fresh layer's.
* An allocation that fails: the next device allocation of a layer object is
  made to fail; the forward returns S2_OUT_OF_MEMORY (the reference's -100)
  and the next forward succeeds.
* A rank that never joins: rank 0 of a 2-rank communicator waits for a peer
  that is never started; s2_comm_init_timeout returns S2_INFERENCE_FAILED at
  its deadline (NCCL aborted) instead of blocking. Run in a child process with
  NVLS off; no collective is ever launched.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys
import time

import numpy as np
import pytest

import s2b200
from s2b200 import synth

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    assert s2b200.device_check(0) == 0, s2b200.last_error()
    return torch


def _layer(gam, fr, grid, heads):
    layer = s2b200.SeedVR2DiTBlockAttention(device=0, mode=s2b200.MODE_F16)
    layer.load_param(shifted=0, dim=heads * 128, heads=heads)
    layer.load_model(gam[0], gam[1], fr, gam[2], gam[3])
    layer.set_runtime_shape(*grid)
    return layer


def test_attention_wait_limit_expires_and_layer_recovers(torch_cuda):
    torch = torch_cuda
    grid, heads = (2, 16, 30), 4
    vid, txt, gam, fr = synth.layer_inputs(grid, heads=heads, seed=3)
    v = torch.from_numpy(vid).to("cuda", torch.float16)
    t = torch.from_numpy(txt).to("cuda", torch.float16)
    layer = _layer(gam, fr, grid, heads)
    lib = s2b200.lib()
    assert lib.s2_debug_attention_fault(1, 20_000_000) == 0   # leave out K tile 1 of CTA 0; 20 ms limit
    t0 = time.perf_counter()
    layer.forward(v, t)
    code = ctypes.c_int32(0)
    rc = lib.s2_attention_layer_device_error(layer.handle, ctypes.byref(code))
    elapsed = time.perf_counter() - t0
    # the first wait to give up records its code: the tensor-core role's wait for the missing K tile (2),
    # the producer's wait for a slot that role never released (2, 3) or a softmax group's wait for the S
    # tile that was never computed (5); all run out at the same limit
    assert rc == s2b200.S2_INFERENCE_FAILED and code.value in (2, 3, 5), (rc, code.value, s2b200.last_error())
    assert elapsed < 5.0, f"the failed launch took {elapsed:.2f} s"
    # the same object runs clean afterwards and matches a fresh layer
    vo, to = layer.forward(v, t)
    torch.cuda.synchronize()
    assert layer.device_error() == 0
    fresh = _layer(gam, fr, grid, heads)
    fo, ft = fresh.forward(v, t)
    torch.cuda.synchronize()
    assert torch.equal(vo, fo) and torch.equal(to, ft)


def test_allocation_failure_returns_out_of_memory(torch_cuda):
    torch = torch_cuda
    grid, heads = (2, 8, 12), 2
    vid, txt, gam, fr = synth.layer_inputs(grid, heads=heads, seed=5)
    v = torch.from_numpy(vid).cuda()
    t = torch.from_numpy(txt).cuda()
    layer = _layer(gam, fr, grid, heads)
    s2b200.lib().s2_debug_fail_allocations(1)
    try:
        with pytest.raises(s2b200.S2Error) as e:
            layer.forward(v, t)
        assert e.value.status == s2b200.S2_OUT_OF_MEMORY
    finally:
        s2b200.lib().s2_debug_fail_allocations(0)
    vo, _ = layer.forward(v, t)
    torch.cuda.synchronize()
    assert layer.device_error() == 0 and bool(torch.isfinite(vo.float()).all())


_NEVER_JOINS = r"""
import ctypes, sys, time
sys.path.insert(0, sys.argv[1])
import s2b200
lib = s2b200.lib()
uid = ctypes.create_string_buffer(128)
assert lib.s2_comm_unique_id(uid) == 0, s2b200.last_error()
h = ctypes.c_void_p()
t0 = time.time()
rc = lib.s2_comm_init_timeout(0, 2, 0, uid, 3000, ctypes.byref(h))
print("rc", rc, "elapsed", round(time.time() - t0, 2), "msg", s2b200.last_error(), flush=True)
sys.exit(0 if rc == -5 and not h.value else 1)
"""


def test_rank_that_never_joins_times_out():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", CUDA_VISIBLE_DEVICES=os.environ.get("CUDA_VISIBLE_DEVICES", "0"))
    r = subprocess.run([sys.executable, "-c", _NEVER_JOINS, os.path.join(ROOT, "seedvr2-ncnn-valkan_b200")],
                       capture_output=True, text=True, timeout=180, env=env)
    print(r.stdout, r.stderr[-2000:])
    assert r.returncode == 0, r.stdout + r.stderr[-2000:]
    elapsed = float(r.stdout.split("elapsed")[1].split()[0])
    assert 2.5 <= elapsed < 60.0, r.stdout

"""GPU checks of the block's tcgen05 GEMM (s2_gemm, the InnerProduct of
SeedVR2DiTBlock, seedvr2_dit_block.cpp:28-56) called through the C ABI.

Split-K (a GEMM of at most 128 rows whose tiles fill less than half the grid
splits K over several CTAs and a finish kernel adds the fp32 partial sums in
split order) must agree with the unsplit GEMM for every epilogue, and both
with a PyTorch fp32 reference of the same operation. Shapes are the block's
text-row GEMMs at dim 2560 (58 rows).

Tolerance of split vs unsplit: the tensor core's fp32 accumulation is not an
IEEE-ordered sum (it aligns the products of each K group before adding), so
another split of K moves results by up to ~1e-5 (K = 2560) to ~7e-5
(K = 6912) on O(1) outputs, measured. fp32 outputs are gated at 2e-4
absolute; fp16 outputs at one fp16 ulp of the value plus 1e-4.
"""
from __future__ import annotations

import numpy as np
import pytest

import s2b200

pytestmark = pytest.mark.gpu

M_TEXT = 58


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    assert s2b200.device_check(0) == 0, s2b200.last_error()
    return torch


def _operands(torch, M, N, K, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    a = torch.randn(M, K, generator=g).half().cuda()
    b = (torch.randn(N, K, generator=g) * 0.02).half().cuda()
    return a, b, g


def _workspace(torch):
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    return torch.empty(128 * 256 * sms, dtype=torch.float32, device="cuda"), sms


def _ref(a, b):
    return a.float() @ b.float().T


SPLIT_F32_ATOL = 2e-4


def _fp16_close(x, y, what):
    """fp16 outputs of two accumulations in another K split: within one fp16
    rounding step of the value plus the accumulation difference."""
    x = x.float().cpu().numpy()
    y = y.float().cpu().numpy()
    ulp = np.spacing(np.abs(y).astype(np.float16)).astype(np.float32)
    bad = np.abs(x - y) > ulp + 1e-4
    assert not bad.any(), f"{what}: {int(bad.sum())} elements beyond one fp16 ulp + 1e-4"


@pytest.mark.parametrize("M", [M_TEXT, 128])
def test_splitk_fused_qkv(torch_cuda, M):
    torch = torch_cuda
    d = 2560
    a, b, _ = _operands(torch, M, 3 * d, d, 1)
    ws, _ = _workspace(torch)
    outs = {}
    for name, w in (("split", ws), ("plain", None)):
        o = [torch.empty(M, d, dtype=torch.float16, device="cuda") for _ in range(3)]
        extra = s2b200.gemm(s2b200.GEMM_SPLIT_F16, a, b, outs=o, split=d, workspace=w)
        outs[name] = (torch.cat(o, dim=1), extra)
    torch.cuda.synchronize()
    assert outs["plain"][1] == 0
    if M == M_TEXT:
        assert outs["split"][1] == 1, "58-row QKV should take the split-K path"
    _fp16_close(outs["split"][0], outs["plain"][0], "split vs plain")
    ref = _ref(a, b)
    torch.testing.assert_close(outs["plain"][0].float(), ref, atol=2e-3, rtol=2e-3)


@pytest.mark.parametrize("split_row", [0, 40])
@pytest.mark.parametrize("K", [2560, 6912])
def test_splitk_gated_residual(torch_cuda, split_row, K):
    torch = torch_cuda
    d, M = 2560, M_TEXT
    a, b, g = _operands(torch, M, d, K, 2 + split_row)
    bias = (torch.randn(d, generator=g) * 0.02).cuda()
    gmul = (torch.randn(d, generator=g) * 0.02 + 1.0).cuda()
    resid = torch.randn(M, d, generator=g).cuda()
    ws, _ = _workspace(torch)
    res = {}
    for name, w in (("split", ws), ("plain", None)):
        y = torch.full((M, d), float("nan"), device="cuda")
        y2 = torch.full((M, d), float("nan"), device="cuda")
        kw = {}
        if split_row:
            kw = dict(split_row=split_row, resid2=resid[split_row:], y2=y2)
        extra = s2b200.gemm(s2b200.GEMM_GATED_RESID_F32, a, b, bias=bias, gmul=gmul,
                            resid=resid, y=y, workspace=w, **kw)
        out = torch.cat([y[:split_row], y2[:M - split_row]]) if split_row else y
        res[name] = (out, extra)
    torch.cuda.synchronize()
    assert res["plain"][1] == 0 and res["split"][1] == 1
    torch.testing.assert_close(res["split"][0], res["plain"][0], atol=SPLIT_F32_ATOL, rtol=0)
    ref = (_ref(a, b) + bias) * gmul + resid
    torch.testing.assert_close(res["plain"][0], ref, atol=5e-4, rtol=1e-4)


@pytest.mark.parametrize("M,K,split_row", [(300, 2560, 0), (4160, 2560, 0), (4160, 6912, 4102)])
def test_gated_residual_row_scatter(torch_cuda, M, K, split_row):
    """The row scatter of the gated-residual epilogue (each row of the block's MLP
    output stored at its next owner's row; here a permutation within y): every row
    equals the plain epilogue's row bit for bit at its destination, rows past the
    split still go to y2. M = 4160 runs the CTA-pair GEMM, 300 the single-CTA one."""
    torch = torch_cuda
    d = 2560
    a, b, g = _operands(torch, M, d, K, 11 + M)
    bias = (torch.randn(d, generator=g) * 0.02).cuda()
    gmul = (torch.randn(d, generator=g) * 0.02 + 1.0).cuda()
    resid = torch.randn(M, d, generator=g).cuda()
    rows = split_row or M
    perm = torch.randperm(rows, generator=g)
    dest = torch.stack([torch.zeros(rows, dtype=torch.int32), perm.to(torch.int32)], 1).contiguous().cuda()
    kw = dict(split_row=split_row, resid2=resid[split_row:]) if split_row else {}
    y_plain = torch.full((rows, d), float("nan"), device="cuda")
    y_sc = torch.full((rows, d), float("nan"), device="cuda")
    y2_plain = torch.full((max(M - rows, 1), d), float("nan"), device="cuda")
    y2_sc = torch.full((max(M - rows, 1), d), float("nan"), device="cuda")
    s2b200.gemm(s2b200.GEMM_GATED_RESID_F32, a, b, bias=bias, gmul=gmul, resid=resid, y=y_plain,
                y2=y2_plain if split_row else None, **kw)
    s2b200.gemm(s2b200.GEMM_GATED_RESID_F32, a, b, bias=bias, gmul=gmul, resid=resid, y=y_sc,
                y2=y2_sc if split_row else None, row_dest=dest, **kw)
    torch.cuda.synchronize()
    assert torch.equal(y_sc[perm.cuda()], y_plain)
    if split_row:
        assert torch.equal(y2_sc, y2_plain)


def test_splitk_gated_residual_last_block_rule(torch_cuda):
    """The last block's text rule: no gate, output scale 2: y = 2 (acc + b + resid)."""
    torch = torch_cuda
    d, M = 2560, M_TEXT
    a, b, g = _operands(torch, M, d, d, 5)
    bias = (torch.randn(d, generator=g) * 0.02).cuda()
    resid = torch.randn(M, d, generator=g).cuda()
    ws, _ = _workspace(torch)
    ys = []
    for w in (ws, None):
        y = torch.empty(M, d, device="cuda")
        s2b200.gemm(s2b200.GEMM_GATED_RESID_F32, a, b, bias=bias, resid=resid, y=y, out_scale=2.0, workspace=w)
        ys.append(y)
    torch.cuda.synchronize()
    torch.testing.assert_close(ys[0], ys[1], atol=2 * SPLIT_F32_ATOL, rtol=0)
    torch.testing.assert_close(ys[1], 2 * (_ref(a, b) + bias + resid), atol=1e-3, rtol=1e-4)


def test_splitk_swiglu(torch_cuda):
    torch = torch_cuda
    d, hidden, M = 2560, 6912, M_TEXT
    a, b, _ = _operands(torch, M, 2 * hidden, d, 3)
    ws, _ = _workspace(torch)
    res = {}
    for name, w in (("split", ws), ("plain", None)):
        o = torch.empty(M, hidden, dtype=torch.float16, device="cuda")
        extra = s2b200.gemm(s2b200.GEMM_SWIGLU_F16, a, b, outs=[o], workspace=w)
        res[name] = (o, extra)
    torch.cuda.synchronize()
    assert res["plain"][1] == 0 and res["split"][1] == 1
    _fp16_close(res["split"][0], res["plain"][0], "swiglu split vs plain")
    acc = _ref(a, b).view(M, hidden // 128, 2, 128)
    gate, inp = acc[:, :, 0, :], acc[:, :, 1, :]
    ref = (torch.nn.functional.silu(gate) * inp).reshape(M, hidden)
    torch.testing.assert_close(res["plain"][0].float(), ref, atol=2e-3, rtol=2e-3)


def test_gemm_rejects_bad_shapes(torch_cuda):
    torch = torch_cuda
    a = torch.zeros(8, 100, dtype=torch.float16, device="cuda")
    b = torch.zeros(64, 100, dtype=torch.float16, device="cuda")
    with pytest.raises(s2b200.S2Error) as e:
        s2b200.gemm(s2b200.GEMM_SPLIT_F16, a, b, outs=[torch.empty(8, 64, dtype=torch.float16, device="cuda")],
                    split=64)
    assert e.value.status == s2b200.S2_INVALID_ARGUMENT

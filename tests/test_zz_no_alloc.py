"""The allocation-free NorMuon apply entry point (b2o_normuon_apply_static).

It exists for callers that cannot give the library a scratch buffer (device
memory fully reserved by another allocator, or no allocation allowed while a
step is in flight). Its scratch is a fixed 1 MiB array inside the library, so
here it must reproduce the regular entry point (caller-provided scratch) on
the same inputs, call after call, and refuse batches that do not fit.

This file is collected last on purpose: it is a separate addition, and a
failure here must not stop a first-failure run before the other tests ran.
"""
import math

import pytest
import torch

from sol_b200 import _lib


def _batch(dev, S, r, c, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    o = (torch.randn(S, r, c, generator=g, device=dev) / math.sqrt(c)).to(torch.bfloat16)
    ntn = (c + 255) // 256
    pad = ntn * 256 - c
    sq = torch.nn.functional.pad(o.float().pow(2), (0, pad)).view(S, r, ntn, 256).sum(-1)  # [S][r][ntn]
    rowsq = sq.permute(0, 2, 1).contiguous()                                                # [S][ntn][r]
    return o, rowsq


def _state(dev, S, r, c, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    p = [(torch.randn(r, c, generator=g, device=dev) * 0.02).to(torch.bfloat16) for _ in range(S)]
    rem = [(torch.randn(r, c, generator=g, device=dev) * 1e-5).to(torch.bfloat16) for _ in range(S)]
    ema = [x.float().clone() for x in p]
    vrow = [torch.rand(r, 1, generator=g, device=dev) * 1e-3 for _ in range(S)]
    return p, rem, ema, vrow


def _call(lib, static, o, rowsq, st, scratch=None, lr=8e-3, wd=0.1, beta2=0.95, decay=0.999):
    p, rem, ema, vrow = st
    S, r, c = o.shape
    pa = _lib.ptr_array([x.data_ptr() for x in p])
    ra = _lib.ptr_array([x.data_ptr() for x in rem])
    ea = _lib.ptr_array([x.data_ptr() for x in ema])
    va = _lib.ptr_array([x.data_ptr() for x in vrow])
    args = (o.data_ptr(), rowsq.data_ptr(), S, r, c, pa, ra, ea, va, _lib.BF16, -lr, lr * wd, 1.0 - lr * wd, 1, 1,
            math.sqrt(max(1.0, r / c)), 1.0 - beta2, 1.0 - decay)
    if static:
        rc = lib.b2o_normuon_apply_static(*args, _lib.stream_ptr())
    else:
        rc = lib.b2o_normuon_apply(*args, scratch.data_ptr(), _lib.stream_ptr())
    _lib.check(rc, "normuon_apply_static" if static else "normuon_apply")


@pytest.mark.gpu
@pytest.mark.parametrize("S,r,c", [(3, 384, 128), (2, 128, 640), (14, 1024, 1024)])
def test_static_scratch_matches_caller_scratch(S, r, c):
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    dev = torch.device("cuda")
    lib = _lib.load()
    ref_state = _state(dev, S, r, c, seed=1)
    new_state = tuple([x.clone() for x in group] for group in ref_state)
    scratch = torch.empty(lib.b2o_normuon_apply_scratch_floats(S, r), dtype=torch.float32, device=dev)
    for call in range(2):  # two calls in a row: the shared array keeps the previous call's contents
        o, rowsq = _batch(dev, S, r, c, seed=10 + call)
        _call(lib, False, o, rowsq, ref_state, scratch=scratch)
        _call(lib, True, o, rowsq, new_state)
        torch.cuda.synchronize()
        assert _lib.device_error() == 0
        # same kernels, same inputs: identical results (the suite's tolerances
        # for this pass are bit-exactness of the bf16 split and 2 fp32 ulp)
        for name, a_list, b_list in zip(("param", "rem", "ema", "v_row"), ref_state, new_state):
            for a, b in zip(a_list, b_list):
                assert torch.equal(a, b), f"call {call}: {name} differs"


def test_static_scratch_rejects_batches_that_do_not_fit():
    """Host-side size guard only (nothing is launched), so it runs without a GPU too."""
    lib = _lib.load()
    limit = lib.b2o_normuon_apply_static_max_floats()
    assert limit == 1 << 18
    S, r, c = 64, 8192, 8  # 64 * 8196 floats > 262144
    dummy = _lib.ptr_array([1] * S)
    rc = lib.b2o_normuon_apply_static(1, 1, S, r, c, dummy, None, None, dummy, _lib.BF16, -1e-3, 0.0, 1.0, 0, 0,
                                      1.0, 0.05, 0.0, None)
    assert rc < 0
    msg = _lib.last_error()
    assert "scratch" in msg and str(limit) in msg

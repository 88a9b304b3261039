"""nllb_linear_int8_noalloc: the INT8 linear layer for callers that cannot let
a library allocate device memory while they run (a serving process whose
memory is all handed out by its own pool, a loop with a fixed memory plan).

It must give what nllb_linear_int8 gives, on consecutive calls that share
its fixed scratch array, and must not take device memory.  This file is
collected last, so a run that stops at the first failure has already run
every other test; it also passes on its own in a fresh process.
"""
import numpy as np
import pytest

import nllb_attn as na

pytestmark = pytest.mark.gpu


def _inputs(seed, M, K, N, device):
    import torch
    rng = np.random.default_rng(seed)
    x = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).to(device)
    w = torch.from_numpy(rng.integers(-127, 128, size=(N, K), dtype=np.int8)).to(device)
    scale = torch.from_numpy((np.full(N, 3666.19, np.float32) * rng.uniform(0.5, 2.0, N)).astype(np.float32)).to(device)
    bias = torch.from_numpy(rng.standard_normal(N, dtype=np.float32)).to(device)
    return x, w, scale, bias


def _bound(x, w, scale, ref):
    # the tolerance of the linear-layer tests: fp32 accumulation error
    # relative to the sum of |terms|
    inv = (1.0 / scale.cpu().numpy()).astype(np.float64)
    terms = np.abs(x.cpu().numpy().astype(np.float64)) @ np.abs(w.cpu().numpy().astype(np.float64)).T * inv
    return 2e-6 * (terms + 1.0) + 1e-6 * np.abs(ref)


@pytest.mark.parametrize("M,K,N", [(64, 1024, 1024), (200, 4096, 1024), (256, 1024, 4096), (8, 1024, 512),
                                   (64, 96, 1024)])
def test_noalloc_matches_allocating_entry_point_twice(cuda_device, M, K, N):
    import torch
    x, w, scale, bias = _inputs(M + K + N, M, K, N, cuda_device)
    expect = na.linear_int8(x, w, scale, bias, relu=True)
    torch.cuda.synchronize()
    ref = expect.cpu().numpy().astype(np.float64)
    bound = _bound(x, w, scale, ref)
    for call in range(2):  # the second call finds the scratch as the first left it
        out = torch.full((M, N), float("nan"), device=cuda_device)
        na.linear_int8_noalloc(x, w, scale, out, bias, relu=True)
        torch.cuda.synchronize()
        err = np.abs(out.cpu().numpy().astype(np.float64) - ref)
        assert np.isfinite(err).all() and (err <= bound).all(), f"call {call}: max err {np.nanmax(err):.3e}"
        assert na.linear_int8_noalloc_status() == na.OK  # no bounded wait gave up
    assert na.linear_int8_status() == na.OK


def test_noalloc_takes_no_device_memory(cuda_device):
    import torch
    M, K, N = 128, 1024, 1024
    x, w, scale, bias = _inputs(7, M, K, N, cuda_device)
    out = torch.empty((M, N), device=cuda_device)
    na.linear_int8_noalloc(x, w, scale, out, bias)  # first call on the device: address lookup
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        na.linear_int8_noalloc(x, w, scale, out, bias)
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda_device):
    import torch
    x, w, scale, bias = _inputs(9, 300, 1024, 64, cuda_device)
    out = torch.empty((300, 64), device=cuda_device)
    with pytest.raises(na.NllbAttnError) as ei:
        na.linear_int8_noalloc(x, w, scale, out, bias)
    assert ei.value.status == na.ECAPACITY
    assert b"256 rows" in na.load().nllb_attn_last_error()

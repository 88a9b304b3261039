"""nllb_linear_prepare / nllb_linear_run: the INT8 linear layer with its
weights made resident once (a LinearInt8, pico.h:26-32), run by the
TMA-fed tcgen05 kernel for more than 16 rows.

Checked against a float64 evaluation of mat_vec_int8's arithmetic
(tensor.c:144-196): out[m][n] = sum_k x[m][k] * (w[n][k] * (1/scale[n])) + bias[n],
then relu and the residual.  Tolerance: fp32 accumulation error relative to
the sum of |terms|, as for nllb_linear_int8.  The shapes reach every split-K
depth of the cluster reduction (1, 2, 4, 8 CTAs per tile), the persistent
128 x 256-tile kernel (outputs with at least one such tile per SM) and its
256 x 256-tile form on CTA pairs (tcgen05.mma.cta_group::2, from 129 rows), row
counts that are not multiples of the 128-row tile, output counts that are
not multiples of the tile or of 4 (the scalar store path), and the full
vocabulary projection.
"""
import numpy as np
import pytest

import nllb_attn as na

pytestmark = pytest.mark.gpu

SCALE = 127.0 / (0.02 * np.sqrt(3.0))


def _case(seed, M, K, N, bias, residual):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    scale = (np.full(N, SCALE, np.float32) * rng.uniform(0.5, 2.0, N)).astype(np.float32)
    b = rng.standard_normal(N, dtype=np.float32) if bias else None
    r = rng.standard_normal((M, N), dtype=np.float32) if residual else None
    return x, w, scale, b, r


def _reference(x, w, scale, bias, relu, residual):
    inv = (1.0 / scale).astype(np.float64)
    x64, w64 = x.astype(np.float64), w.astype(np.float64)
    y = (x64 @ w64.T) * inv
    terms = (np.abs(x64) @ np.abs(w64).T) * inv
    if bias is not None:
        y = y + bias
    if relu:
        y = np.maximum(y, 0.0)
    if residual is not None:
        y = y + residual
    return y, 2e-6 * (terms + 1.0) + 1e-6 * np.abs(y)


def _dev(a, device):
    import torch
    return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(device)


@pytest.mark.parametrize("M,K,N,epilogue", [
    # split-K cluster kernel (128 x 128 tiles), depth chosen for one wave on 148 SMs
    (17, 1024, 300, "bias_relu"),      # 8 CTAs per tile, 16-row slices, N tail
    (17, 1024, 301, "residual"),       # N % 4 != 0: scalar stores
    (300, 4096, 1024, "residual"),     # 4 CTAs per tile, M tail
    (1024, 4096, 1024, "bias_relu"),   # 2 CTAs per tile
    (2048, 4096, 1024, "plain"),       # no split (plain launch, no cluster)
    (2048, 1024, 1024, "residual"),    # no split, K = 1024
    # split-K kernel at the decoder's small-batch shapes
    (512, 1024, 3072, "bias_relu"),    # q/k/v projection of 128 sentences x 4 beams
    (200, 1024, 4096, "residual"),     # fc1 shape, M tail
    (77, 4096, 1000, "plain"),         # fc2-like (K = 4096), N tail
    (512, 1024, 2050, "residual"),     # N % 4 != 0 (scalar stores)
    # persistent kernel (at least 80 tiles of 128 x 256); on CTA pairs (256 x 256 tiles,
    # tcgen05.mma.cta_group::2) from 129 rows and 296 such tiles (two per SM of a B200)
    (4100, 1024, 4096, "bias_relu"),   # pairs, M tail
    (40, 1024, 256206, "plain"),       # vocabulary projection shape, N tail (one-CTA form)
    (129, 1024, 40000, "bias_relu"),   # pairs: the second CTA of each pair has one row
    (200, 1024, 40000, "residual"),    # pairs: M tail inside the second CTA
    (2000, 1024, 3001, "residual"),    # one-CTA form (one round of tiles), M and N tails, N % 4 != 0
    (1100, 4096, 3072, "bias_relu"),   # one-CTA form, K = 4096
])
def test_prepared_linear_matches_reference(cuda_device, M, K, N, epilogue):
    import torch
    x, w, scale, b, r = _case(M + N + K, M, K, N, epilogue == "bias_relu", epilogue == "residual")
    with na.PreparedLinear(_dev(w, cuda_device), _dev(scale, cuda_device), _dev(b, cuda_device)) as lin:
        out = lin(_dev(x, cuda_device), residual=_dev(r, cuda_device), relu=(epilogue == "bias_relu"))
        torch.cuda.synchronize()
        assert lin.status() == 0
    ref, bound = _reference(x, w, scale, b, epilogue == "bias_relu", r)
    err = np.abs(out.cpu().numpy().astype(np.float64) - ref)
    assert np.isfinite(err).all() and (err <= bound).all(), \
        f"max err {np.nanmax(err):.3e}, worst ratio {np.nanmax(err / bound):.2f}"


def test_prepared_linear_equals_int8_entry_point_across_row_counts(cuda_device):
    """One layer, run at growing and shrinking row counts (the activation
    buffer grows, its tensor map is re-encoded), against nllb_linear_int8."""
    import torch
    K, N = 1024, 1024
    _, w, scale, b, _ = _case(5, 1, K, N, True, False)
    wd, sd, bd = _dev(w, cuda_device), _dev(scale, cuda_device), _dev(b, cuda_device)
    with na.PreparedLinear(wd, sd, bd) as lin:
        for M in (8, 64, 512, 129, 64, 16, 700):
            x = _dev(np.random.default_rng(M).standard_normal((M, K), dtype=np.float32), cuda_device)
            got = lin(x, relu=True)
            want = na.linear_int8(x, wd, sd, bd, relu=True)
            torch.cuda.synchronize()
            ref, bound = _reference(x.cpu().numpy(), w, scale, b, True, None)
            for name, o in (("prepared", got), ("int8", want)):
                err = np.abs(o.cpu().numpy().astype(np.float64) - ref)
                assert (err <= bound).all(), f"{name} M={M}: max err {err.max():.3e}"
        assert lin.status() == 0


def test_bounded_wait_runs_out_and_layer_recovers(cuda_device):
    """A split-K launch (4 CTAs per tile) whose MMA thread's wait runs out
    (about 1 ms, the layer's test hook): it writes nothing, the status call
    reports NLLB_ATTN_ETIMEOUT once, and the same layer then computes the
    right result.  No fault, trap or endless wait is involved."""
    import torch
    M, K, N = 300, 4096, 1024
    x, w, scale, b, _ = _case(11, M, K, N, True, False)
    with na.PreparedLinear(_dev(w, cuda_device), _dev(scale, cuda_device), _dev(b, cuda_device)) as lin:
        dx = _dev(x, cuda_device)
        sentinel = torch.full((M, N), 7.0, device=cuda_device)
        lin.test_expire_next_wait()
        lin(dx, out=sentinel)
        torch.cuda.synchronize()
        assert lin.status() == na.ETIMEOUT
        assert bool((sentinel == 7.0).all()), "the timed-out launch wrote output"
        assert lin.status() == na.OK
        out = lin(dx)
        torch.cuda.synchronize()
        assert lin.status() == na.OK
    ref, bound = _reference(x, w, scale, b, False, None)
    err = np.abs(out.cpu().numpy().astype(np.float64) - ref)
    assert (err <= bound).all(), f"after the timeout: max err {err.max():.3e}"


def test_prepared_linear_rejects_bad_arguments(cuda_device):
    import torch
    w = torch.zeros((64, 100), dtype=torch.int8, device=cuda_device)
    s = torch.ones(64, device=cuda_device)
    with pytest.raises(na.NllbAttnError) as ei:
        na.PreparedLinear(w, s)  # K not a multiple of 64
    assert ei.value.status == na.EINVAL


@pytest.mark.parametrize("M,K,N,entry", [
    (4, 1024, 1024, "prepared"),      # few rows: the weight-streaming GEMV
    (512, 1024, 1024, "prepared"),    # split-K cluster kernel (4 CTAs per tile)
    (4096, 1024, 1024, "prepared"),   # one-CTA persistent kernel (128 tiles of 128 x 256)
    (4096, 1024, 3072, "prepared"),   # CTA pairs (384 tiles of 128 x 256)
    (300, 1024, 1024, "int8"),        # nllb_linear_int8: split-K with the last-CTA reduction
    (2048, 1024, 1024, "int8"),       # nllb_linear_int8: no split
])
def test_residual_in_place(cuda_device, M, K, N, entry):
    """x += f(x) as the decoder's residual layers run it: the output buffer is
    also the residual.  The kernels load a run of residual values before
    storing any of them; every element must still see its own old value."""
    import torch
    x, w, scale, b, r = _case(7 * M + N, M, K, N, True, True)
    wd, sd, bd = _dev(w, cuda_device), _dev(scale, cuda_device), _dev(b, cuda_device)
    buf = _dev(r, cuda_device)
    if entry == "prepared":
        with na.PreparedLinear(wd, sd, bd) as lin:
            lin(_dev(x, cuda_device), out=buf, residual=buf)
            torch.cuda.synchronize()
            assert lin.status() == 0
    else:
        na.linear_int8(_dev(x, cuda_device), wd, sd, bd, out=buf, residual=buf)
        torch.cuda.synchronize()
        assert na.linear_int8_status() == 0
    ref, bound = _reference(x, w, scale, b, False, r)
    err = np.abs(buf.cpu().numpy().astype(np.float64) - ref)
    assert np.isfinite(err).all() and (err <= bound).all(), \
        f"max err {np.nanmax(err):.3e}, worst ratio {np.nanmax(err / bound):.2f}"

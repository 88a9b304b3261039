"""The INT8-weight linear layer (mat_vec_int8, tensor.c:144-196, for many
rows) on the GPU against a float64 evaluation of the reference arithmetic:
out[m][n] = sum_k x[m][k] * (w[n][k] * (1/scale[n])) + bias[n].

Rows <= 16 take the SIMT kernel, more rows the tcgen05 kernel (int8 weights
exact in fp16, activations split into two fp16 parts); the tolerance is
fp32 accumulation error relative to the sum of |terms|.
"""
import numpy as np
import pytest

import nllb_attn as na

pytestmark = pytest.mark.gpu


def reference(x, w, scale, bias, relu, residual):
    inv = (1.0 / scale.astype(np.float32)).astype(np.float64)
    terms_abs = np.abs(x.astype(np.float64)) @ np.abs(w.astype(np.float64)).T * inv
    y = (x.astype(np.float64) @ w.astype(np.float64).T) * inv
    if bias is not None:
        y = y + bias
    if relu:
        y = np.maximum(y, 0.0)
    if residual is not None:
        y = y + residual
    return y, terms_abs


@pytest.mark.parametrize("M,K,N", [(1, 1024, 1024), (4, 1024, 3072), (16, 4096, 1024), (17, 1024, 300),
                                   (128, 1024, 1024), (300, 4096, 1024), (64, 1024, 256206 // 64)])
@pytest.mark.parametrize("epilogue", ["plain", "bias_relu", "residual"])
def test_linear_int8_matches_reference(cuda_device, M, K, N, epilogue):
    import torch
    rng = np.random.default_rng(M * 7 + K + N)
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    scale = np.full(N, 127.0 / (0.02 * np.sqrt(3.0)), dtype=np.float32) * rng.uniform(0.5, 2.0, N).astype(np.float32)
    bias = rng.standard_normal(N, dtype=np.float32) if epilogue == "bias_relu" else None
    residual = rng.standard_normal((M, N), dtype=np.float32) if epilogue == "residual" else None
    dev = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(cuda_device)
    out = na.linear_int8(dev(x), dev(w), dev(scale), dev(bias), residual=dev(residual),
                         relu=(epilogue == "bias_relu"))
    torch.cuda.synchronize()
    ref, terms = reference(x, w, scale, bias, epilogue == "bias_relu", residual)
    err = np.abs(out.cpu().numpy().astype(np.float64) - ref)
    bound = 2e-6 * (terms + 1.0) + 1e-6 * np.abs(ref)
    assert (err <= bound).all(), f"max err {err.max():.3e}, worst ratio {(err / bound).max():.2f}"


@pytest.mark.parametrize("name", ["lin_m1_n4096", "lin_m4_n1024", "lin_m17_n4096", "lin_m300_n1024"])
def test_linear_int8_matches_reference_golden(cuda_device, name):
    """Op-level pin: nllb_linear_int8 against the reference's own compiled
    mat_vec_int8 (tensor.c:144-196) on the golden inputs (tests/golden/cases.py),
    within the fp32 accumulation bound; both the SIMT (<= 16 rows) and the
    tensor-core (17, 300 rows) paths.  The error word stays clear."""
    import torch
    import cases
    x, w, scale, bias, rows = cases.linear_case(name)
    gold = cases.load_golden()[name].astype(np.float64)
    dev = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(cuda_device)
    out = na.linear_int8(dev(x), dev(w), dev(scale), dev(bias))
    assert na.linear_int8_status() == na.OK
    got = out.cpu().numpy()[rows].astype(np.float64)
    _, terms = reference(x[rows], w, scale, bias, False, None)
    err = np.abs(got - gold)
    bound = 2e-6 * (terms + 1.0) + 1e-6 * np.abs(gold)
    assert (err <= bound).all(), f"{name}: max err {err.max():.3e}, worst ratio {(err / bound).max():.2f}"
    # the prepared-weight path (the engine's layers) on the same golden
    with na.PreparedLinear(dev(w), dev(scale), dev(bias)) as lin:
        out2 = lin(dev(x))
        assert lin.status() == 0
    err2 = np.abs(out2.cpu().numpy()[rows].astype(np.float64) - gold)
    assert (err2 <= bound).all(), f"{name} prepared: max err {err2.max():.3e}"

"""The CPU restatement (oracle/attn_oracle.c) against the reference's outputs.

The golden outputs were produced by the reference's own C code
(tensor.c / decoder.c compiled from its sources); the restatement must agree
to rounding before it is trusted as the checker of the CUDA kernels.
"""
import numpy as np
import pytest

import cases
import pyoracle as po

# The reference builds with -ffast-math; the restatement without it.
PIN_ATOL = 2e-6


@pytest.fixture(scope="module")
def golden():
    return cases.load_golden()


@pytest.mark.parametrize("name", cases.PREFILL_CASES)
def test_prefill_oracle_matches_reference(golden, name):
    q, k, v, vl = cases.prefill_case(name)
    out = po.prefill(q, k, v, vl)
    np.testing.assert_allclose(out, golden[name], atol=PIN_ATOL, rtol=1e-5)


def test_head_flash_mask_oracle(golden):
    Q, K, V, mask = cases.head_mask_case()
    np.testing.assert_allclose(po.attention_head_flash(Q, K, V, mask), golden["head_flash_mask"],
                               atol=PIN_ATOL, rtol=1e-5)


def test_head_mask_oracle(golden):
    Q, K, V, mask = cases.head_mask_case()
    np.testing.assert_allclose(po.attention_head(Q, K, V, mask), golden["head_mask"],
                               atol=PIN_ATOL, rtol=1e-5)


@pytest.mark.parametrize("name", sorted(cases.DECODE_CASES))
def test_decode_oracle_matches_reference(golden, name):
    q, k, v, parents = cases.decode_case(name)
    out = po.decode_sweep(q, k, v, parents)
    steps = list(cases.DECODE_CASES[name])
    np.testing.assert_allclose(out[steps], golden[name], atol=PIN_ATOL, rtol=1e-5)


@pytest.mark.parametrize("name", cases.CROSS_CASES)
def test_cross_oracle_matches_reference(golden, name):
    K, V, q = cases.cross_case(name)
    np.testing.assert_allclose(po.cross(K, V, q), golden[name], atol=PIN_ATOL, rtol=1e-5)


def test_masked_key_semantics():
    """Key padding in the restatement is the reference's additive -1e9 mask
    (tensor.c:309): identical to a prefill over the unpadded keys only."""
    q = po.det_uniform(900, (1, 1, 20, 64))
    k = po.det_uniform(901, (1, 1, 20, 64))
    v = po.det_uniform(902, (1, 1, 20, 64))
    padded = po.prefill(q, k, v, np.array([13], np.int32))
    short = po.prefill(q[:, :, :, :], k[:, :, :13], v[:, :, :13], None,
                       strides=(20 * 64, 20 * 64, 64), shape=(1, 1, 13))
    np.testing.assert_allclose(padded[:, :, :13], short[:, :, :13], atol=1e-6)


def test_decode_reorder_is_copy_semantics():
    """Identity parents give the same result as no reorder at all."""
    q, k, v, _ = cases.decode_case("decode_dup40")
    ident = np.tile(np.arange(4, dtype=np.int32), (40, 1))
    np.testing.assert_array_equal(po.decode_sweep(q, k, v, ident), po.decode_sweep(q, k, v, None))


@pytest.mark.skipif(not po.ref_available(), reason="reference harness not built here")
def test_reference_harness_reproduces_golden(golden):
    """The compiled reference still produces the committed fixtures."""
    q, k, v, vl = cases.prefill_case("prefill_small")
    np.testing.assert_array_equal(po.ref_prefill_flash(q, k, v, vl), golden["prefill_small"])
    K, V, qc = cases.cross_case("cross_77")
    np.testing.assert_array_equal(po.ref_cross(K, V, qc), golden["cross_77"])


@pytest.mark.parametrize("name", cases.PENALTY_CASES)
def test_penalties_oracle_matches_reference(golden, name):
    """Bit for bit: the same fp32 operations in the same order."""
    logits, tokens, lens, pen, ngram = cases.penalties_case(name)
    out = po.penalties(logits, tokens, lens, pen, ngram).reshape(-1)
    idx = np.nonzero(out != logits.reshape(-1))[0]
    np.testing.assert_array_equal(idx, golden[name + "_idx"])
    np.testing.assert_array_equal(out[idx], golden[name + "_val"])


@pytest.mark.parametrize("name", cases.TOPK_CASES)
def test_logsoftmax_topk_oracle_matches_reference(golden, name):
    """Token ids exactly; log-probabilities to 1e-4: the reference sums the
    256206 exponentials in one fp32 running sum, which drifts by ~5e-5 from
    the float64 sum of the restatement."""
    logits, k = cases.topk_case(name)
    tok, lp = po.logsoftmax_topk(logits, k)
    np.testing.assert_array_equal(tok, golden[name + "_tok"])
    np.testing.assert_allclose(lp, golden[name + "_logp"], atol=1e-4, rtol=1e-5)


def linear_f64(x, w, scale, bias):
    """mat_vec_int8's arithmetic (tensor.c:144-196) in float64 -- the checker
    of the GPU linear-layer tests -- and the sum of |terms| per output."""
    inv = (1.0 / scale.astype(np.float32)).astype(np.float64)
    y = (x.astype(np.float64) @ w.astype(np.float64).T) * inv
    terms = (np.abs(x.astype(np.float64)) @ np.abs(w.astype(np.float64)).T) * inv
    if bias is not None:
        y = y + bias.astype(np.float64)
    return y, terms


@pytest.mark.parametrize("name", cases.LINEAR_CASES)
def test_linear_restatement_matches_reference(golden, name):
    """The float64 restatement against the reference's compiled mat_vec_int8:
    within the fp32 accumulation bound the GPU linear tests use."""
    x, w, scale, bias, rows = cases.linear_case(name)
    y, terms = linear_f64(x[rows], w, scale, bias)
    err = np.abs(golden[name].astype(np.float64) - y)
    bound = 2e-6 * (terms + 1.0) + 1e-6 * np.abs(y)
    assert (err <= bound).all(), f"{name}: max err {err.max():.3e}, worst ratio {(err / bound).max():.2f}"


def test_head_scores_golden_is_a_softmax(golden):
    """The reference's scores_buf after attention_head: each row the softmax of
    q.k/8 + mask (float64 restatement within fp32 rounding)."""
    Q, K, V, mask = cases.head_mask_case()
    s = (Q.astype(np.float64) @ K.astype(np.float64).T) * 0.125 + mask
    s = np.exp(s - s.max(axis=1, keepdims=True))
    s /= s.sum(axis=1, keepdims=True)
    np.testing.assert_allclose(golden["head_mask_scores"], s, atol=2e-6, rtol=1e-5)

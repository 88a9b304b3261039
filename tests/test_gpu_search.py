"""Per-step vocabulary operations of the beam search on the GPU.

nllb_apply_penalties (apply_repetition_penalty + apply_no_repeat_ngram,
main.c:186-213) must match the reference bit for bit; nllb_logsoftmax_topk
(log_softmax_inplace + find_topk, main.c:154-182) must pick the same token ids
in the same order -- up to the order inside runs of equal fp32 log-probability,
see assert_topk_equal_up_to_ties -- with log-probabilities within max-abs 1e-4
/ rel 1e-3 (the sum of exponentials is taken in another order).  Checked against the golden
outputs of the reference's own functions and, at the engine's sizes, against
the restatement in oracle/pyoracle.py.
"""
import numpy as np
import pytest
import torch

import cases
import nllb_attn as na
import pyoracle as po

pytestmark = pytest.mark.gpu

LOGP_ATOL, LOGP_RTOL = 1e-4, 1e-3


@pytest.fixture(scope="module")
def golden():
    return cases.load_golden()


def assert_topk_equal_up_to_ties(tok, ref_tok, ref_lp, logits, what):
    """Same ids in the same order, except inside a run of equal reference
    log-probabilities: logits a few ulps apart can round to the same fp32
    log-probability, which the reference then ranks by index while the kernel
    ranks by logit.  Inside a run the ids must be the same set; a run that
    reaches the k-th entry may also end with other ids whose logits lie within
    4 ulps of the run's."""
    for r in range(ref_tok.shape[0]):
        k = ref_tok.shape[1]
        j = 0
        while j < k:
            e = j + 1
            while e < k and ref_lp[r, e] == ref_lp[r, j]:
                e += 1
            ours, ref = list(tok[r, j:e]), list(ref_tok[r, j:e])
            if e - j == 1 and e < k:
                assert ours == ref, f"{what} row {r} entry {j}: {ours} vs {ref}"
            elif e < k:
                assert sorted(ours) == sorted(ref), f"{what} row {r} tie run {j}..{e}: {ours} vs {ref}"
            else:
                x0 = np.float32(logits[r, ref[0]])
                for t in ours:
                    if t not in ref:
                        gap = abs(int(np.float32(logits[r, t]).view(np.int32)) - int(x0.view(np.int32)))
                        assert gap <= 4, f"{what} row {r}: {t} not among {ref} and {gap} ulps away"
            j = e


def run_penalties(logits, tokens, lens, pen, ngram, ld=None):
    rows, V = logits.shape
    ld = ld or V
    buf = torch.full((rows, ld), 7.0, dtype=torch.float32, device="cuda")
    buf[:, :V] = torch.from_numpy(logits).cuda()
    tk = torch.from_numpy(np.ascontiguousarray(tokens, np.int32)).cuda()
    nt = torch.from_numpy(np.ascontiguousarray(lens, np.int32)).cuda()
    na.apply_penalties(buf, tk, nt, pen, ngram)
    out = buf.cpu().numpy()
    assert (out[:, V:] == 7.0).all()  # nothing written past the row
    return out[:, :V]


def run_topk(logits, k, ld=None):
    rows, V = logits.shape
    ld = ld or V
    buf = torch.zeros((rows, ld), dtype=torch.float32, device="cuda")
    buf[:, :V] = torch.from_numpy(logits).cuda()
    before = buf.clone()
    tok, lp = na.logsoftmax_topk(buf, k, vocab=V)
    assert torch.equal(buf, before)  # the logits are left as they were
    return tok.cpu().numpy(), lp.cpu().numpy()


@pytest.mark.parametrize("name", cases.PENALTY_CASES)
@pytest.mark.parametrize("pad", [0, 3])
def test_penalties_match_reference(cuda_device, golden, name, pad):
    logits, tokens, lens, pen, ngram = cases.penalties_case(name)
    out = run_penalties(logits, tokens, lens, pen, ngram, ld=logits.shape[1] + pad).reshape(-1)
    idx = np.nonzero(out != logits.reshape(-1))[0]
    np.testing.assert_array_equal(idx, golden[name + "_idx"])
    np.testing.assert_array_equal(out[idx], golden[name + "_val"])


@pytest.mark.parametrize("name", cases.TOPK_CASES)
@pytest.mark.parametrize("pad", [0, 1, 3])
def test_logsoftmax_topk_matches_reference(cuda_device, golden, name, pad):
    logits, k = cases.topk_case(name)
    tok, lp = run_topk(logits, k, ld=logits.shape[1] + pad)  # odd ld: rows start off 16-byte boundaries
    assert_topk_equal_up_to_ties(tok, golden[name + "_tok"], golden[name + "_logp"], logits, name)
    np.testing.assert_allclose(lp, golden[name + "_logp"], atol=LOGP_ATOL, rtol=LOGP_RTOL)


@pytest.mark.parametrize("rows,k", [(512, 8), (1, 8), (4096, 4)])
def test_logsoftmax_topk_engine_sizes(cuda_device, rows, k):
    """The vocabulary of NLLB-600M at the row counts of a decode step (4 beams
    x 128 / 1024 sentences) and of a single beam."""
    V = 256206
    g = torch.Generator(device="cuda").manual_seed(rows * 31 + k)
    logits = torch.randn((rows, V), generator=g, device="cuda") * 3.0
    tok, lp = na.logsoftmax_topk(logits, k)
    sample = list(range(0, rows, max(1, rows // 24)))[:24] + [rows - 1]
    x = logits[sample].cpu().numpy()
    ref_tok, ref_lp = po.logsoftmax_topk(x, k)
    assert_topk_equal_up_to_ties(tok[sample].cpu().numpy(), ref_tok, ref_lp, x, f"{rows} rows")
    np.testing.assert_allclose(lp[sample].cpu().numpy(), ref_lp, atol=LOGP_ATOL, rtol=LOGP_RTOL)
    # every row: best first, distinct ids, log-probabilities of a distribution
    lpa = lp.cpu().numpy()
    assert (np.diff(lpa, axis=1) <= 0).all() and (lpa < 0).all()
    t = tok.cpu().numpy()
    assert all(len(set(r)) == k for r in t)


def test_penalties_engine_sizes(cuda_device):
    """512 beam rows of 256206 logits with 130-token histories."""
    rows, V, T = 512, 256206, 130
    logits = po.det_uniform(701, (rows, V), 3.0)
    tokens = po.det_ints(702, rows * T, 0, 300).reshape(rows, T)
    tokens[:, 0] = 2
    lens = po.det_ints(703, rows, 0, T + 1)
    out = run_penalties(logits, tokens, lens, 1.2, 2)
    sample = list(range(0, rows, 16))
    ref = po.penalties(logits[sample], tokens[sample], lens[sample], 1.2, 2)
    np.testing.assert_array_equal(out[sample], ref)


def test_search_argument_errors(cuda_device):
    x = torch.zeros((2, 100), device="cuda")
    with pytest.raises(na.NllbAttnError) as ei:
        na.logsoftmax_topk(x, k=5)
    assert ei.value.status == na.EINVAL
    tk = torch.zeros((2, 4), dtype=torch.int32, device="cuda")
    nt = torch.zeros(2, dtype=torch.int32, device="cuda")
    with pytest.raises(na.NllbAttnError) as ei:
        na.apply_penalties(x, tk, nt, 1.2, 3)
    assert ei.value.status == na.EINVAL
    with pytest.raises(na.NllbAttnError) as ei:
        na.apply_penalties(x, tk, nt, 0.0, 2)
    assert ei.value.status == na.EINVAL


def test_penalties_skip_ids_outside_the_row(cuda_device):
    """A history may hold ids that are no token of the row (negative, or past
    its end) and a length longer than its row: nothing is read or written
    outside the logits, and every other logit is what the reference gives
    for the same history with those ids replaced by an otherwise unused token
    (whose own column is left out of the comparison)."""
    rows, V, T = 3, 777, 40
    logits = po.det_uniform(801, (rows, V), 3.0)
    tokens = po.det_ints(802, rows * T, 0, 20).reshape(rows, T)
    tokens[:, 0] = 2
    bad = [(0, 5, -5), (0, 9, V + 3), (1, 3, 2 ** 30), (1, 30, -1), (2, 17, V)]
    for r, g, t in bad:
        tokens[r, g] = t
    lens = np.array([40, 200, 25], np.int32)  # row 1 claims more tokens than its row holds
    out = run_penalties(logits, tokens, lens, 1.2, 2)
    sentinel = V - 1
    assert not (tokens == sentinel).any()
    clean = tokens.copy()
    for r, g, _ in bad:
        clean[r, g] = sentinel
    ref = po.penalties(logits, clean, np.minimum(lens, T), 1.2, 2)
    np.testing.assert_array_equal(out[:, :sentinel], ref[:, :sentinel])
    np.testing.assert_array_equal(out[:, sentinel], logits[:, sentinel])

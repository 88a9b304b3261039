"""Golden cases: seeded inputs whose outputs were produced by the reference.

Each case builds its inputs from integer-only generators (oracle/pyoracle.py:
det_uniform, det_ints, det_perms), so the same bits come back on any machine;
the .npz next to this file holds only the reference's outputs, written by
make_golden.py from the reference's own C (compiled into oracle/_ref).

Routines pinned (reference file:line):
  prefill_*        attention_head_flash   tensor.c:286-332 (key padding as -1e9)
  head_flash_mask  attention_head_flash   tensor.c:286-332 (general additive mask)
  head_mask        attention_head         tensor.c:255-282 (and head_mask_scores: the
                   softmaxed score matrix it leaves in scores_buf, tensor.c:266-277)
  decode_*         decoder_self_attn_cached decoder.c:48-99, reorder by copy main.c:481-482
  cross_*          decoder_cross_attn_cached decoder.c:103-152
  pen_*            apply_repetition_penalty + apply_no_repeat_ngram main.c:186-213
                   (stored as the flat indices and values of the changed logits)
  topk_*           log_softmax_inplace + find_topk main.c:154-182
  lin_*            mat_vec_int8 tensor.c:144-196 on each input row (stored rows
                   only for the 300-row case: every 7th)
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "oracle"))
import pyoracle as po  # noqa: E402

GOLDEN_NPZ = os.path.join(HERE, "golden_outputs.npz")

# decode sweeps store outputs of these steps only (keeps the fixture small)
DECODE256_STEPS = (0, 1, 2, 3, 7, 15, 31, 63, 64, 127, 128, 200, 255)
DECODE_DUP_STEPS = (0, 1, 2, 5, 13, 39)


def prefill_case(name):
    if name == "prefill_small":
        B, H, S = 2, 2, 40
        vl = np.array([40, 29], np.int32)
        seed = 101
    elif name == "prefill_cfg1_slice":
        B, H, S = 1, 2, 128
        vl = np.array([111], np.int32)
        seed = 111
    elif name == "prefill_nomask_odd":
        B, H, S = 1, 3, 67
        vl = None
        seed = 121
    else:
        raise KeyError(name)
    q = po.det_uniform(seed, (B, H, S, 64))
    k = po.det_uniform(seed + 1, (B, H, S, 64))
    v = po.det_uniform(seed + 2, (B, H, S, 64))
    return q, k, v, vl


PREFILL_CASES = ("prefill_small", "prefill_cfg1_slice", "prefill_nomask_odd")


def head_mask_case():
    S = 37
    Q = po.det_uniform(201, (S, 64))
    K = po.det_uniform(202, (S, 64))
    V = po.det_uniform(203, (S, 64))
    sel = po.det_ints(204, S * S, 0, 6).reshape(S, S)
    mask = np.where(sel == 0, np.float32(-1e9), po.det_uniform(205, (S, S), 0.5)).astype(np.float32)
    mask[:, 0] = 0.0  # every row keeps at least one unmasked key
    return Q, K, V, mask


def decode_case(name):
    NB, H = 4, 16
    if name == "decode_perm256":
        T, seed = 256, 301
        parents = po.det_perms(seed + 3, T, NB)
    elif name == "decode_dup40":
        T, seed = 40, 311
        parents = po.det_ints(seed + 3, T * NB, 0, NB).reshape(T, NB)
    else:
        raise KeyError(name)
    q = po.det_uniform(seed, (T, NB, H * 64))
    k = po.det_uniform(seed + 1, (T, NB, H * 64))
    v = po.det_uniform(seed + 2, (T, NB, H * 64))
    return q, k, v, parents


DECODE_CASES = {"decode_perm256": DECODE256_STEPS, "decode_dup40": DECODE_DUP_STEPS}


def cross_case(name):
    H, NB = 16, 4
    n_src, steps, seed = {"cross_512": (512, 3, 401), "cross_77": (77, 2, 411),
                          "cross_1": (1, 2, 421)}[name]
    K = po.det_uniform(seed, (n_src, H * 64))
    V = po.det_uniform(seed + 1, (n_src, H * 64))
    q = po.det_uniform(seed + 2, (steps, NB, H * 64))
    return K, V, q


CROSS_CASES = ("cross_512", "cross_77", "cross_1")


def penalties_case(name):
    """Logits, token histories and lengths for the penalty functions: tokens
    from a small range so that most repeat, token 2 mixed in, lengths from 0
    (nothing to do) to the full history."""
    rows, V, T, seed, ngram = {"pen_small": (9, 4099, 140, 501, 2), "pen_vocab": (4, 256206, 132, 511, 2),
                               "pen_nongram": (5, 1031, 64, 521, 0)}[name]
    logits = po.det_uniform(seed, (rows, V), 3.0)
    tokens = po.det_ints(seed + 1, rows * T, 0, 48).reshape(rows, T)
    tokens[:, 0] = 2
    tokens[:, 1] = V - 1
    tokens[po.det_ints(seed + 2, rows * T, 0, 9).reshape(rows, T) == 0] = 2
    lens = po.det_ints(seed + 3, rows, 0, T + 1)
    lens[0], lens[-1] = 0, T
    if rows > 2:
        lens[1] = 1
    return logits, tokens, lens, 1.2, ngram


PENALTY_CASES = ("pen_small", "pen_vocab", "pen_nongram")


def topk_case(name):
    """Logits for log-softmax + top-k: the full vocabulary; values on a coarse
    grid (many equal logits, so the lower-index-first rule decides); a small
    vocabulary; rows with banned (-1e30) entries."""
    rows, V, k, seed, grid = {"topk_vocab8": (3, 256206, 8, 601, 0.0), "topk_vocab4": (2, 256206, 4, 611, 0.0),
                              "topk_ties": (6, 5003, 8, 621, 0.25), "topk_small": (7, 37, 4, 631, 0.0)}[name]
    logits = po.det_uniform(seed, (rows, V), 4.0)
    if grid:
        logits = (np.round(logits / grid) * grid).astype(np.float32)
    banned = po.det_ints(seed + 1, rows * V, 0, 5).reshape(rows, V) == 0
    logits[banned] = np.float32(-1e30)
    return logits, k


TOPK_CASES = ("topk_vocab8", "topk_vocab4", "topk_ties", "topk_small")


def linear_case(name):
    """x [M][K], int8 w [N][K] over [-127, 127], per-row scales around the
    synthetic model's 3666.19 (x0.5 .. x2), bias or None; the stored rows."""
    M, K, N, seed, with_bias = {"lin_m1_n4096": (1, 1024, 4096, 701, True),
                                "lin_m4_n1024": (4, 1024, 1024, 711, False),
                                "lin_m17_n4096": (17, 1024, 4096, 721, True),
                                "lin_m300_n1024": (300, 1024, 1024, 731, True)}[name]
    x = po.det_uniform(seed, (M, K))
    w = (po.det_ints(seed + 1, N * K, -127, 128).reshape(N, K)).astype(np.int8)
    f = (np.float32(0.5) + po.det_ints(seed + 2, N, 0, 16).astype(np.float32) * np.float32(0.1)).astype(np.float32)
    scale = (np.float32(127.0 / (0.02 * np.sqrt(3.0))) * f).astype(np.float32)
    bias = po.det_uniform(seed + 3, (N,), 0.5) if with_bias else None
    rows = np.arange(0, M, 7) if M > 32 else np.arange(M)
    return x, w, scale, bias, rows


LINEAR_CASES = ("lin_m1_n4096", "lin_m4_n1024", "lin_m17_n4096", "lin_m300_n1024")


def load_golden():
    return np.load(GOLDEN_NPZ)

"""Golden cases: seeded inputs whose outputs were produced by the reference.

Each case builds its inputs from integer-only generators (oracle/pyoracle.py:
det_uniform, det_ints, det_perms), so the same bits come back on any machine;
the .npz next to this file holds only the reference's outputs, written by
make_golden.py from the reference's own C (compiled into oracle/_ref).

Routines pinned (reference file:line):
  prefill_*        attention_head_flash   tensor.c:286-332 (key padding as -1e9)
  head_flash_mask  attention_head_flash   tensor.c:286-332 (general additive mask)
  head_mask        attention_head         tensor.c:255-282
  decode_*         decoder_self_attn_cached decoder.c:48-99, reorder by copy main.c:481-482
  cross_*          decoder_cross_attn_cached decoder.c:103-152
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


def load_golden():
    return np.load(GOLDEN_NPZ)

"""Python access to the CPU checkers.  TEST INFRASTRUCTURE ONLY.

Two checkers live under oracle/:
  * ``_build/liboracle.so`` -- our C restatement of the reference attention
    (attn_oracle.c); runs anywhere, including the GPU box.
  * ``_ref/libnllb_ref.so`` -- the reference's own tensor.c/decoder.c compiled
    from its sources by oracle/Makefile (ref_attn_harness.c drives the live
    static functions).  Built in the container that has the reference; the
    prebuilt file travels with the repository snapshot.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use
this module.  The product (libnllb_attn.so) never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional

import numpy as np

ORACLE_DIR = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(ORACLE_DIR, "_build", "liboracle.so")
REF_SO = os.path.join(ORACLE_DIR, "_ref", "libnllb_ref.so")

_fp = ctypes.c_void_p
_ll = ctypes.c_longlong
_oracle: Optional[ctypes.CDLL] = None
_ref: Optional[ctypes.CDLL] = None


def build(quiet: bool = True) -> None:
    """make -C oracle (the reference part only where its sources exist)."""
    subprocess.run(["make", "-C", ORACLE_DIR, "all"], check=True,
                   stdout=subprocess.DEVNULL if quiet else None)


def oracle_lib() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_SO):
            build()
        lib = ctypes.CDLL(ORACLE_SO)
        lib.oracle_softmax.argtypes = [_fp, ctypes.c_int]
        lib.oracle_attention_head_flash.argtypes = [_fp] * 5 + [ctypes.c_int] * 2
        lib.oracle_attention_head.argtypes = [_fp] * 6 + [ctypes.c_int] * 2
        lib.oracle_prefill.argtypes = ([_fp] * 4 + [ctypes.c_int] * 4 + [_ll] * 3 + [_fp, _fp]
                                       + [_ll] * 2 + [ctypes.c_float])
        lib.oracle_decode_self_beam.argtypes = [_fp] + [ctypes.c_int] * 4 + [_fp] * 4
        lib.oracle_cross_beam.argtypes = [_fp, _fp, _ll] + [ctypes.c_int] * 3 + [_fp, _fp]
        lib.oracle_decode_sweep.argtypes = [_fp] + [ctypes.c_int] * 5 + [_fp] * 5
        _oracle = lib
    return _oracle


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref_lib() -> ctypes.CDLL:
    """The compiled reference harness; raises if it was never built."""
    global _ref
    if _ref is None:
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(f"{REF_SO} missing: run make -C {ORACLE_DIR} ref where the "
                                    "reference sources are present")
        lib = ctypes.CDLL(REF_SO)
        for n in ("ref_kv_cache_floats", "ref_kv_layer_floats", "ref_xattn_cache_floats"):
            getattr(lib, n).restype = ctypes.c_long
        lib.ref_sa_offset.restype = ctypes.c_long
        lib.ref_sa_offset.argtypes = [ctypes.c_int] * 4
        lib.ref_xa_offset.restype = ctypes.c_long
        lib.ref_xa_offset.argtypes = [ctypes.c_int] * 3
        lib.ref_decode_self_beam.argtypes = [_fp, ctypes.c_int, ctypes.c_int] + [_fp] * 4 + [ctypes.c_int]
        lib.ref_cross_beam.argtypes = [_fp, ctypes.c_int, ctypes.c_int, _fp, _fp, ctypes.c_int]
        lib.ref_prefill_flash.argtypes = [_fp] * 5 + [ctypes.c_int] * 3
        lib.attention_head_flash.argtypes = [_fp] * 5 + [ctypes.c_int] * 2
        lib.attention_head.argtypes = [_fp] * 6 + [ctypes.c_int] * 2
        lib.ref_mat_vec_int8_rows.argtypes = [_fp, _fp, _fp, ctypes.c_int, ctypes.c_int, _fp, ctypes.c_int, _fp]
        lib.ref_time_decode_sweep.restype = ctypes.c_double
        lib.ref_time_decode_sweep.argtypes = [ctypes.c_int] * 4 + [ctypes.c_ulonglong]
        lib.ref_time_cross.restype = ctypes.c_double
        lib.ref_time_cross.argtypes = [ctypes.c_int] * 5 + [ctypes.c_ulonglong]
        lib.ref_time_prefill.restype = ctypes.c_double
        lib.ref_time_prefill.argtypes = [ctypes.c_int] * 3 + [_fp, ctypes.c_int, ctypes.c_int,
                                                              ctypes.c_ulonglong]
        _ref = lib
    return _ref


def _p(a: Optional[np.ndarray]) -> Optional[int]:
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


# ---------------------------------------------------------------------------
# deterministic inputs (integer arithmetic only: identical on every machine)
# ---------------------------------------------------------------------------
def det_uniform(seed: int, shape, scale: float = 1.0) -> np.ndarray:
    """Uniform(-sqrt(3), sqrt(3)) * scale (unit variance), from splitmix64 of
    (seed, index); float32, reproducible bit for bit."""
    n = int(np.prod(shape))
    with np.errstate(over="ignore"):
        x = np.arange(n, dtype=np.uint64) + np.uint64((seed * 0x9E3779B97F4A7C15) & (2**64 - 1))
        z = x * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    u = ((z >> np.uint64(40)).astype(np.int64) - (1 << 23)).astype(np.float64) / float(1 << 23)
    return (u * (np.sqrt(3.0) * scale)).astype(np.float32).reshape(shape)


def det_ints(seed: int, n: int, lo: int, hi: int) -> np.ndarray:
    """n integers in [lo, hi), reproducible bit for bit."""
    with np.errstate(over="ignore"):
        x = np.arange(n, dtype=np.uint64) + np.uint64((seed * 0xD1B54A32D192ED03) & (2**64 - 1))
        z = x * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(31))) * np.uint64(0xBF58476D1CE4E5B9)
        z = z ^ (z >> np.uint64(29))
    return (lo + (z % np.uint64(hi - lo)).astype(np.int64)).astype(np.int32)


def det_perms(seed: int, n_steps: int, n_beams: int) -> np.ndarray:
    """[n_steps][n_beams] permutations of range(n_beams) (Fisher-Yates on det_ints)."""
    r = det_ints(seed, n_steps * n_beams, 0, 1 << 30)
    out = np.empty((n_steps, n_beams), dtype=np.int32)
    for t in range(n_steps):
        p = list(range(n_beams))
        for b in range(n_beams - 1, 0, -1):
            j = int(r[t * n_beams + b]) % (b + 1)
            p[b], p[j] = p[j], p[b]
        out[t] = p
    return out


# ---------------------------------------------------------------------------
# restatement (attn_oracle.c)
# ---------------------------------------------------------------------------
def prefill(q, k, v, valid_len=None, mask=None, scale=0.125, strides=None, shape=None,
            mask_strides=(0, 0)) -> np.ndarray:
    """oracle_prefill on [B,H,S,64] arrays (or explicit strides + shape=(B,H,S))."""
    q, k, v = (np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v))
    if strides is None:
        B, H, S, D = q.shape
        strides = (H * S * D, S * D, D)
    else:
        B, H, S = shape
    out = np.zeros_like(q)
    vl = None if valid_len is None else np.ascontiguousarray(valid_len, dtype=np.int32)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.float32)
    oracle_lib().oracle_prefill(_p(q), _p(k), _p(v), _p(out), B, H, S, 64, *strides, _p(vl),
                                _p(m), mask_strides[0], mask_strides[1], scale)
    return out


def attention_head_flash(Q, K, V, mask=None) -> np.ndarray:
    Q, K, V = (np.ascontiguousarray(a, dtype=np.float32) for a in (Q, K, V))
    out = np.zeros_like(Q)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.float32)
    oracle_lib().oracle_attention_head_flash(_p(Q), _p(K), _p(V), _p(m), _p(out), Q.shape[0],
                                             Q.shape[1])
    return out


def attention_head(Q, K, V, mask=None) -> np.ndarray:
    Q, K, V = (np.ascontiguousarray(a, dtype=np.float32) for a in (Q, K, V))
    out = np.zeros_like(Q)
    sb = np.zeros((Q.shape[0], Q.shape[0]), dtype=np.float32)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.float32)
    oracle_lib().oracle_attention_head(_p(Q), _p(K), _p(V), _p(m), _p(out), _p(sb), Q.shape[0],
                                       Q.shape[1])
    return out


def decode_sweep(q, k, v, parents=None, n_heads=16, max_gen=None) -> np.ndarray:
    """q,k,v: [T][NB][n_heads*64]; parents [T][NB] (reorder before each step) or None."""
    q, k, v = (np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v))
    T, NB, _ = q.shape
    max_gen = max_gen or T
    caches = np.zeros(2 * NB * 2 * n_heads * max_gen * 64, dtype=np.float32)
    out = np.zeros_like(q)
    par = None if parents is None else np.ascontiguousarray(parents, dtype=np.int32)
    oracle_lib().oracle_decode_sweep(_p(caches), NB, n_heads, 64, max_gen, T, _p(par), _p(q),
                                     _p(k), _p(v), _p(out))
    return out


def cross(K, V, q, n_heads=16) -> np.ndarray:
    """K,V: [n_src][n_heads*64] rows; q: [..., n_heads*64] -> same shape."""
    K, V = (np.ascontiguousarray(a, dtype=np.float32) for a in (K, V))
    q = np.ascontiguousarray(q, dtype=np.float32)
    flat = q.reshape(-1, n_heads * 64)
    out = np.zeros_like(flat)
    lib = oracle_lib()
    for i in range(flat.shape[0]):
        lib.oracle_cross_beam(_p(K), _p(V), K.shape[1], K.shape[0], n_heads, 64,
                              flat[i].ctypes.data, out[i].ctypes.data)
    return out.reshape(q.shape)


# ---------------------------------------------------------------------------
# the reference itself (oracle/_ref)
# ---------------------------------------------------------------------------
def ref_prefill_flash(q, k, v, valid_len=None) -> np.ndarray:
    """attention_head_flash per (b,h) of [B,H,S,64] inputs, key padding as -1e9."""
    q, k, v = (np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v))
    B, H, S, _ = q.shape
    out = np.zeros_like(q)
    vl = None if valid_len is None else np.ascontiguousarray(valid_len, dtype=np.int32)
    ref_lib().ref_prefill_flash(_p(q), _p(k), _p(v), _p(vl), _p(out), B, H, S)
    return out


def ref_linear(x, w, scale, bias=None) -> np.ndarray:
    """The reference's mat_vec_int8 (tensor.c:144-196) on each row of x [M][K]
    with w [N][K] int8, scale [N], bias [N] or None: [M][N] fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.int8)
    scale = np.ascontiguousarray(scale, dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    M, K = x.shape
    N = w.shape[0]
    out = np.zeros((M, N), np.float32)
    ref_lib().ref_mat_vec_int8_rows(_p(w), _p(scale), _p(b), N, K, _p(x), M, _p(out))
    return out


def ref_attention_head(Q, K, V, mask, flash: bool, return_scores: bool = False):
    """The reference's attention_head_flash (tensor.c:286) or attention_head
    (tensor.c:255); with return_scores (attention_head only) also the
    softmaxed score matrix it leaves in scores_buf (tensor.c:266-277)."""
    Q, K, V = (np.ascontiguousarray(a, dtype=np.float32) for a in (Q, K, V))
    out = np.zeros_like(Q)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.float32)
    lib = ref_lib()
    if flash:
        lib.attention_head_flash(_p(Q), _p(K), _p(V), _p(m), _p(out), Q.shape[0], Q.shape[1])
        return out
    sb = np.zeros((Q.shape[0], Q.shape[0]), dtype=np.float32)
    lib.attention_head(_p(Q), _p(K), _p(V), _p(m), _p(out), _p(sb), Q.shape[0], Q.shape[1])
    return (out, sb) if return_scores else out


def ref_decode_sweep(q, k, v, parents=None) -> np.ndarray:
    """decoder_self_attn_cached (decoder.c:48) per beam per step, layer 0, with
    the reference's reorder-by-copy (main.c:481-482) between steps."""
    lib = ref_lib()
    q, k, v = (np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v))
    T, NB, _ = q.shape
    per = lib.ref_kv_layer_floats()
    pools = [[np.zeros(per, dtype=np.float32) for _ in range(NB)] for _ in range(2)]
    cur = 0
    out = np.zeros_like(q)
    for t in range(T):
        if parents is not None:
            for b in range(NB):
                pools[1 - cur][b][:] = pools[cur][int(parents[t][b])]
            cur = 1 - cur
        for b in range(NB):
            ob = np.zeros(q.shape[2], dtype=np.float32)
            lib.ref_decode_self_beam(_p(pools[cur][b]), 0, t, q[t, b].ctypes.data,
                                     k[t, b].ctypes.data, v[t, b].ctypes.data, _p(ob), 1)
            out[t, b] = ob
    return out


def ref_cross(K, V, q) -> np.ndarray:
    """decoder_cross_attn_cached (decoder.c:103) at step > 0 over a memory
    written straight into the reference's shared cache layout."""
    lib = ref_lib()
    K, V = (np.ascontiguousarray(a, dtype=np.float32) for a in (K, V))
    n_src, dm = K.shape
    cache = np.zeros(lib.ref_xattn_cache_floats(), dtype=np.float32)
    k0, v0 = lib.ref_xa_offset(0, 0, 0), lib.ref_xa_offset(0, 1, 0)
    cache[k0:k0 + n_src * dm] = K.reshape(-1)
    cache[v0:v0 + n_src * dm] = V.reshape(-1)
    flat = np.ascontiguousarray(q, dtype=np.float32).reshape(-1, dm)
    out = np.zeros_like(flat)
    for i in range(flat.shape[0]):
        ob = np.zeros(dm, dtype=np.float32)
        lib.ref_cross_beam(_p(cache), 0, n_src, flat[i].ctypes.data, _p(ob), 1)
        out[i] = ob
    return out.reshape(np.shape(q))


# ---------------------------------------------------------------------------
# per-step vocabulary operations of the beam search (main.c:154-213)
# ---------------------------------------------------------------------------
REF_SEARCH_SO = os.path.join(ORACLE_DIR, "_ref", "libnllb_ref_search.so")
_ref_search: Optional[ctypes.CDLL] = None


def ref_search_available() -> bool:
    return os.path.exists(REF_SEARCH_SO)


def ref_search_lib() -> ctypes.CDLL:
    """main.c's own penalty / log-softmax / top-k functions (ref_search_harness.c)."""
    global _ref_search
    if _ref_search is None:
        if not os.path.exists(REF_SEARCH_SO):
            raise FileNotFoundError(f"{REF_SEARCH_SO} missing: run make -C {ORACLE_DIR} ref-main where the "
                                    "reference sources are present")
        lib = ctypes.CDLL(REF_SEARCH_SO)
        lib.ref_apply_penalties.argtypes = [_fp, ctypes.c_long, ctypes.c_int, _fp, ctypes.c_int, _fp,
                                            ctypes.c_float, ctypes.c_int]
        lib.ref_log_softmax_topk.argtypes = [_fp, ctypes.c_long, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             _fp, _fp]
        _ref_search = lib
    return _ref_search


def penalties(logits: np.ndarray, tokens: np.ndarray, n_tokens, penalty: float = 1.2,
              ngram: int = 2) -> np.ndarray:
    """apply_repetition_penalty (main.c:186-194) then apply_no_repeat_ngram
    (main.c:196-213, bigrams) on each row; returns a new fp32 array.  Every
    occurrence at positions 2..n-1 (token 2 excepted) divides a positive logit
    by the penalty or multiplies a non-positive one, in sequence.  The division
    is the multiplication by the fp32 reciprocal that every release build of
    the reference (-ffast-math, Makefile:15,19,33) compiles it to."""
    out = np.array(logits, dtype=np.float32, copy=True)
    pen = np.float32(penalty)
    inv = np.float32(1.0) / pen
    for r in range(out.shape[0]):
        lg, tk, n = out[r], tokens[r], int(n_tokens[r])
        for g in range(2, n):
            t = int(tk[g])
            if t == 2:
                continue
            lg[t] = lg[t] * inv if lg[t] > 0 else lg[t] * pen
        if ngram == 2 and n >= 2:
            cur = int(tk[n - 1])
            for i in range(0, n - 1):
                if int(tk[i]) == cur and int(tk[i + 1]) != 2:
                    lg[int(tk[i + 1])] = np.float32(-1e30)
    return out


def ref_penalties(logits: np.ndarray, tokens: np.ndarray, n_tokens, penalty: float = 1.2,
                  ngram: int = 2) -> np.ndarray:
    """The same through the reference's own functions (compiled main.c)."""
    lib = ref_search_lib()
    out = np.array(logits, dtype=np.float32, copy=True, order="C")
    tk = np.ascontiguousarray(tokens, dtype=np.int32)
    nt = np.ascontiguousarray(n_tokens, dtype=np.int32)
    lib.ref_apply_penalties(_p(out), out.shape[1], out.shape[0], _p(tk), tk.shape[1], _p(nt), penalty, ngram)
    return out


def logsoftmax_topk(logits: np.ndarray, k: int):
    """log_softmax_inplace (main.c:154-161) and find_topk (main.c:165-182) per
    row: the k largest log-probabilities, best first, the lower index first
    among equal values (find_topk's strict comparison), entries at or below
    -1e30 never taken.  Max and log in fp32 as the reference; the sum of
    exponentials in float64 (its order is not part of the result's contract)."""
    lg = np.asarray(logits, dtype=np.float32)
    rows = lg.shape[0]
    tok = np.zeros((rows, k), np.int32)
    lp = np.zeros((rows, k), np.float32)
    for r in range(rows):
        x = lg[r]
        mx = np.float32(x.max())
        se = np.exp((x - mx).astype(np.float64)).sum()
        ln = np.float32(mx + np.float32(np.log(se)))
        y = (x - ln).astype(np.float32)
        cand = np.nonzero(y > np.float32(-1e30))[0]
        part = cand[np.argpartition(-y[cand], min(k, len(cand)) - 1)[:k]] if len(cand) > k else cand
        kth = y[part].min()
        pool = cand[y[cand] >= kth]
        order = pool[np.lexsort((pool, -y[pool]))][:k]
        tok[r, :len(order)] = order
        lp[r, :len(order)] = y[order]
    return tok, lp


def ref_logsoftmax_topk(logits: np.ndarray, k: int):
    """The same through the reference's own functions (compiled main.c)."""
    lib = ref_search_lib()
    lg = np.array(logits, dtype=np.float32, copy=True, order="C")
    rows, n = lg.shape
    tok = np.zeros((rows, k), np.int32)
    sc = np.zeros((rows, k), np.float32)
    lib.ref_log_softmax_topk(_p(lg), n, n, rows, k, _p(tok), _p(sc))
    return tok, sc

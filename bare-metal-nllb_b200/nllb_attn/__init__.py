"""ctypes binding of libnllb_attn.so, the C ABI declared in include/nllb_attn.h.

The product is the shared library; this module only gives Python callers
(tests, bench.py) the same calls a C host makes.  Device-pointer calls take
torch CUDA tensors (or raw integer addresses); ``*_host`` calls take numpy
arrays.  Nothing here computes attention: every call goes through the
library, and a missing library raises at import of :func:`load`.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "libnllb_attn.so")

OK, EINVAL, ECAPACITY, ECUDA, ETIMEOUT, ENODEV, ESTATE = range(7)

# Every function include/nllb_attn.h declares, with (restype, argtypes).
_c_int, _c_void_p, _c_size_t = ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t
_fp = ctypes.c_void_p  # float*/const float*/int* passed as raw addresses


class Dims(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in (
        "n_layers", "n_heads", "head_dim", "max_sentences", "n_beams", "max_tgt", "max_src")]


class PrefillArgs(ctypes.Structure):
    _fields_ = [
        ("q", _fp), ("k", _fp), ("v", _fp), ("out", _fp),
        ("batch", ctypes.c_int), ("n_heads", ctypes.c_int), ("seq_len", ctypes.c_int),
        ("head_dim", ctypes.c_int),
        ("stride_batch", ctypes.c_int64), ("stride_head", ctypes.c_int64),
        ("stride_row", ctypes.c_int64),
        ("valid_len", _fp), ("mask", _fp),
        ("mask_stride_batch", ctypes.c_int64), ("mask_stride_head", ctypes.c_int64),
        ("scale", ctypes.c_float),
    ]


class TranslateOpts(ctypes.Structure):
    _fields_ = [("max_gen", ctypes.c_int), ("repetition_penalty", ctypes.c_float),
                ("no_repeat_ngram", ctypes.c_int)]


class TranslateStats(ctypes.Structure):
    _fields_ = [("encode_ms", ctypes.c_double), ("decode_ms", ctypes.c_double),
                ("steps", ctypes.c_int), ("tokens_out", ctypes.c_longlong)]


class KernelProfile(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 32), ("launches", ctypes.c_longlong), ("ms", ctypes.c_double),
                ("flops", ctypes.c_double), ("bytes", ctypes.c_double)]


PROF_CLASSES = 14

SIGNATURES = {
    "nllb_attn_create": (_c_int, [_c_int, ctypes.POINTER(Dims), ctypes.POINTER(_c_void_p)]),
    "nllb_attn_destroy": (None, [_c_void_p]),
    "nllb_attn_device_bytes": (_c_size_t, [ctypes.POINTER(Dims)]),
    "nllb_attn_set_stream": (_c_int, [_c_void_p, _c_void_p]),
    "nllb_attn_get_stream": (_c_void_p, [_c_void_p]),
    "nllb_attn_sync": (_c_int, [_c_void_p]),
    "nllb_attn_reset": (_c_int, [_c_void_p]),
    "nllb_attn_strerror": (ctypes.c_char_p, [_c_int]),
    "nllb_attn_last_error": (ctypes.c_char_p, []),
    "nllb_attn_prefill": (_c_int, [_c_void_p, ctypes.POINTER(PrefillArgs)]),
    "nllb_attn_prefill_host": (_c_int, [_c_void_p, ctypes.POINTER(PrefillArgs)]),
    "nllb_attn_decode_self": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _fp, _fp, _fp, _fp]),
    "nllb_attn_decode_self_host": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _fp, _fp, _fp, _fp]),
    "nllb_attn_reorder": (_c_int, [_c_void_p, _c_int, _fp]),
    "nllb_attn_reorder_host": (_c_int, [_c_void_p, _c_int, _fp]),
    "nllb_attn_test_expire_next_wait": (_c_int, [_c_void_p]),
    "nllb_attn_test_expire_next_cross_wait": (_c_int, [_c_void_p]),
    "nllb_attn_set_memory": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _fp, _fp,
                                      ctypes.c_int64, ctypes.c_int64]),
    "nllb_attn_set_memory_host": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _fp, _fp,
                                           ctypes.c_int64, ctypes.c_int64]),
    "nllb_attn_cross": (_c_int, [_c_void_p, _c_int, _c_int, _fp, _fp]),
    "nllb_attn_cross_host": (_c_int, [_c_void_p, _c_int, _c_int, _fp, _fp]),
    "nllb_attention_head": (None, [_fp, _fp, _fp, _fp, _fp, _fp, _c_int, _c_int]),
    "nllb_attention_head_flash": (None, [_fp, _fp, _fp, _fp, _fp, _c_int, _c_int]),
    "nllb_attn_last_status": (_c_int, []),
    # include/nllb_translate.h
    "nllb_model_load": (_c_int, [ctypes.c_char_p, _c_int, _c_int, _c_int, _c_int,
                                 ctypes.POINTER(_c_void_p)]),
    "nllb_model_free": (None, [_c_void_p]),
    "nllb_translate": (_c_int, [_c_void_p, _c_int, _fp, _fp, _c_int, ctypes.POINTER(TranslateOpts),
                                _fp, _fp, _fp, ctypes.POINTER(TranslateStats)]),
    "nllb_translate_margins": (_c_int, [_c_void_p, _c_int, _fp, _c_int]),
    "nllb_translate_profile": (_c_int, [_c_void_p, _c_int]),
    "nllb_translate_profile_read": (_c_int, [_c_void_p, ctypes.POINTER(KernelProfile), _c_int]),
    "nllb_linear_int8": (_c_int, [_fp, _c_int, _c_int, _fp, _fp, _fp, _c_int, _fp, _fp, _c_int, _c_void_p]),
    "nllb_linear_int8_status": (_c_int, []),
    "nllb_linear_int8_noalloc": (_c_int, [_fp, _c_int, _c_int, _fp, _fp, _fp, _c_int, _fp, _fp, _c_int,
                                          _c_void_p]),
    "nllb_linear_int8_noalloc_status": (_c_int, [_c_void_p]),
    "nllb_linear_prepare": (_c_int, [_fp, _fp, _fp, _c_int, _c_int, _c_void_p, ctypes.POINTER(_c_void_p)]),
    "nllb_linear_run": (_c_int, [_c_void_p, _fp, _c_int, _fp, _fp, _c_int, _c_void_p]),
    "nllb_linear_status": (_c_int, [_c_void_p]),
    "nllb_linear_test_expire_next_wait": (_c_int, [_c_void_p]),
    "nllb_linear_free": (None, [_c_void_p]),
    "nllb_apply_penalties": (_c_int, [_fp, ctypes.c_longlong, _c_int, _fp, _c_int, _fp, ctypes.c_float, _c_int,
                                      _c_void_p]),
    "nllb_logsoftmax_topk_ws_bytes": (_c_size_t, [_c_int, _c_int, _c_int]),
    "nllb_logsoftmax_topk": (_c_int, [_fp, ctypes.c_longlong, _c_int, _c_int, _c_int, _fp, _fp, _fp, _c_void_p]),
}

_LIB: Optional[ctypes.CDLL] = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the library (once) and declare every signature."""
    global _LIB
    if _LIB is not None and path == LIB_PATH:
        return _LIB
    if not os.path.exists(path):
        raise FileNotFoundError(
            f"{path} is missing: build it with `make -C {PKG_DIR}` (nvcc, sm_100a)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path == LIB_PATH:
        _LIB = lib
    return lib


class NllbAttnError(RuntimeError):
    def __init__(self, status: int, what: str, detail: str):
        super().__init__(f"{what}: status {status} ({detail})")
        self.status = status


def _check(lib, rc: int, what: str) -> None:
    if rc != OK:
        raise NllbAttnError(rc, what, lib.nllb_attn_last_error().decode())


def ptr(x) -> Optional[int]:
    """Raw address of a torch tensor, numpy array or int (None passes NULL)."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        if not x.is_contiguous():
            raise ValueError("tensor must be contiguous")
        return x.data_ptr()
    if hasattr(x, "ctypes"):
        if not x.flags["C_CONTIGUOUS"]:
            raise ValueError("array must be C-contiguous")
        return x.ctypes.data
    raise TypeError(f"cannot take the address of {type(x)!r}")


class Context:
    """One nllb_attn_ctx: caches, encoder memory and beam history on one GPU."""

    def __init__(self, device: int = 0, n_layers: int = 12, n_heads: int = 16,
                 max_sentences: int = 1, n_beams: int = 4, max_tgt: int = 256,
                 max_src: int = 512, lib: Optional[ctypes.CDLL] = None):
        self.lib = lib or load()
        self.dims = Dims(n_layers, n_heads, 64, max_sentences, n_beams, max_tgt, max_src)
        h = ctypes.c_void_p()
        _check(self.lib, self.lib.nllb_attn_create(device, ctypes.byref(self.dims), ctypes.byref(h)),
               "nllb_attn_create")
        self.handle = h
        self.n_beams, self.n_heads = n_beams, n_heads

    def close(self) -> None:
        if self.handle:
            self.lib.nllb_attn_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- plumbing --
    def set_stream(self, stream_handle: int) -> None:
        _check(self.lib, self.lib.nllb_attn_set_stream(self.handle, stream_handle), "set_stream")

    def sync(self) -> None:
        _check(self.lib, self.lib.nllb_attn_sync(self.handle), "nllb_attn_sync")

    def reset(self) -> None:
        _check(self.lib, self.lib.nllb_attn_reset(self.handle), "nllb_attn_reset")

    # -- prefill --
    @staticmethod
    def prefill_args(q, k, v, out, batch, n_heads, seq_len, strides, valid_len=None,
                     mask=None, mask_strides=(0, 0), scale=0.125) -> PrefillArgs:
        sb, sh, sr = strides
        return PrefillArgs(ptr(q), ptr(k), ptr(v), ptr(out), batch, n_heads, seq_len, 64,
                           sb, sh, sr, ptr(valid_len), ptr(mask), mask_strides[0],
                           mask_strides[1], scale)

    def prefill(self, args: PrefillArgs) -> None:
        _check(self.lib, self.lib.nllb_attn_prefill(self.handle, ctypes.byref(args)), "prefill")

    def prefill_host(self, args: PrefillArgs) -> None:
        _check(self.lib, self.lib.nllb_attn_prefill_host(self.handle, ctypes.byref(args)),
               "prefill_host")

    # -- decoder self-attention --
    def decode_self(self, layer, step, n_sent, q, k_new, v_new, out) -> None:
        _check(self.lib, self.lib.nllb_attn_decode_self(
            self.handle, layer, step, n_sent, ptr(q), ptr(k_new), ptr(v_new), ptr(out)),
            "decode_self")

    def decode_self_host(self, layer, step, n_sent, q, k_new, v_new, out) -> None:
        _check(self.lib, self.lib.nllb_attn_decode_self_host(
            self.handle, layer, step, n_sent, ptr(q), ptr(k_new), ptr(v_new), ptr(out)),
            "decode_self_host")

    def reorder(self, n_sent, parent) -> None:
        """nllb_attn_reorder: `parent` (a device tensor) must stay unchanged
        until the next decode_self, reorder, sync or reset on this context."""
        _check(self.lib, self.lib.nllb_attn_reorder(self.handle, n_sent, ptr(parent)), "reorder")

    def test_expire_next_wait(self) -> None:
        """nllb_attn_test_expire_next_wait: the next self-attention launch's
        bounded wait runs out (a chunk that is never requested)."""
        _check(self.lib, self.lib.nllb_attn_test_expire_next_wait(self.handle), "test_expire_next_wait")

    def test_expire_next_cross_wait(self) -> None:
        """nllb_attn_test_expire_next_cross_wait: the next cross-attention
        launch's bounded wait runs out (a chunk that is never requested)."""
        _check(self.lib, self.lib.nllb_attn_test_expire_next_cross_wait(self.handle), "test_expire_next_cross_wait")

    def reorder_host(self, n_sent, parent) -> None:
        _check(self.lib, self.lib.nllb_attn_reorder_host(self.handle, n_sent, ptr(parent)),
               "reorder_host")

    # -- cross-attention --
    def set_memory(self, layer, sentence, n_src, k, v, stride_head, stride_row) -> None:
        _check(self.lib, self.lib.nllb_attn_set_memory(
            self.handle, layer, sentence, n_src, ptr(k), ptr(v), stride_head, stride_row),
            "set_memory")

    def set_memory_host(self, layer, sentence, n_src, k, v, stride_head, stride_row) -> None:
        _check(self.lib, self.lib.nllb_attn_set_memory_host(
            self.handle, layer, sentence, n_src, ptr(k), ptr(v), stride_head, stride_row),
            "set_memory_host")

    def cross(self, layer, n_sent, q, out) -> None:
        _check(self.lib, self.lib.nllb_attn_cross(self.handle, layer, n_sent, ptr(q), ptr(out)),
               "cross")

    def cross_host(self, layer, n_sent, q, out) -> None:
        _check(self.lib, self.lib.nllb_attn_cross_host(self.handle, layer, n_sent, ptr(q),
                                                       ptr(out)), "cross_host")


def attention_head_flash(Q, K, V, mask, out, seq_len: int, head_dim: int = 64) -> int:
    """The drop-in for attention_head_flash (tensor.c:286); returns its status."""
    lib = load()
    lib.nllb_attention_head_flash(ptr(Q), ptr(K), ptr(V), ptr(mask), ptr(out), seq_len, head_dim)
    return lib.nllb_attn_last_status()


def attention_head(Q, K, V, mask, out, scores_buf, seq_len: int, head_dim: int = 64) -> int:
    """The drop-in for attention_head (tensor.c:255); returns its status."""
    lib = load()
    lib.nllb_attention_head(ptr(Q), ptr(K), ptr(V), ptr(mask), ptr(out), ptr(scores_buf),
                            seq_len, head_dim)
    return lib.nllb_attn_last_status()


class Model:
    """A synthetic-or-real NLLB INT8 model on one GPU (include/nllb_translate.h)."""

    def __init__(self, path: str, device: int = 0, max_sentences: int = 1, max_src: int = 256,
                 max_gen: int = 36, lib: Optional[ctypes.CDLL] = None):
        self.lib = lib or load()
        h = ctypes.c_void_p()
        _check(self.lib, self.lib.nllb_model_load(path.encode(), device, max_sentences, max_src,
                                                  max_gen, ctypes.byref(h)), "nllb_model_load")
        self.handle, self.max_gen = h, max_gen

    def close(self) -> None:
        if self.handle:
            self.lib.nllb_model_free(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def translate(self, sources, tgt_lang: int, max_gen: Optional[int] = None,
                  repetition_penalty: float = 1.2, no_repeat_ngram: int = 2):
        """sources: list of token-id lists ([src_lang] ... [2]).  Returns
        (list of output token lists, normalised scores, TranslateStats)."""
        import numpy as np
        flat = np.ascontiguousarray(np.concatenate([np.asarray(x, np.int32) for x in sources]))
        offs = np.zeros(len(sources) + 1, np.int32)
        offs[1:] = np.cumsum([len(x) for x in sources])
        G = max_gen or self.max_gen
        out = np.full((len(sources), self.max_gen), -1, np.int32)
        lens = np.zeros(len(sources), np.int32)
        scores = np.zeros(len(sources), np.float32)
        opts = TranslateOpts(G, repetition_penalty, no_repeat_ngram)
        st = TranslateStats()
        _check(self.lib, self.lib.nllb_translate(self.handle, len(sources), ptr(flat), ptr(offs), tgt_lang,
                                                 ctypes.byref(opts), ptr(out), ptr(lens), ptr(scores),
                                                 ctypes.byref(st)), "nllb_translate")
        toks = [out[i, :lens[i]].tolist() for i in range(len(sources))]
        return toks, scores, st

    def profile(self, enable: bool = True) -> None:
        """nllb_translate_profile: time the following translate calls' kernel
        launches by class (clears the totals)."""
        _check(self.lib, self.lib.nllb_translate_profile(self.handle, 1 if enable else 0), "nllb_translate_profile")

    def profile_read(self):
        """Per-class totals: {name: {launches, ms, flops, bytes}}."""
        buf = (KernelProfile * PROF_CLASSES)()
        n = self.lib.nllb_translate_profile_read(self.handle, buf, PROF_CLASSES)
        return {buf[i].name.decode(): {"launches": int(buf[i].launches), "ms": float(buf[i].ms),
                                       "flops": float(buf[i].flops), "bytes": float(buf[i].bytes)}
                for i in range(n)}

    def margins(self, sentence: int, max_steps: int = 1024):
        import numpy as np
        buf = np.zeros(max_steps, np.float32)
        n = self.lib.nllb_translate_margins(self.handle, sentence, ptr(buf), max_steps)
        return buf[:n]


LINEAR_RELU = 1


def linear_int8(x, w, weight_scale, bias=None, out=None, residual=None, relu=False, stream=None):
    """nllb_linear_int8 on torch CUDA tensors: x [M][K] fp32, w [N][K] int8."""
    lib = load()
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        import torch
        out = torch.empty((M, N), dtype=torch.float32, device=x.device)
    _check(lib, lib.nllb_linear_int8(ptr(x), M, K, ptr(w), ptr(weight_scale), ptr(bias), N, ptr(out),
                                     ptr(residual), LINEAR_RELU if relu else 0, stream), "nllb_linear_int8")
    return out


def linear_int8_noalloc(x, w, weight_scale, out, bias=None, residual=None, relu=False, stream=None):
    """nllb_linear_int8_noalloc on torch CUDA tensors; `out` must be given
    (the call allocates nothing, the caller owns every buffer)."""
    lib = load()
    M, K = x.shape
    N = w.shape[0]
    _check(lib, lib.nllb_linear_int8_noalloc(ptr(x), M, K, ptr(w), ptr(weight_scale), ptr(bias), N, ptr(out),
                                             ptr(residual), LINEAR_RELU if relu else 0, stream),
           "nllb_linear_int8_noalloc")
    return out


def linear_int8_status() -> int:
    """nllb_linear_int8_status: synchronises the device, reads and clears the
    error word of nllb_linear_int8 (returns the status, does not raise)."""
    return load().nllb_linear_int8_status()


def linear_int8_noalloc_status(stream=None) -> int:
    """nllb_linear_int8_noalloc_status: waits for `stream`, reads and clears
    the no-alloc entry point's error word (returns the status, does not raise)."""
    return load().nllb_linear_int8_noalloc_status(stream)


def apply_penalties(logits, tokens, n_tokens, penalty=1.2, no_repeat_ngram=2, stream=None):
    """nllb_apply_penalties on torch CUDA tensors, in place: logits [rows][ld]
    fp32, tokens [rows][tokens_ld] int32, n_tokens [rows] int32."""
    lib = load()
    rows = logits.shape[0]
    _check(lib, lib.nllb_apply_penalties(ptr(logits), logits.stride(0), rows, ptr(tokens), tokens.stride(0),
                                         ptr(n_tokens), penalty, no_repeat_ngram, stream), "nllb_apply_penalties")
    return logits


def logsoftmax_topk(logits, k=8, vocab=None, stream=None):
    """nllb_logsoftmax_topk on a torch CUDA tensor logits [rows][ld] fp32:
    returns (tokens [rows][k] int32, log-probabilities [rows][k] fp32)."""
    import torch
    lib = load()
    rows = logits.shape[0]
    V = logits.shape[1] if vocab is None else vocab
    tok = torch.empty((rows, k), dtype=torch.int32, device=logits.device)
    lp = torch.empty((rows, k), dtype=torch.float32, device=logits.device)
    ws = torch.empty(max(1, lib.nllb_logsoftmax_topk_ws_bytes(V, max(rows, 1), k)), dtype=torch.uint8,
                     device=logits.device)
    _check(lib, lib.nllb_logsoftmax_topk(ptr(logits), logits.stride(0), V, rows, k, ptr(tok), ptr(lp), ptr(ws),
                                         stream), "nllb_logsoftmax_topk")
    return tok, lp


class PreparedLinear:
    """nllb_linear_prepare / nllb_linear_run: one LinearInt8 resident on the
    GPU.  Keeps references to the weight tensors, which the layer reads."""

    def __init__(self, w, weight_scale, bias=None, stream=None):
        self._lib = load()
        self._keep = (w, weight_scale, bias)
        self.N, self.K = w.shape
        h = _c_void_p()
        _check(self._lib, self._lib.nllb_linear_prepare(ptr(w), ptr(weight_scale), ptr(bias), self.N, self.K,
                                                         stream, ctypes.byref(h)), "nllb_linear_prepare")
        self._h = h

    def __call__(self, x, out=None, residual=None, relu=False, stream=None):
        M = x.shape[0]
        if out is None:
            import torch
            out = torch.empty((M, self.N), dtype=torch.float32, device=x.device)
        _check(self._lib, self._lib.nllb_linear_run(self._h, ptr(x), M, ptr(out), ptr(residual),
                                                     LINEAR_RELU if relu else 0, stream), "nllb_linear_run")
        return out

    def status(self) -> int:
        return self._lib.nllb_linear_status(self._h)

    def test_expire_next_wait(self) -> None:
        """The next run on the split-K kernel times out (tests of the bounded waits)."""
        _check(self._lib, self._lib.nllb_linear_test_expire_next_wait(self._h), "nllb_linear_test_expire_next_wait")

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.nllb_linear_free(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def exported_symbols(header_path: str) -> Sequence[str]:
    """Function names declared in the C header (for the export check)."""
    import re
    text = open(header_path).read()
    return sorted(set(re.findall(r"NLLB_ATTN_API\s+[\w\s\*]*?\b(nllb_\w+)\s*\(", text)))

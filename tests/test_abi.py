"""The C ABI library loads without a GPU and exports what include/nllb_attn.h declares."""
import ctypes
import os
import subprocess

import pytest

import nllb_attn as na

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "nllb_attn.h")
HEADERS = [HEADER, os.path.join(REPO, "include", "nllb_translate.h")]


def test_library_exports_every_declared_symbol():
    declared = sorted(set().union(*(na.exported_symbols(h) for h in HEADERS)))
    assert len(declared) >= 20
    lib = ctypes.CDLL(na.LIB_PATH)
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", na.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert set(declared) <= exported
    # nothing of the implementation leaks into the dynamic symbol table
    assert all(n.startswith(("nllb_", "__cudaRegisterLinkedBinary")) for n in exported), exported


def test_binding_declares_every_header_function():
    declared = set().union(*(na.exported_symbols(h) for h in HEADERS))
    assert declared == set(na.SIGNATURES)


def test_header_compiles_as_c11(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#include "nllb_attn.h"\n#include "nllb_translate.h"\n'
                   'int main(void){nllb_attn_dims d={12,16,64,1,4,256,512};'
                   'nllb_translate_opts o={36,1.2f,2};(void)o;'
                   'return nllb_attn_device_bytes(&d) == 0;}\n')
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(REPO, "include"),
                    "-c", str(src), "-o", str(tmp_path / "t.o")], check=True)


def test_strerror_and_device_bytes():
    lib = na.load()
    assert lib.nllb_attn_strerror(na.OK) == b"ok"
    assert lib.nllb_attn_strerror(na.ENODEV) == b"no usable sm_100 device"
    d = na.Dims(12, 16, 64, 1, 4, 256, 512)
    b = lib.nllb_attn_device_bytes(ctypes.byref(d))
    kv = 2 * 12 * 1 * 16 * 256 * 4 * 64 * 4
    mem = 2 * 12 * 1 * 16 * 512 * 64 * 4
    assert kv + mem <= b < kv + mem + 16 * 2**20
    bad = na.Dims(12, 16, 32, 1, 4, 256, 512)
    assert lib.nllb_attn_device_bytes(ctypes.byref(bad)) == 0


@pytest.mark.parametrize("fields,needle", [
    ((12, 16, 32, 1, 4, 256, 512), b"head_dim"),
    ((12, 16, 64, 1, 3, 256, 512), b"n_beams"),
    ((0, 16, 64, 1, 4, 256, 512), b"n_layers"),
])
def test_create_rejects_bad_dims_before_touching_cuda(fields, needle):
    lib = na.load()
    d = na.Dims(*fields)
    h = ctypes.c_void_p()
    assert lib.nllb_attn_create(0, ctypes.byref(d), ctypes.byref(h)) == na.EINVAL
    assert needle in lib.nllb_attn_last_error()
    assert not h.value


def test_create_without_gpu_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(na.NllbAttnError) as ei:
        na.Context(0, n_layers=1, max_sentences=1)
    assert ei.value.status == na.ENODEV


def test_dropin_without_gpu_reports_status():
    import numpy as np
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    q = np.zeros((4, 64), np.float32)
    out = np.full_like(q, 7.0)
    assert na.attention_head_flash(q, q, q, None, out, 4) == na.ENODEV
    assert (out == 7.0).all()  # nothing was computed on the CPU instead

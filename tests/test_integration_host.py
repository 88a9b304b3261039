"""The reference's own C host with its attention routed to libnllb_attn
(integration/): the edits apply to the reference revision they were written
for, the programs link the library, and without a usable GPU they stop at
the first attention call with the library's message -- the GPU path has no
CPU fallback.  The GPU run itself is tests/test_gpu_integration.py."""
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INTEG = os.path.join(REPO, "integration")
REF_DIR = os.environ.get("REF_DIR", os.path.join(os.path.dirname(REPO), "reference"))
PROG = os.path.join(INTEG, "_build", "metalnllb_gpu_g36")

sys.path.insert(0, INTEG)
import apply_edits  # noqa: E402


@pytest.mark.skipif(not os.path.exists(os.path.join(REF_DIR, "main.c")), reason="reference sources not present")
def test_edits_apply_to_the_reference(tmp_path):
    apply_edits.sys.argv = ["apply_edits.py", REF_DIR, str(tmp_path)]
    apply_edits.main()
    calls = {"encoder.c": ["nllb_gpu_encoder_attention"],
             "decoder.c": ["nllb_gpu_self_attention", "nllb_gpu_cross_attention"],
             "main.c": ["nllb_gpu_beam_cache", "nllb_gpu_copy_beam", "nllb_gpu_expect_beams",
                        "nllb_gpu_stage_copy"]}
    for name, edits in apply_edits.EDITS.items():
        ref = open(os.path.join(REF_DIR, name)).read().splitlines()
        out = open(tmp_path / name).read()
        removed = sum(last - first + 1 for first, last, _ in edits)
        added = sum(text.count("\n") for _, _, text in edits)
        assert len(out.splitlines()) == len(ref) - removed + added, name
        for c in calls.get(name, []):
            assert c in out, (name, c)
    # main.c keeps no copy of a whole KV cache
    assert "KV_CACHE_TOTAL_FLOATS * sizeof(float)" not in open(tmp_path / "main.c").read()


@pytest.mark.skipif(not os.path.exists(PROG), reason="integration programs not built")
def test_program_links_the_library():
    out = subprocess.run(["ldd", PROG], capture_output=True, text=True).stdout
    assert "libnllb_attn.so" in out and "not found" not in out


@pytest.mark.skipif(not os.path.exists(PROG), reason="integration programs not built")
def test_program_has_no_cpu_fallback(synth_model_path):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: the GPU run is tests/test_gpu_integration.py")
    r = subprocess.run([PROG, synth_model_path, "eng_Latn", "fra_Latn", "5", "6", "7"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 1
    assert "[nllb-gpu] nllb_attn_create" in r.stderr
    assert "\ntokens:" not in r.stdout  # no translation was printed

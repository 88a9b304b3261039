"""Write the reference's C host with its attention routed to libnllb_attn.

Reads main.c, encoder.c, decoder.c, loader.c and tensor.c of the reference
from REF_DIR, checks that each is the revision these edits were written
against (sha256), replaces the line ranges below with calls into
nllb_gpu_shim.h and writes the results to OUT_DIR (a build directory that is
not version-controlled).  Every other line of the reference is kept as it
is: its loader, INT8 mat-vecs, LayerNorm, vocabulary projection, penalties,
top-k, per-beam thread pool and beam search.

    python integration/apply_edits.py REF_DIR OUT_DIR
"""
from __future__ import annotations

import hashlib
import os
import sys

# file -> sha256 of the reference revision the line numbers below refer to
REVISION = {
    "main.c": "08882d4ee0c907eb0a61e5f0878320890b77303740b438b3bca31876b8cabd0d",
    "encoder.c": "8a12f921d7c1af2973bed93b545eaf067c93fd317a4bdde4864ab3a2b5782da0",
    "decoder.c": "5c15d6c625358907c3971206aa7002c6f185893ceca4eff438339348292835fd",
    "loader.c": "f2846c32b7d04712a35c34dae9b86325a3bd8fcaf31abce21911e8361c02d7ee",
    "tensor.c": "39914969c438fd774b3b06c3290da0c27bf90b1720716d491e1845da2a584187",
}

# file -> [(first line, last line, replacement)], 1-based and inclusive
EDITS = {
    "encoder.c": [
        # multi_head_self_attn_flash: the per-head, per-query attention loop
        (165, 205, "    nllb_gpu_encoder_attention(sc->Q, sc->K, sc->V, sc->head_out, seq_len);\n"),
    ],
    "decoder.c": [
        # decoder_self_attn_cached: cache append and attention over step+1 positions
        (61, 96, "    float attn_out_full[D_MODEL];\n"
                 "    nllb_gpu_self_attention(kv_cache, layer_idx, step, q_full, k_full, v_full, attn_out_full);\n"),
        # decoder_cross_attn_cached: attention over the n_src memory rows (the
        # step-0 projection of those rows into the shared cache stays)
        (127, 149, "    float attn_out_full[D_MODEL];\n"
                   "    nllb_gpu_cross_attention(layer_idx, step, n_src, K, V, q_full, attn_out_full);\n"),
    ],
    "main.c": [
        # per-beam KV caches: handles (the caches are on the GPU)
        (301, 301, "            beam_kv[p][b] = nllb_gpu_beam_cache(p, b);\n"),
        # bootstrap copies after steps 0 and 1: every beam continues beam 0
        (338, 339, "        if (b > 0) nllb_gpu_copy_beam(beam_kv[cur_pool][b], beam_kv[cur_pool][0]);\n"),
        (390, 391, "        if (b > 0) nllb_gpu_copy_beam(beam_kv[cur_pool][b], beam_kv[cur_pool][0]);\n"),
        # the beam threads of this step meet at each attention call
        (444, 444, "        nllb_gpu_expect_beams(step, n_active);\n"
                   "        dispatch_beam_tasks(tasks, beams);\n"),
        # child i continues parent par: an index reorder before the next step
        (481, 482, "            nllb_gpu_stage_copy(beam_kv[np][i], beam_kv[cur_pool][par]);\n"),
    ],
    "loader.c": [],
    "tensor.c": [],
}


def main() -> None:
    ref_dir, out_dir = sys.argv[1], sys.argv[2]
    os.makedirs(out_dir, exist_ok=True)
    for name, edits in EDITS.items():
        with open(os.path.join(ref_dir, name), "rb") as f:
            raw = f.read()
        digest = hashlib.sha256(raw).hexdigest()
        if digest != REVISION[name]:
            raise SystemExit(f"{name}: not the reference revision these edits were written for ({digest})")
        lines = raw.decode().splitlines(keepends=True)
        for first, last, text in sorted(edits, reverse=True):  # bottom-up keeps earlier line numbers
            lines[first - 1:last] = [text]
        with open(os.path.join(out_dir, name), "w") as f:
            f.writelines(lines)
    print(f"wrote {len(EDITS)} sources to {out_dir}")


if __name__ == "__main__":
    main()

"""Synthetic NLLB-600M-shaped INT8 model in the reference's safetensors layout.

The real NLLB weights are not available here, so translation is measured on a
random-initialised model of the same architecture: d_model 1024, 16 heads of
64, FFN 4096, 12 encoder + 12 decoder layers, 256206-row shared embedding,
pre-LayerNorm.  Tensor names, shapes and dtypes are the CTranslate2 ones the
reference loader resolves (loader.c:104-174 encoder, :178-283 decoder,
:322-368 embeddings and final norms), so the reference engine and the GPU
engine read the same file.

Values:
  * int8 weights uniform in [-127, 127];
  * weight_scale = 127 / (0.02 * sqrt(3)) per row: the reference DIVIDES by
    the stored scale (tensor.c:75), so this gives weights uniform in
    +-0.0346 (std 0.02), the intended distribution;
  * biases and LayerNorm beta 0, gamma 1.

Random bytes come from a counter-based splitmix64 in integer numpy
arithmetic, so the file is identical on every machine for a given seed.
"""
from __future__ import annotations

import json
import os
import struct
from typing import Dict, List, Tuple

import numpy as np

VOCAB, D, FFN, LAYERS = 256206, 1024, 4096, 12
WEIGHT_SCALE = 127.0 / (0.02 * np.sqrt(3.0))

LANG = {"eng_Latn": 256047, "fra_Latn": 256057, "spa_Latn": 256168, "deu_Latn": 256050,
        "zho_Hans": 256158, "ara_Arab": 256027, "hin_Deva": 256069, "por_Latn": 256148,
        "rus_Cyrl": 256154, "jpn_Jpan": 256090, "kor_Hang": 256098, "swh_Latn": 256175,
        "hau_Latn": 256066, "yor_Latn": 256219, "ibo_Latn": 256073}


def _splitmix_int8(seed: int, start: int, n: int) -> np.ndarray:
    """n int8 values uniform in [-127, 127] for counters start..start+n-1."""
    with np.errstate(over="ignore"):
        z = (np.arange(start, start + n, dtype=np.uint64)
             + np.uint64((seed * 0x9E3779B97F4A7C15) & (2**64 - 1)))
        z = z * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return (((z >> np.uint64(32)) % np.uint64(255)).astype(np.int16) - 127).astype(np.int8)


def tensor_specs() -> List[Tuple[str, str, Tuple[int, ...]]]:
    """(name, dtype, shape) of every tensor, in file order."""
    specs: List[Tuple[str, str, Tuple[int, ...]]] = []

    def linear(prefix, out_f, in_f):
        specs.append((f"{prefix}/weight", "I8", (out_f, in_f)))
        specs.append((f"{prefix}/weight_scale", "F32", (out_f,)))
        specs.append((f"{prefix}/bias", "F32", (out_f,)))

    def norm(prefix):
        specs.append((f"{prefix}/gamma", "F32", (D,)))
        specs.append((f"{prefix}/beta", "F32", (D,)))

    specs.append(("encoder/embeddings_0/weight", "I8", (VOCAB, D)))
    specs.append(("decoder/embeddings/weight", "I8", (VOCAB, D)))
    specs.append(("decoder/embeddings/weight_scale", "F32", (VOCAB,)))
    for i in range(LAYERS):
        p = f"encoder/layer_{i}"
        linear(f"{p}/self_attention/linear_0", 3 * D, D)   # fused q, k, v
        linear(f"{p}/self_attention/linear_1", D, D)
        norm(f"{p}/self_attention/layer_norm")
        linear(f"{p}/ffn/linear_0", FFN, D)
        linear(f"{p}/ffn/linear_1", D, FFN)
        norm(f"{p}/ffn/layer_norm")
    norm("encoder/layer_norm")
    for i in range(LAYERS):
        p = f"decoder/layer_{i}"
        linear(f"{p}/self_attention/linear_0", 3 * D, D)
        linear(f"{p}/self_attention/linear_1", D, D)
        norm(f"{p}/self_attention/layer_norm")
        linear(f"{p}/attention/linear_0", D, D)            # cross q
        linear(f"{p}/attention/linear_1", 2 * D, D)        # cross k, v
        linear(f"{p}/attention/linear_2", D, D)            # cross out
        norm(f"{p}/attention/layer_norm")
        linear(f"{p}/ffn/linear_0", FFN, D)
        linear(f"{p}/ffn/linear_1", D, FFN)
        norm(f"{p}/ffn/layer_norm")
    norm("decoder/layer_norm")
    return specs


def write_model(path: str, seed: int = 0, chunk: int = 1 << 24) -> Dict[str, int]:
    """Write the model to `path` (about 860 MB).  Returns {name: byte offset}
    of each tensor's data within the data region.  The shared embedding is
    written twice (encoder and decoder names, same bytes), as the reference
    resolves both names (loader.c:327-330)."""
    specs = tensor_specs()
    header, offsets, off = {}, {}, 0
    for name, dt, shape in specs:
        n = int(np.prod(shape)) * (1 if dt == "I8" else 4)
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + n]}
        offsets[name] = off
        off += n
    hjson = json.dumps(header, separators=(",", ":")).encode()
    hjson += b" " * ((8 - len(hjson) % 8) % 8)
    tmp = path + ".tmp"
    counter = 0
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(hjson)))
        f.write(hjson)
        emb_start = None
        for name, dt, shape in specs:
            n = int(np.prod(shape))
            if dt == "I8":
                if name == "decoder/embeddings/weight":
                    start = emb_start          # same bytes as the encoder embedding
                else:
                    start = counter
                    counter += n
                    if name == "encoder/embeddings_0/weight":
                        emb_start = start
                for s in range(0, n, chunk):
                    f.write(_splitmix_int8(seed, start + s, min(chunk, n - s)).tobytes())
            elif name.endswith("weight_scale"):
                f.write(np.full(n, WEIGHT_SCALE, dtype=np.float32).tobytes())
            elif name.endswith("gamma"):
                f.write(np.ones(n, dtype=np.float32).tobytes())
            else:  # bias, beta
                f.write(np.zeros(n, dtype=np.float32).tobytes())
    os.replace(tmp, path)
    return offsets


def default_model_path(seed: int = 0) -> str:
    """Where the seeded model is kept: $NLLB_SYNTH_MODEL when set, else
    .synth/ at the root of this repository (kept out of version control)."""
    env = os.environ.get("NLLB_SYNTH_MODEL")
    if env:
        return env
    repo = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    return os.path.join(repo, ".synth", f"synth_nllb600m_seed{seed}.safetensors")


def ensure_model(path: str, seed: int = 0) -> str:
    """Write the model unless a complete file is already there."""
    specs = tensor_specs()
    total = sum(int(np.prod(s)) * (1 if d == "I8" else 4) for _, d, s in specs)
    if os.path.exists(path) and os.path.getsize(path) > total:
        return path
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    write_model(path, seed)
    return path


def source_lengths(seed: int, n: int, lo: int, hi: int) -> List[int]:
    """n source lengths uniform in [lo, hi) from a splitmix-style integer hash
    of (seed, index): the same on every machine."""
    with np.errstate(over="ignore"):
        x = np.arange(n, dtype=np.uint64) + np.uint64((seed * 0xD1B54A32D192ED03) & (2**64 - 1))
        z = x * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(31))) * np.uint64(0xBF58476D1CE4E5B9)
        z = z ^ (z >> np.uint64(29))
    return [int(v) for v in (lo + (z % np.uint64(hi - lo)).astype(np.int64))]


def source_ids(seed: int, n_tokens: int, src_lang: str = "eng_Latn") -> List[int]:
    """[src_lang] + n_tokens ids uniform in [4, 256000) + [2] (</s>), the way
    the reference builds its source (main.c:274-290)."""
    with np.errstate(over="ignore"):
        z = (np.arange(n_tokens, dtype=np.uint64)
             + np.uint64((seed * 0xD1B54A32D192ED03 + 0x1234567) & (2**64 - 1)))
        z = z * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(31))) * np.uint64(0xBF58476D1CE4E5B9)
        z = z ^ (z >> np.uint64(29))
    ids = (4 + (z % np.uint64(256000 - 4))).astype(np.int64).tolist()
    return [LANG[src_lang]] + [int(t) for t in ids] + [2]


def config4_sources(n: int = 1024, seed: int = 4) -> List[List[int]]:
    """The sentence-batched translation workload: n sources of U[16,128]
    tokens (ids U[4,256000)), each [eng_Latn] ... [2]; sentence i is the same
    whatever n is."""
    lengths = source_lengths(seed, n, 16, 129)
    return [source_ids(seed * 1000003 + i, lengths[i]) for i in range(n)]

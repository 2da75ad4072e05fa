"""Write ``tests/golden/tiny.fgm``: a small .fgm model file made by the
reference's own writer, to pin this repository's .fgm readers.

Run where the reference tree exists:

    python tests/golden/make_fgm_fixture.py [--ref /path/to/fastgemma]

The file is written with ``FgmWriter`` from the reference's ``convert/fgm.py``
(magic, header length, JSON header, 64-byte aligned blobs), and the weights
are packed with the reference's ``convert/quant.py`` (``pack_b_tiles``,
``pack_nibbles``, quant.py:76-117), using the tensor naming and metadata of
the converter (``convert_gemma4.py:174-205``: ``<name>`` with
``{"hadamard", "group"}`` meta, ``<name>.scale`` f16 [K/group][N] or f32 [N],
an optional int8 twin ``<name>.i8`` with ``<name>.i8.scale``).  The integer
weights and scales come from seeded generators, so the tests can rebuild
every expected value.
"""
from __future__ import annotations

import argparse
import importlib.util
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# name, bits, N, K, group, hadamard, int8 twin, seed
LINEARS = [
    ("layers.0.mlp.gate_proj", 4, 128, 256, 64, 128, True, 11),
    ("layers.0.self_attn.q_proj", 4, 64, 256, 128, 0, False, 12),
    ("layers.0.self_attn.o_proj", 8, 64, 128, 0, 64, False, 13),
]
CONFIG = {"hidden_size": 256, "num_hidden_layers": 1, "intermediate_size": 128,
          "vocab_size": 64, "rms_norm_eps": 1e-6, "hadamard": 128,
          "quant": {"ffn": 4, "attn": 4, "ple": 8, "emb": 4}}


def _load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def weights(bits, n, k, group, seed):
    """Seeded integer weights and scales: (q int8 [N, K], scales)."""
    rng = np.random.default_rng(seed)
    if bits == 4:
        q = rng.integers(-8, 8, size=(n, k), dtype=np.int8)
        s = rng.uniform(0.005, 0.02, size=(k // group, n)).astype(np.float16)
    else:
        q = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
        s = rng.uniform(0.001, 0.01, size=n).astype(np.float32)
    return q, s


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("FGM_REFERENCE") or os.path.join(
        os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "reference"))
    ap.add_argument("--out", default=os.path.join(HERE, "tiny.fgm"))
    args = ap.parse_args()
    fgm = _load(os.path.join(args.ref, "convert", "fgm.py"), "ref_fgm")
    quant = _load(os.path.join(args.ref, "convert", "quant.py"), "ref_quant")
    w = fgm.FgmWriter(args.out)
    w.start_body(1 << 14)
    for name, bits, n, k, group, had, twin, seed in LINEARS:
        q, s = weights(bits, n, k, group, seed)
        if bits == 4:
            blob = quant.pack_nibbles(quant.pack_b_tiles(q, n, k))
            w.add(name, blob, "q4g", shape=(n, k), meta={"hadamard": had, "group": group})
            w.add(name + ".scale", np.ascontiguousarray(s), "f16", shape=s.shape)
        else:
            w.add(name, quant.pack_b_tiles(q, n, k), "q8c", shape=(n, k), meta={"hadamard": had, "group": 0})
            w.add(name + ".scale", s, "f32", shape=s.shape)
        if twin:
            q8, s8 = weights(8, n, k, 0, seed + 100)
            w.add(name + ".i8", quant.pack_b_tiles(q8, n, k), "q8c", shape=(n, k),
                  meta={"hadamard": had, "group": 0})
            w.add(name + ".i8.scale", s8, "f32", shape=s8.shape)
    norm = np.random.default_rng(7).standard_normal(256).astype(np.float32)
    w.add("layers.0.input_layernorm.weight", norm, "f32", shape=norm.shape)
    w.meta["generator"] = "tests/golden/make_fgm_fixture.py"
    w.close(CONFIG)
    print(args.out, os.path.getsize(args.out), "bytes")


if __name__ == "__main__":
    main()

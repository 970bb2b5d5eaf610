"""Regenerate tests/golden/golden.npz from the reference itself (run in a container that has
the reference tree; the tests only read the committed .npz).

  - Q8_0 / Q4_K packed bytes from the reference converter's own packers
    (tools/convert_to_gguf.py quant_q8_0 / quant_q4_k), imported from the reference tree;
  - logits and the 51 named tensors of the reference's own CPU executor
    (src/mg-cpu/mg-cpu.cpp via oracle/_ref/libmgref.so) on the dequantised twin of a small
    synthetic Q8_0 / Q4_K model;
  - the token grid of the reference's own generate() (src/mg-generate.cpp) driven by the
    oracle forward on the small Q8_0 model.

usage: python tests/golden/make_golden.py /path/to/reference
   (or set MGC_REFERENCE_DIR; there is no default location)
"""
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
if len(sys.argv) > 1:
    REF = Path(sys.argv[1])
elif os.environ.get("MGC_REFERENCE_DIR"):
    REF = Path(os.environ["MGC_REFERENCE_DIR"])
else:
    sys.exit("usage: make_golden.py /path/to/reference  (or set MGC_REFERENCE_DIR)")
sys.path.insert(0, str(REF / "tools"))

import convert_to_gguf as cg  # noqa: E402  (the reference's packer)

from edge_maskgit_b200 import synth  # noqa: E402
from oracle import oracle as O  # noqa: E402

SMALL = dict(n_layer=2, n_tokens=16)


def weights():
    """Packer inputs with the edge cases the formats have."""
    rng = np.random.default_rng(1234)
    ws = []
    w = (rng.standard_normal((6, 512)) * 0.02).astype(np.float32)
    w[0, :32] = 0.0                       # all-zero block (d = 0)
    w[1, :] = np.abs(w[1, :])             # non-negative row (Q4_K min = 0)
    w[2, :] = -np.abs(w[2, :])            # non-positive row
    w[3, 5] = 0.3                         # outlier
    w[4, :256] = 0.01                     # constant super-block
    ws.append(w)
    ws.append(rng.uniform(-3, 3, (4, 768)).astype(np.float32))
    ws.append((rng.standard_normal((3, 256)) * 1e-6).astype(np.float32))   # fp16-subnormal scales
    return ws


def main():
    out = {}
    for i, w in enumerate(weights()):
        out[f"w{i}"] = w
        out[f"q8_{i}"] = np.frombuffer(cg.quant_q8_0(w), np.uint8)
        out[f"q4_{i}"] = np.frombuffer(cg.quant_q4_k(w), np.uint8)
    tmp = Path("/tmp/mg_golden")
    tmp.mkdir(exist_ok=True)
    for q in ("gq8", "gq4"):
        spec = synth.ModelSpec(quant=q, **SMALL)
        synth.make_model(tmp / f"{q}.gguf", spec, dequant_twin=tmp / f"{q}_f32.gguf")
        tok = synth.config1_tokens(spec)
        logits, named = O.ref_forward(tmp / f"{q}_f32.gguf", tok, spec.n_embd, spec.n_layer, spec.vocab_size,
                                      dump=True)
        for k, v in named.items():
            out[f"ref_{q}_{k}"] = v
    spec = synth.ModelSpec(quant="gq8", **SMALL)
    m = O.OracleModel(tmp / "gq8.gguf")
    out["ref_grid_gq8"] = O.ref_generate(tmp / "gq8.gguf", lambda t: m.forward(t), spec.vocab_size,
                                         spec.n_tokens, class_id=207, seed=42, steps=8)
    np.savez_compressed(Path(__file__).with_name("golden.npz"), **out)
    print("wrote", Path(__file__).with_name("golden.npz"))


if __name__ == "__main__":
    main()

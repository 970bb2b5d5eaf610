"""CPU: the Python GGUF reader and weight row slicing used by the tensor-parallel path."""
import numpy as np

from conftest import SMALL


def test_reader_round_trip_and_row_slices(tmp_path):
    from edge_maskgit_b200 import runtime as rt, synth
    from edge_maskgit_b200.gguf import GGUF
    for q, wt in (("gq8", 8), ("gq4", 12)):
        spec = synth.ModelSpec(quant=q, **SMALL)
        path = synth.make_model(tmp_path / f"{q}.gguf", spec)
        m = GGUF(path)
        assert m.hp("n_layer") == spec.n_layer and m.hp("n_embd") == spec.n_embd
        assert m["token_embd.weight"].f32().shape == (spec.vocab_size, spec.n_embd)
        w = m["blk.1.ffn_up.weight"]
        assert w.type == wt and w.ne == (spec.n_embd, spec.n_ffn)
        full = rt.dequant(wt, np.asarray(w.data), spec.n_ffn, spec.n_embd)
        a, b = 100, 612
        part = rt.dequant(wt, np.asarray(w.rows(a, b)), b - a, spec.n_embd)
        assert np.array_equal(part, full[a:b])

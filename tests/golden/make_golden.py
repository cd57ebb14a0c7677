"""Generate tests/golden/reference_vectors.npz with the REFERENCE's own compiled code.

Run in the development container, where oracle/Makefile can build oracle/_ref from the reference
sources:  python tests/golden/make_golden.py
Inputs are seeded synthetic GGUF blocks (the benchmark recipes) plus edge-case activations; the
outputs are what the reference's x86 Release build (oracle/_ref/libedgexpu_ref_avx2.so) returns:
activation bytes, linear outputs (cpu_kernel.c:545-644) and per-row logits scores with the greedy
choice (native.c:2355-2397 rule).
"""

import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
import _oracle  # noqa: E402

from test_oracle import edge_vectors  # noqa: E402


def main():
    assert _oracle.ensure_ref(), "reference library not buildable here"
    ref = _oracle.Ref(_oracle.REF_AVX2)
    _oracle.load_pkg()
    from edgexpu_llm_b200 import synth

    rng = np.random.default_rng(2024)
    out = {}
    for n in (64, 576):
        xs = np.stack(edge_vectors(n, rng))
        out[f"q8_0_x_{n}"] = xs
        out[f"q8_0_q_{n}"] = ref.quantize(xs, 8)
    for n in (256, 1024):
        xs = np.stack(edge_vectors(n, rng))
        out[f"q8_k_x_{n}"] = xs
        out[f"q8_k_q_{n}"] = ref.quantize(xs, 12)
    for tag, wtype, n_out, n_in, m in (("q8_0", 8, 24, 576, 3), ("q4_k", 12, 16, 1024, 2)):
        w = synth.weight(rng, wtype, n_out, n_in)
        x = synth.activations(rng, m, n_in)
        b = rng.standard_normal(n_out).astype(np.float32)
        out[f"lin_{tag}_w"], out[f"lin_{tag}_x"], out[f"lin_{tag}_b"] = w, x, b
        out[f"lin_{tag}_y"] = ref.linear(x, w, wtype, n_out, b)
    for tag, wtype, vocab, n_embd in (("q8_0", 8, 200, 64), ("q4_k", 12, 150, 512)):
        w = synth.weight(rng, wtype, vocab, n_embd)
        h = synth.activations(rng, 1, n_embd)[0]
        tok, _, scores = ref.logits(w, wtype, h, vocab)
        out[f"lg_{tag}_w"], out[f"lg_{tag}_h"] = w, h
        out[f"lg_{tag}_scores"], out[f"lg_{tag}_tok"] = scores, np.array([tok], np.int64)
    np.savez_compressed(HERE / "reference_vectors.npz", **out)
    print("wrote", HERE / "reference_vectors.npz", sum(v.nbytes for v in out.values()), "bytes")


if __name__ == "__main__":
    main()

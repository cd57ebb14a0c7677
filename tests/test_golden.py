"""Golden vectors produced by the reference's own compiled code (tests/golden/make_golden.py):
the oracle restatement (CPU) and the CUDA path (GPU) must reproduce them -- bytes exactly,
floats within 1e-5 * sum|w*x|, greedy ids exactly when the top-2 margin allows."""

import pathlib

import numpy as np
import pytest

from _oracle import TYPE_Q4_K, TYPE_Q8_0

GOLD = np.load(pathlib.Path(__file__).resolve().parent / "golden" / "reference_vectors.npz")
TYPES = {"q8_0": TYPE_Q8_0, "q4_k": TYPE_Q4_K}


def _check_logits(scores, tok, tag, port):
    w, h = GOLD[f"lg_{tag}_w"], GOLD[f"lg_{tag}_h"]
    want, want_tok = GOLD[f"lg_{tag}_scores"], int(GOLD[f"lg_{tag}_tok"][0])
    bound = port.logits_bound(w, TYPES[tag], h, range(len(want)))
    if scores is not None:
        assert np.all(np.abs(scores.astype(np.float64) - want) <= 1e-5 * bound)
    srt = np.sort(want)
    if srt[-1] - srt[-2] > 2e-5 * bound.max():
        assert tok == want_tok
    else:
        assert want[tok] >= srt[-1] - 2e-5 * bound.max()


@pytest.mark.parametrize("key", ["q8_0_64", "q8_0_576", "q8_k_256", "q8_k_1024"])
def test_oracle_quantize_matches_golden(port, key):
    kind, n = key.rsplit("_", 1)
    xs, q = GOLD[f"{kind}_x_{n}"], GOLD[f"{kind}_q_{n}"]
    np.testing.assert_array_equal(port.quantize(xs, TYPE_Q8_0 if kind == "q8_0" else TYPE_Q4_K), q)


@pytest.mark.parametrize("tag", ["q8_0", "q4_k"])
def test_oracle_linear_and_logits_match_golden(port, tag):
    w, x, b, y = (GOLD[f"lin_{tag}_{k}"] for k in "wxby")
    got = port.linear(x, w, TYPES[tag], w.shape[0], b)
    bound = port.linear_bound(x, w, TYPES[tag], w.shape[0])
    assert np.all(np.abs(got.astype(np.float64) - y) <= 1e-5 * bound + 1e-6 * np.abs(b))
    tok, _, scores = port.logits(GOLD[f"lg_{tag}_w"], TYPES[tag], GOLD[f"lg_{tag}_h"], len(GOLD[f"lg_{tag}_scores"]))
    _check_logits(scores, tok, tag, port)


@pytest.mark.gpu
@pytest.mark.parametrize("key", ["q8_0_64", "q8_0_576", "q8_k_256", "q8_k_1024"])
def test_gpu_quantize_matches_golden(gpu, key):
    kind, n = key.rsplit("_", 1)
    xs, q = GOLD[f"{kind}_x_{n}"], GOLD[f"{kind}_q_{n}"]
    wtype = TYPE_Q8_0 if kind == "q8_0" else TYPE_Q4_K
    got = np.stack([gpu.quantize(v, wtype) for v in xs])
    np.testing.assert_array_equal(got, q)


@pytest.mark.gpu
@pytest.mark.parametrize("tag", ["q8_0", "q4_k"])
def test_gpu_linear_and_logits_match_golden(gpu, port, tag):
    w, x, b, y = (GOLD[f"lin_{tag}_{k}"] for k in "wxby")
    h = gpu.upload_weight(w, TYPES[tag], w.shape[0], x.shape[1])
    try:
        got = gpu.linear_quant_batch(x, h, TYPES[tag], w.shape[0], b)
    finally:
        gpu.free_weight(h)
    bound = port.linear_bound(x, w, TYPES[tag], w.shape[0])
    assert np.all(np.abs(got.astype(np.float64) - y) <= 1e-5 * bound + 1e-6 * np.abs(b))
    lw, lh = GOLD[f"lg_{tag}_w"], GOLD[f"lg_{tag}_h"]
    h = gpu.upload_weight(lw, TYPES[tag], lw.shape[0], lh.size)
    try:
        tok, score = gpu.logits_greedy(h, TYPES[tag], lh, lw.shape[0])
    finally:
        gpu.free_weight(h)
    _check_logits(None, tok, tag, port)

"""GPU checks of the recorded synchronous calls (host buffers in and out).

edgexpu_cuda_linear_quant_batch and edgexpu_cuda_logits_argmax -- what the reference-named host
shim calls for every projection and every greedy token (cpu_kernel.c:545-644, native.c:2355-2397)
-- record their three launches (pull, product, finish) into a CUDA graph on the first call of a
shape and replay it afterwards.  A replay must read the new call's inputs and bias, not the
recorded call's; it must be recorded again once a scratch buffer moved, and dropped when a weight
is freed.  Every output is checked against the oracle (relaxed float order, 1e-5 * sum |w x|).
"""

import numpy as np
import pytest

from _oracle import TYPE_Q4_K, TYPE_Q8_0
from test_gpu_parity import TOL, assert_close
from test_oracle import _synth

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def relaxed_order(gpu):
    cuda = gpu.load_cuda()
    assert cuda.edgexpu_cuda_set_float_order(gpu.ORDER_RELAXED) == 1
    yield
    cuda.edgexpu_cuda_set_float_order(gpu.ORDER_X86)


def _check_linear(gpu, port, h, w, wtype, x, n_out, bias=None):
    got = gpu.linear_quant_batch(x, h, wtype, n_out, bias)
    want = port.linear(x, w, wtype, n_out, bias)
    bound = port.linear_bound(x, w, wtype, n_out)
    assert_close(got, want, bound, 1e-6 * (0 if bias is None else 1 + np.abs(bias)))
    return got


@pytest.mark.parametrize("wtype,n_out,n_in,m", [(TYPE_Q4_K, 512, 1024, 1), (TYPE_Q8_0, 300, 576, 3)])
def test_replayed_calls_read_each_calls_inputs(gpu, port, wtype, n_out, n_in, m):
    s = _synth()
    rng = np.random.default_rng(n_out + m)
    w = s.weight(rng, wtype, n_out, n_in)
    h = gpu.upload_weight(w, wtype, n_out, n_in)
    try:
        outs = []
        for i in range(4):  # call 0 records, calls 1..3 replay
            x = s.activations(rng, m, n_in)
            bias = rng.standard_normal(n_out).astype(np.float32) if i % 2 else None
            outs.append(_check_linear(gpu, port, h, w, wtype, x, n_out, bias))
        assert not np.array_equal(outs[1], outs[3])  # new inputs, new outputs
        # a larger call moves the scratch buffers; the first shape is then recorded again
        big_m = 12
        _check_linear(gpu, port, h, w, wtype, s.activations(rng, big_m, n_in), n_out)
        for _ in range(2):
            _check_linear(gpu, port, h, w, wtype, s.activations(rng, m, n_in), n_out)
    finally:
        gpu.free_weight(h)


def test_replay_dropped_when_the_weight_is_freed(gpu, port):
    s = _synth()
    rng = np.random.default_rng(9)
    n_out, n_in = 256, 512
    x = s.activations(rng, 1, n_in)
    for _ in range(3):  # same shape, a new tensor each time (possibly at the same address)
        w = s.weight(rng, TYPE_Q4_K, n_out, n_in)
        h = gpu.upload_weight(w, TYPE_Q4_K, n_out, n_in)
        try:
            for _ in range(2):
                _check_linear(gpu, port, h, w, TYPE_Q4_K, x, n_out)
        finally:
            gpu.free_weight(h)


@pytest.mark.parametrize("wtype,vocab,n_embd", [(TYPE_Q4_K, 3000, 1024), (TYPE_Q8_0, 4000, 576)])
def test_replayed_greedy_logits(gpu, port, wtype, vocab, n_embd):
    s = _synth()
    rng = np.random.default_rng(vocab)
    w = s.weight(rng, wtype, vocab, n_embd)
    h = gpu.upload_weight(w, wtype, vocab, n_embd)
    try:
        for i in range(4):
            hidden = s.activations(rng, 1, n_embd)[0]
            bias = rng.standard_normal(vocab).astype(np.float32) if i >= 2 else None
            tok, score = gpu.logits_greedy(h, wtype, hidden, vocab, bias)
            tok_o, score_o, scores = port.logits(w, wtype, hidden, vocab, bias)
            top2 = np.argsort(scores)[-2:]
            bound = port.logits_bound(w, wtype, hidden, [tok, tok_o, *top2])
            assert abs(score - score_o) <= TOL * bound.max() + (0 if bias is None else 1e-6 * (1 + abs(score_o)))
            if scores[top2[1]] - scores[top2[0]] > 2 * TOL * bound.max() + 1e-5:
                assert tok == tok_o
    finally:
        gpu.free_weight(h)

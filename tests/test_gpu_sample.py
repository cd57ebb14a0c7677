"""Temperature sampling on the device against the reference's own sampler.

* edgexpu_cuda_sample_softmax against edgexpu_cpu_sample_softmax (src/cpu_kernel.c:762-849,
  compiled from the reference in oracle/_ref) on the same logits and xorshift state: the same
  state afterwards, probabilities within 2 ulp, and the same id.
* edgexpu_cuda_logits_sample against the reference's temperature branch (native.c:2322-2353):
  the oracle's x86-order scores (bit-identical to the device's) divided by the temperature, then
  the reference sampler.
* End to end: the integrated runtime and the unchanged reference runtime sample the same ids at
  temperature 0.8, top_p 0.9 through the reference's own layer loop (the hidden states are
  bit-identical, so only the sampler could differ).

The device's exp and double sums follow a fixed order of their own (sample.cu); an id could
differ only when the draw lands within ~1e-7 of a running-sum boundary, which none of these
seeded cases does.
"""

import ctypes

import numpy as np
import pytest

import _oracle
from _oracle import TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_0

pytestmark = pytest.mark.gpu


def _ref_sampler():
    if not _oracle.ensure_ref():
        pytest.skip("reference library not built")
    lib = ctypes.CDLL(str(_oracle.REF_AVX2))
    f = lib.edgexpu_cpu_sample_softmax
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.POINTER(ctypes.c_uint64),
                  ctypes.POINTER(ctypes.c_uint32)]
    return f


def _ref_sample(f, logits, top_p, state):
    io = np.ascontiguousarray(logits, np.float32).copy()
    rng = ctypes.c_uint64(state)
    out = ctypes.c_uint32(0xFFFFFFFF)
    assert f(io.ctypes.data, io.size, top_p, ctypes.byref(rng), ctypes.byref(out)) == 1
    return out.value, rng.value, io


def _dev_sample(cuda, logits, top_p, state):
    io = np.ascontiguousarray(logits, np.float32).copy()
    rng = ctypes.c_uint64(state)
    out = ctypes.c_uint32(0xFFFFFFFF)
    err = ctypes.create_string_buffer(256)
    assert cuda.edgexpu_cuda_sample_softmax(io.ctypes.data, io.size, top_p, ctypes.byref(rng), ctypes.byref(out), err,
                                            256), err.value
    return out.value, rng.value, io


CASES = [(n, scale, top_p) for n in (1, 7, 1000, 49152, 128256) for scale in (0.5, 4.0, 30.0)
         for top_p in (0.0, 0.5, 0.9, 1.0)]


@pytest.mark.parametrize("n,scale,top_p", CASES)
def test_sample_softmax_matches_reference(gpu, n, scale, top_p):
    f = _ref_sampler()
    cuda = gpu.load_cuda()
    rng = np.random.default_rng(n * 7 + int(scale * 10) + int(top_p * 100))
    logits = (rng.standard_normal(n) * scale).astype(np.float32)
    if n >= 1000:
        logits[rng.integers(0, n, 5)] = logits.max()  # exact ties: the lower id first
    for state in (0, 0x12345678ABCDEF, int(rng.integers(1, 2**63))):
        want, want_rng, p_ref = _ref_sample(f, logits, top_p, state)
        got, got_rng, p_dev = _dev_sample(cuda, logits, top_p, state)
        assert got_rng == want_rng
        np.testing.assert_allclose(p_dev, p_ref, rtol=2.5e-7, atol=1e-45)
        assert got == want, f"state {state:#x}: device id {got}, reference id {want}"


@pytest.mark.parametrize("wtype,vocab,n_embd", [(TYPE_Q8_0, 49152, 576), (TYPE_Q4_K, 1000, 512),
                                                (TYPE_Q6_K, 777, 256)])
@pytest.mark.parametrize("temperature,top_p", [(0.7, 0.9), (1.0, 1.0), (1.3, 0.5)])
def test_logits_sample_matches_reference_branch(gpu, port, wtype, vocab, n_embd, temperature, top_p):
    from test_oracle import _synth

    f = _ref_sampler()
    cuda = gpu.load_cuda()
    assert cuda.edgexpu_cuda_set_float_order(gpu.ORDER_X86) == 1
    rng = np.random.default_rng(vocab + n_embd)
    w = _synth().weight(rng, wtype, vocab, n_embd)
    hidden = _synth().activations(rng, 1, n_embd)[0] * 3.0
    bias = rng.standard_normal(vocab).astype(np.float32) * 0.1
    _, _, scores = port.logits(w, wtype, hidden, vocab, bias, x86=True)
    logits = (np.asarray(scores, np.float32) / np.float32(temperature)).astype(np.float32)  # native.c:2338
    h = gpu.upload_weight(w, wtype, vocab, n_embd)
    try:
        for state in (0, 987654321):
            want, want_rng, _ = _ref_sample(f, logits, top_p, state)
            st = ctypes.c_uint64(state)
            tok = ctypes.c_uint32(0xFFFFFFFF)
            err = ctypes.create_string_buffer(256)
            assert cuda.edgexpu_cuda_logits_sample(h, wtype, hidden.ctypes.data, n_embd, vocab, bias.ctypes.data,
                                                   temperature, top_p, ctypes.byref(st), ctypes.byref(tok), err, 256), \
                err.value
            assert st.value == want_rng and tok.value == want
    finally:
        gpu.free_weight(h)


def test_sampled_decode_through_reference_loop_matches(tmp_path):
    """Config 1's model (8 layers), 32-token prompt, 48 tokens at temperature 0.8 / top_p 0.9."""
    from test_e2e_native import B200_RUNTIME, REF_RUNTIME, _bind

    from edgexpu_llm_b200 import gguf_synth as gs

    shape = gs.SMOLLM2_135M_Q8_0.with_layers(8)
    path = gs.write_llama_gguf(tmp_path / "s.gguf", shape, seed=4)
    prompt = gs.prompt_ids(shape, 32, seed=4)
    ids = {}
    for name, lib_path in (("ref", REF_RUNTIME), ("b200", B200_RUNTIME)):
        fn = _bind(lib_path).edgexpu_generate_run
        fn.restype = ctypes.c_int
        fn.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                       ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
        out = np.zeros(48, np.uint32)
        err = ctypes.create_string_buffer(1024)
        made = fn(str(path).encode(), prompt.ctypes.data, prompt.size, 48, 0.8, 0.9, out.ctypes.data, None, 0, None,
                  err, 1024)
        assert made == 48, err.value
        ids[name] = out
    np.testing.assert_array_equal(ids["b200"], ids["ref"])
    assert len(set(ids["ref"].tolist())) > 4  # really sampled, not a fixed point

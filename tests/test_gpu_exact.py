"""GPU outputs in the reference x86 build's float order: bit-identical, not just within tolerance.

The default float order of the C ABI (EDGEXPU_CUDA_ORDER_X86, include/edgexpu_cuda.h) sums the exact
integer partials in the same float steps as the reference's x86 Release build (AVX2 + FMA SIMD
branches of gguf_dot_q8.c and gguf_quant.c).  The oracle's x86-order restatement is pinned bit for
bit to that build (tests/test_oracle.py::test_x86_order_*), so every float the GPU writes here must
equal the oracle's bits: linear outputs for all six GGUF types at several batch sizes (one and
several GEMV passes, Q4_K prefill-sized batches included), grouped launches, and the greedy logits
(scores and chosen ids, ties and biases included).
"""

import ctypes

import numpy as np
import pytest

from _oracle import TYPE_Q4_0, TYPE_Q4_K, TYPE_Q5_0, TYPE_Q5_K, TYPE_Q6_K, TYPE_Q8_0
from test_gpu_parity import _stream, _sync, _torch
from test_oracle import _synth

pytestmark = pytest.mark.gpu

ALL = (TYPE_Q4_0, TYPE_Q5_0, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K)


def _k(wtype, nblocks):
    return nblocks * (32 if wtype in (TYPE_Q4_0, TYPE_Q5_0, TYPE_Q8_0) else 256)


def bits_equal(got, want, what=""):
    g = np.ascontiguousarray(got, np.float32).view(np.uint32)
    w = np.ascontiguousarray(want, np.float32).view(np.uint32)
    bad = np.argwhere(g != w)
    assert bad.size == 0, f"{what}: {bad.shape[0]} outputs differ, first {bad[:3].tolist()}: " \
        f"{np.asarray(got).flat[0] if bad.size == 0 else np.asarray(got)[tuple(bad[0])]!r} vs " \
        f"{np.asarray(want)[tuple(bad[0])]!r}"


@pytest.fixture(autouse=True)
def x86_order(gpu):
    assert gpu.load_cuda().edgexpu_cuda_float_order() == gpu.ORDER_X86


@pytest.mark.parametrize("wtype", ALL)
@pytest.mark.parametrize("n_out,nblk,m", [(333, 16, 1), (97, 7, 2), (64, 18, 5), (130, 3, 8), (41, 4, 13)])
def test_linear_bit_identical_to_x86_reference(gpu, port, wtype, n_out, nblk, m):
    s = _synth()
    n_in = _k(wtype, nblk)
    rng = np.random.default_rng(wtype * 977 + n_out + m)
    w = s.weight(rng, wtype, n_out, n_in)
    x = s.activations(rng, m, n_in)
    x[:, 1::9] = 0.0
    bias = rng.standard_normal(n_out).astype(np.float32) if m % 2 else None
    h = gpu.upload_weight(w, wtype, n_out, n_in)
    try:
        got = gpu.linear_quant_batch(x, h, wtype, n_out, bias)
    finally:
        gpu.free_weight(h)
    bits_equal(got, port.linear(x, w, wtype, n_out, bias, x86=True), f"type {wtype}")


@pytest.mark.parametrize("m", [64, 130])
def test_q4_k_prefill_batches_bit_identical(gpu, port, m):
    """In the x86 order prefill-sized Q4_K batches take the GEMV (several passes), not the GEMM."""
    s = _synth()
    n_out, n_in = 200, 1024
    rng = np.random.default_rng(m)
    w = s.weight(rng, TYPE_Q4_K, n_out, n_in)
    x = s.activations(rng, m, n_in)
    h = gpu.upload_weight(w, TYPE_Q4_K, n_out, n_in)
    try:
        got = gpu.linear_quant_batch(x, h, TYPE_Q4_K, n_out)
    finally:
        gpu.free_weight(h)
    bits_equal(got, port.linear(x, w, TYPE_Q4_K, n_out, None, x86=True), f"m {m}")


def test_grouped_launch_bit_identical(gpu, port):
    torch = _torch()
    cuda = gpu.load_cuda()
    s = _synth()
    rng = np.random.default_rng(5)
    n_in, m, sizes = 2048, 3, (512, 128, 128)
    ws = [s.weight(rng, TYPE_Q4_K, n, n_in) for n in sizes]
    x = s.activations(rng, m, n_in)
    hs = [gpu.upload_weight(w, TYPE_Q4_K, n, n_in) for w, n in zip(ws, sizes)]
    try:
        xd = torch.from_numpy(x).cuda()
        outs = [torch.empty((m, n), dtype=torch.float32, device="cuda") for n in sizes]
        P = ctypes.c_void_p * 3
        ok = cuda.edgexpu_cuda_linear_quant_multi_dev(3, P(*[o.data_ptr() for o in outs]), P(*hs),
                                                      (ctypes.c_int * 3)(*sizes), None, TYPE_Q4_K, xd.data_ptr(),
                                                      m, n_in, _stream())
        assert ok, cuda.edgexpu_cuda_last_error()
        _sync(gpu)
        for w, n, o in zip(ws, sizes, outs):
            bits_equal(o.cpu().numpy(), port.linear(x, w, TYPE_Q4_K, n, None, x86=True), f"segment {n}")
    finally:
        for h in hs:
            gpu.free_weight(h)


@pytest.mark.parametrize("wtype", ALL)
@pytest.mark.parametrize("with_bias", [False, True])
def test_logits_bit_identical_to_x86_reference(gpu, port, wtype, with_bias):
    s = _synth()
    n_in = _k(wtype, 18 if wtype in (TYPE_Q4_0, TYPE_Q5_0, TYPE_Q8_0) else 3)
    vocab = 3001
    rng = np.random.default_rng(wtype + 11 * with_bias)
    w = s.weight(rng, wtype, vocab, n_in)
    hid = s.activations(rng, 1, n_in)[0]
    bias = rng.standard_normal(vocab).astype(np.float32) * 0.1 if with_bias else None
    # plant an exact tie at the top: a copy of the best row at a higher id must not win
    best0 = port.logits(w, wtype, hid, vocab, bias, x86=True)[0]
    w[2999] = w[best0]
    if bias is not None:
        bias[2999] = bias[best0]
    tok_o, score_o, _ = port.logits(w, wtype, hid, vocab, bias, x86=True)
    h = gpu.upload_weight(w, wtype, vocab, n_in)
    try:
        tok, score = gpu.logits_greedy(h, wtype, hid, vocab, bias)
    finally:
        gpu.free_weight(h)
    assert tok == tok_o == best0
    bits_equal(np.float32(score), np.float32(score_o), "best score")


def test_host_shim_quantized_dots_bit_identical(gpu, port, ref):
    """edgexpu_gguf_dot_quant_q8 / _q8k through the host shim equal the reference build's values."""
    host = gpu.load_host()
    s = _synth()
    for wtype in ALL:
        n = _k(wtype, 8 if wtype in (TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K) else 24)
        rng = np.random.default_rng(wtype + 1234)
        w = s.weight(rng, wtype, 4, n)
        xq = port.quantize(s.activations(rng, 1, n), wtype)[0]
        fn = host.edgexpu_gguf_dot_quant_q8 if wtype in (TYPE_Q4_0, TYPE_Q5_0, TYPE_Q8_0) else host.edgexpu_gguf_dot_quant_q8k
        for o in range(4):
            got = np.float32(fn(wtype, w[o].ctypes.data, xq.ctypes.data, n))
            bits_equal(got, np.float32(ref.dot_q8(wtype, w[o], xq, n)), f"type {wtype} row {o}")

"""GPU parity for the other GGUF weight types behind the same dispatch (Q4_0, Q5_0, Q5_K, Q6_K, and
F16/F32 weights), the single-row quant API of the host shim, and row dequantization.

The bars are those of test_gpu_parity.py: per-block int32 partials bit-exact with the oracle (which
tests/test_oracle.py pins to the reference build), fp32 outputs within 1e-5 * sum_k |w_k * x_k|,
dequantized rows bit-identical, greedy ids identical whenever the top-2 margin exceeds the
tolerance.  Shapes include rows whose blocks are only 2-byte aligned (Q4_0 / Q5_0 / Q6_K with an odd
block count) and batches above the GEMV's 8 rows per launch.
"""

import ctypes

import numpy as np
import pytest

from _oracle import TYPE_Q4_0, TYPE_Q4_K, TYPE_Q5_0, TYPE_Q5_K, TYPE_Q6_K, TYPE_Q8_0
from test_gpu_parity import _stream, _sync, _torch, assert_close
from test_oracle import _synth

pytestmark = pytest.mark.gpu

TOL = 1e-5
OTHER = (TYPE_Q4_0, TYPE_Q5_0, TYPE_Q5_K, TYPE_Q6_K)
TYPE_F32, TYPE_F16 = 0, 1


def _k(wtype, nblocks):
    return nblocks * (32 if wtype in (TYPE_Q4_0, TYPE_Q5_0, TYPE_Q8_0) else 256)


@pytest.mark.parametrize("wtype", OTHER)
@pytest.mark.parametrize("n_out,nblk,m", [(300, 16, 1), (257, 7, 2), (1000, 16, 3), (64, 56, 8), (129, 3, 16)])
def test_linear_other_types(gpu, port, wtype, n_out, nblk, m):
    s = _synth()
    n_in = _k(wtype, nblk)
    rng = np.random.default_rng(wtype * 1000 + n_out + m)
    w = s.weight(rng, wtype, n_out, n_in)
    x = s.activations(rng, m, n_in)
    bias = rng.standard_normal(n_out).astype(np.float32)
    h = gpu.upload_weight(w, wtype, n_out, n_in)
    try:
        got = gpu.linear_quant_batch(x, h, wtype, n_out, bias)
    finally:
        gpu.free_weight(h)
    want = port.linear(x, w, wtype, n_out, bias)
    assert_close(got, want, port.linear_bound(x, w, wtype, n_out), 1e-6 * np.abs(bias))


@pytest.mark.parametrize("wtype", OTHER)
@pytest.mark.parametrize("n_out,nblk,m", [(97, 16, 1), (40, 5, 3), (33, 9, 8)])
def test_block_partials_other_types(gpu, port, wtype, n_out, nblk, m):
    torch = _torch()
    s = _synth()
    n_in = _k(wtype, nblk)
    rng = np.random.default_rng(wtype + n_out + m)
    w = s.weight(rng, wtype, n_out, n_in)
    xq = port.quantize(s.activations(rng, m, n_in), wtype)
    want = port.partials(w, xq, wtype, n_in)
    h = gpu.upload_weight(w, wtype, n_out, n_in)
    try:
        xq_d = torch.from_numpy(xq).cuda()
        got = torch.empty(want.size, dtype=torch.int32, device="cuda")
        assert gpu.load_cuda().edgexpu_cuda_block_partials_dev(got.data_ptr(), xq_d.data_ptr(), h, wtype, m, n_out,
                                                               n_in, _stream())
        _sync(gpu)
        np.testing.assert_array_equal(got.cpu().numpy().reshape(want.shape), want)
    finally:
        gpu.free_weight(h)


def test_q6_k_partials_at_accumulator_extremes(gpu, port):
    """Q6_K with every scale -128 and every quant at 0 (value -32) against an activation of +-127:
    the largest |sumi| the format allows, still exact in int32."""
    torch = _torch()
    n_in, n_out = 512, 4
    w = np.zeros((n_out, 2, 210), np.uint8)
    w[:, :, 192:208] = np.uint8(0x80)  # int8 scale -128
    w[:, :, 208:210] = np.array([0x3C00], np.uint16).view(np.uint8)
    w[1, :, :128] = 0xFF  # quants 63 (value +31) in row 1
    w[1, :, 128:192] = 0xFF
    w = w.reshape(n_out, 420)
    x = np.where(np.arange(n_in) % 2 == 0, 1.0, -1.0).astype(np.float32)[None].repeat(2, 0)
    x[1] = 1.0
    xq = port.quantize(x, TYPE_Q6_K)
    want = port.partials(w, xq, TYPE_Q6_K, n_in)
    h = gpu.upload_weight(w, TYPE_Q6_K, n_out, n_in)
    try:
        xq_d = torch.from_numpy(xq).cuda()
        got = torch.empty(want.size, dtype=torch.int32, device="cuda")
        assert gpu.load_cuda().edgexpu_cuda_block_partials_dev(got.data_ptr(), xq_d.data_ptr(), h, TYPE_Q6_K, 2,
                                                               n_out, n_in, _stream())
        _sync(gpu)
        np.testing.assert_array_equal(got.cpu().numpy().reshape(want.shape), want)
        assert abs(int(want[1, 0, 0, 0])) == 128 * 32 * 127 * 256
    finally:
        gpu.free_weight(h)


@pytest.mark.parametrize("wtype", OTHER)
def test_logits_other_types(gpu, port, wtype):
    s = _synth()
    n_in = _k(wtype, 8 if wtype in (TYPE_Q5_K, TYPE_Q6_K) else 18)
    vocab = 5000
    rng = np.random.default_rng(wtype + 77)
    w = s.weight(rng, wtype, vocab, n_in)
    w[4000] = w[123]  # an exact tie: the lower id wins
    hid = s.activations(rng, 1, n_in)[0]
    h = gpu.upload_weight(w, wtype, vocab, n_in)
    try:
        tok, score = gpu.logits_greedy(h, wtype, hid, vocab)
    finally:
        gpu.free_weight(h)
    tok_o, score_o, scores = port.logits(w, wtype, hid, vocab)
    bound = port.logits_bound(w, wtype, hid, [tok_o, tok])
    srt = np.sort(scores)
    if srt[-1] - srt[-2] > 2 * TOL * bound.max():
        assert tok == tok_o
    assert abs(float(scores[tok]) - score_o) <= 2 * TOL * bound.max()
    assert tok != 4000


@pytest.mark.parametrize("wtype", (TYPE_F32, TYPE_F16))
def test_float_weights_linear_and_logits(gpu, wtype):
    """F16/F32 weights take the fp32 activations (cpu_kernel.c:565-568, :633-643; logit_dot_row)."""
    rng = np.random.default_rng(wtype + 3)
    n_out, n_in, m = 333, 576, 3
    wf = (rng.standard_normal((n_out, n_in)) * 0.02).astype(np.float32)
    w = wf.astype(np.float16) if wtype == TYPE_F16 else wf
    wd = w.astype(np.float64)
    x = rng.standard_normal((m, n_in)).astype(np.float32)
    bias = rng.standard_normal(n_out).astype(np.float32)
    h = gpu.upload_weight(w.view(np.uint8).reshape(n_out, -1), wtype, n_out, n_in)
    try:
        got = gpu.linear_quant_batch(x, h, wtype, n_out, bias)
        tok, _ = gpu.logits_greedy(h, wtype, x[0], n_out)
    finally:
        gpu.free_weight(h)
    want = x.astype(np.float64) @ wd.T + bias
    bound = np.abs(x.astype(np.float64)) @ np.abs(wd).T
    assert_close(got, want, bound, 1e-6 * np.abs(bias))
    scores = x[0].astype(np.float64) @ wd.T
    srt = np.sort(scores)
    if srt[-1] - srt[-2] > 1e-4:
        assert tok == int(np.argmax(scores))


@pytest.mark.parametrize("wtype", OTHER + (TYPE_Q8_0, TYPE_Q4_K))
def test_host_shim_single_row_dots(gpu, port, ref, wtype):
    """edgexpu_gguf_dot_quant_q8 / _q8k / edgexpu_gguf_dot_quant through the host shim, for a row
    in host memory (the reference's mmap'd bytes) and a row of an uploaded tensor."""
    host = gpu.load_host()
    s = _synth()
    n = _k(wtype, 4 if wtype in (TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K) else 24)
    rng = np.random.default_rng(wtype + 500)
    w = s.weight(rng, wtype, 3, n)
    x = s.activations(rng, 1, n)[0]
    xq = port.quantize(x, wtype)[0]
    qfn = host.edgexpu_gguf_dot_quant_q8 if wtype in (TYPE_Q4_0, TYPE_Q5_0, TYPE_Q8_0) else host.edgexpu_gguf_dot_quant_q8k
    h = gpu.upload_weight(w, wtype, 3, n)
    try:
        host.edgexpu_b200_clear_error()
        for o in range(3):
            want_q = ref.dot_q8(wtype, w[o], xq, n)
            want_f = ref.dot_f32(wtype, w[o], x, n)
            bq = port.lib.eo_abs_bound_q8(wtype, w[o].ctypes.data, xq.ctypes.data, n)
            bf = port.lib.eo_abs_bound_f32(wtype, w[o].ctypes.data, x.ctypes.data, n)
            rb = w.shape[1]
            for wrow in (w[o].ctypes.data, h + o * rb):
                assert abs(qfn(wtype, wrow, xq.ctypes.data, n) - want_q) <= TOL * bq
                assert abs(host.edgexpu_gguf_dot_quant(wtype, wrow, x.ctypes.data, n) - want_f) <= TOL * bf
        assert host.edgexpu_b200_last_error() == b""
        # the reference's invalid-argument answers: 0.0f, no error
        assert qfn(wtype, w[0].ctypes.data, xq.ctypes.data, n + 1) == 0.0
        assert host.edgexpu_gguf_dot_quant(99, w[0].ctypes.data, x.ctypes.data, n) == 0.0
        other = host.edgexpu_gguf_dot_quant_q8k if qfn == host.edgexpu_gguf_dot_quant_q8 else host.edgexpu_gguf_dot_quant_q8
        assert other(wtype, w[0].ctypes.data, xq.ctypes.data, n) == 0.0
        assert host.edgexpu_b200_last_error() == b""
    finally:
        gpu.free_weight(h)


@pytest.mark.parametrize("wtype", OTHER + (TYPE_Q8_0, TYPE_Q4_K))
def test_dequantize_rows_bit_exact(gpu, port, wtype):
    torch = _torch()
    cuda = gpu.load_cuda()
    s = _synth()
    n = _k(wtype, 3 if wtype in (TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K) else 19)
    rows = 50
    rng = np.random.default_rng(wtype + 900)
    w = s.weight(rng, wtype, rows, n)
    want = np.empty((rows, n), np.float32)
    for r in range(rows):
        assert port.lib.eo_dequantize_row(wtype, w[r].ctypes.data, n, want[r].ctypes.data)
    h = gpu.upload_weight(w, wtype, rows, n)
    buf = ctypes.create_string_buffer(512)
    try:
        one = np.empty(n, np.float32)
        assert cuda.edgexpu_cuda_dequantize_row(h, wtype, 17, n, one.ctypes.data, buf, 512), buf.value
        np.testing.assert_array_equal(one.view(np.uint32), want[17].view(np.uint32))
        assert cuda.edgexpu_cuda_dequantize_row(h, wtype, rows, n, one.ctypes.data, buf, 512) == 0
        ids = np.array([3, 49, 0, 3, 17], np.int32)
        ids_d = torch.from_numpy(ids).cuda()
        out = torch.empty((len(ids), n), dtype=torch.float32, device="cuda")
        assert cuda.edgexpu_cuda_dequantize_rows_dev(out.data_ptr(), h, wtype, ids_d.data_ptr(), len(ids), n, _stream())
        _sync(gpu)
        np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), want[ids].view(np.uint32))
        bad = torch.tensor([1, rows], dtype=torch.int32, device="cuda")
        assert cuda.edgexpu_cuda_dequantize_rows_dev(out.data_ptr(), h, wtype, bad.data_ptr(), 2, n, _stream())
        assert cuda.edgexpu_cuda_stream_sync(_stream(), buf, 512) == 0
        assert b"outside the tensor" in buf.value
        o = out.cpu().numpy()
        np.testing.assert_array_equal(o[0].view(np.uint32), want[1].view(np.uint32))
        assert np.all(np.isnan(o[1]))
    finally:
        gpu.free_weight(h)


def test_can_dot_agrees_with_the_gpu_path(gpu):
    host = gpu.load_host()
    for t in (TYPE_Q4_0, TYPE_Q5_0, TYPE_Q8_0):
        assert host.edgexpu_gguf_can_dot_q8(t) == 1 and host.edgexpu_gguf_can_dot_q8k(t) == 0
    for t in (TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K):
        assert host.edgexpu_gguf_can_dot_q8(t) == 0 and host.edgexpu_gguf_can_dot_q8k(t) == 1
    for t in (3, 7, 9, 10, 11, 15):
        assert host.edgexpu_gguf_can_dot_q8(t) == 0 and host.edgexpu_gguf_can_dot_q8k(t) == 0

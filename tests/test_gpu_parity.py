"""GPU parity tests: the CUDA path (through the C ABI and the reference-named C host shim)
against the oracle on identical seeded inputs.

Bars (from the task's north star):
* activation Q8 bytes and per-block int32 partials: bit-exact;
* fp32 outputs: |gpu - oracle| <= 1e-5 * sum_k |w_k * x_k| (bound computed by the oracle);
* greedy token ids: identical whenever the top-2 score margin exceeds the tolerance.
"""

import ctypes

import numpy as np
import pytest

from _oracle import TYPE_Q4_K, TYPE_Q8_0
from test_oracle import _synth, edge_vectors

pytestmark = pytest.mark.gpu

TOL = 1e-5


def _torch():
    import torch

    return torch


def _stream():
    return _torch().cuda.current_stream().cuda_stream


def _sync(gpu):
    buf = ctypes.create_string_buffer(512)
    ok = gpu.load_cuda().edgexpu_cuda_stream_sync(_stream(), buf, 512)
    assert ok, buf.value


def assert_close(got, want, bound, extra=0.0):
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    lim = TOL * bound + extra + 1e-30
    bad = np.argwhere(err > lim)
    assert bad.size == 0, f"{bad.shape[0]} outputs out of tolerance, first {bad[:3].tolist()}: " \
        f"err {err[tuple(bad[0])]:.3e} lim {lim[tuple(bad[0])] if np.ndim(lim) else lim:.3e}"


# ---- activation quantizers ---------------------------------------------------------------------


@pytest.mark.parametrize("n", [32, 576, 1536, 4096])
def test_quantize_q8_0_bit_exact(gpu, port, n):
    rng = np.random.default_rng(n)
    for v in edge_vectors(n, rng):
        np.testing.assert_array_equal(gpu.quantize(v, TYPE_Q8_0), port.quantize(v, TYPE_Q8_0)[0])


@pytest.mark.parametrize("n", [256, 4096, 14336])
def test_quantize_q8_k_bit_exact(gpu, port, n):
    rng = np.random.default_rng(n + 1)
    for v in edge_vectors(n, rng):
        np.testing.assert_array_equal(gpu.quantize(v, TYPE_Q4_K), port.quantize(v, TYPE_Q4_K)[0])


def test_quantize_through_reference_names(gpu, port):
    host = gpu.load_host()
    rng = np.random.default_rng(5)
    x = rng.standard_normal(4096).astype(np.float32)
    q0 = np.empty(4096 // 32 * 34, np.uint8)
    qk = np.empty(4096 // 256 * 292, np.uint8)
    assert host.edgexpu_gguf_quantize_q8_0(x.ctypes.data, 4096, q0.ctypes.data) == 1
    assert host.edgexpu_gguf_quantize_q8_k(x.ctypes.data, 4096, qk.ctypes.data) == 1
    np.testing.assert_array_equal(q0, port.quantize(x, TYPE_Q8_0)[0])
    np.testing.assert_array_equal(qk, port.quantize(x, TYPE_Q4_K)[0])
    assert host.edgexpu_gguf_quantize_q8_k(x.ctypes.data, 100, qk.ctypes.data) == 0


def test_quantize_dev_batch_bit_exact(gpu, port):
    torch = _torch()
    rng = np.random.default_rng(9)
    for wtype, n in ((TYPE_Q8_0, 1536), (TYPE_Q4_K, 14336)):
        x = rng.standard_normal((16, n)).astype(np.float32)
        xd = torch.from_numpy(x).cuda()
        q = torch.empty(16 * gpu.act_row_bytes(wtype, n), dtype=torch.uint8, device="cuda")
        assert gpu.load_cuda().edgexpu_cuda_quantize_dev(wtype, xd.data_ptr(), 16, n, q.data_ptr(), _stream())
        _sync(gpu)
        np.testing.assert_array_equal(q.cpu().numpy().reshape(16, -1), port.quantize(x, wtype))


# ---- per-block int32 partials of the production kernel ----------------------------------------


@pytest.mark.parametrize("wtype,n_out,n_in,m", [
    (TYPE_Q8_0, 1536, 576, 4),
    (TYPE_Q8_0, 37, 14336, 2),
    (TYPE_Q4_K, 300, 4096, 3),
    (TYPE_Q4_K, 33, 14336, 2),
])
def test_block_partials_bit_exact(gpu, port, wtype, n_out, n_in, m):
    torch = _torch()
    s = _synth()
    rng = np.random.default_rng(n_out + n_in)
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


# ---- linear (the drop-in edgexpu_cpu_linear_quant_batch) --------------------------------------

LINEAR_CASES = [
    # config 0: Q8_0 GEMV 1536x576 at batch 1, 4, 16
    (TYPE_Q8_0, 1536, 576, 1, False),
    (TYPE_Q8_0, 1536, 576, 4, True),
    (TYPE_Q8_0, 1536, 576, 16, False),
    # the other SmolLM2-shaped projections
    (TYPE_Q8_0, 576, 1536, 1, False),
    (TYPE_Q8_0, 192, 576, 3, False),
    # config 2: Q4_K GEMV sweep shapes at batch 1, 8, 16
    (TYPE_Q4_K, 4096, 4096, 1, False),
    (TYPE_Q4_K, 4096, 4096, 8, True),
    (TYPE_Q4_K, 14336, 4096, 16, False),
    (TYPE_Q4_K, 4096, 14336, 1, False),
    (TYPE_Q4_K, 4096, 14336, 16, False),
    # ragged / edge shapes
    (TYPE_Q8_0, 1, 32, 1, True),
    (TYPE_Q8_0, 7, 64, 5, False),
    (TYPE_Q8_0, 1001, 14336, 2, False),
    (TYPE_Q4_K, 1, 256, 1, False),
    (TYPE_Q4_K, 13, 768, 40, True),
    (TYPE_Q4_K, 999, 2048, 2, False),
    # rows longer than a 32 KB stage -> one-row tiles: each warp owns every 15th tile and skips the
    # rest, so it can reach a stage's next fill before the previous one landed (~28 tiles per CTA)
    (TYPE_Q8_0, 4096, 16384, 1, False),
    # Q4_K rows of more than 32 units at batch 1 (relaxed order: sliced rows): 7 full slices, a
    # partly filled last slice (K = 7168, 11008), an odd tile height, and 15 slices (K = 30720)
    (TYPE_Q4_K, 4096, 14336, 1, True),
    (TYPE_Q4_K, 777, 7168, 1, False),
    (TYPE_Q4_K, 301, 11008, 1, True),
    (TYPE_Q4_K, 95, 30720, 1, False),
]


@pytest.fixture(params=["x86", "relaxed"])
def order(request, gpu):
    """Both float orders of the library: the x86 order (the default) and the relaxed order, whose
    kernels differ (sliced rows for K > 4096 at batch 1, the tensor-core GEMM for Q4_K prefill)."""
    cuda = gpu.load_cuda()
    assert cuda.edgexpu_cuda_set_float_order(gpu.ORDER_X86 if request.param == "x86" else gpu.ORDER_RELAXED) == 1
    yield request.param
    cuda.edgexpu_cuda_set_float_order(gpu.ORDER_X86)


@pytest.mark.parametrize("wtype,n_out,n_in,m,with_bias", LINEAR_CASES)
def test_linear_quant_batch_matches_oracle(gpu, port, wtype, n_out, n_in, m, with_bias, order):
    s = _synth()
    rng = np.random.default_rng(n_out * 31 + n_in + m)
    w = s.weight(rng, wtype, n_out, n_in)
    x = s.activations(rng, m, n_in)
    bias = rng.standard_normal(n_out).astype(np.float32) if with_bias else None
    h = gpu.upload_weight(w, wtype, n_out, n_in)
    try:
        got = gpu.linear_quant_batch(x, h, wtype, n_out, bias)
    finally:
        gpu.free_weight(h)
    want = port.linear(x, w, wtype, n_out, bias)
    bound = port.linear_bound(x, w, wtype, n_out)
    assert_close(got, want, bound, 0.0 if bias is None else 1e-7 * np.abs(bias)[None, :] + 1e-6)


def test_linear_logits_shape_q4_k(gpu, port):
    """config 2's largest GEMV (128256 x 4096, 295 MB) at batch 1."""
    s = _synth()
    rng = np.random.default_rng(128256)
    w = s.q4_k_weight(rng, 128256, 4096)
    x = s.activations(rng, 1, 4096)
    h = gpu.upload_weight(w, TYPE_Q4_K, 128256, 4096)
    try:
        got = gpu.linear_quant_batch(x, h, TYPE_Q4_K, 128256)
    finally:
        gpu.free_weight(h)
    assert_close(got, port.linear(x, w, TYPE_Q4_K, 128256), port.linear_bound(x, w, TYPE_Q4_K, 128256))


@pytest.mark.parametrize("wtype,n_out,n_in", [(TYPE_Q4_K, 4096, 14336), (TYPE_Q4_K, 1024, 4096),
                                               (TYPE_Q8_0, 1536, 576)])
@pytest.mark.parametrize("m", [1, 2])
def test_fused_quantization_prologue_is_bit_exact(gpu, port, wtype, n_out, n_in, m):
    """At m <= 2 the GEMV quantizes the fp32 activations in its own prologue.  Fed the oracle's
    quantized bytes instead (the pre-quantized path of the same kernel), it must give the same
    output bits -- so the fused quantization is bit-exact, incl. zero blocks, sign ties and
    constant blocks."""
    torch = _torch()
    s = _synth()
    rng = np.random.default_rng(n_in + m)
    w = s.weight(rng, wtype, n_out, n_in)
    x = s.activations(rng, m, n_in)
    b = 256 if wtype == TYPE_Q4_K else 32     # quantization block
    x[0, :b] = 0.0                            # all-zero block
    x[0, b:2 * b] = 1.0                       # constant block
    x[0, 2 * b + 7] = 9.0
    x[0, 2 * b + b // 2] = -9.0               # equal |max|: the first one sets the sign
    x[m - 1, -b // 4:] = -1e-30               # tiny values in the last block
    h = gpu.upload_weight(w, wtype, n_out, n_in)
    try:
        xd = torch.from_numpy(x).cuda()
        xq = torch.from_numpy(port.quantize(x, wtype)).cuda()
        fused = torch.full((m, n_out), float("nan"), device="cuda")
        pre = torch.full((m, n_out), float("nan"), device="cuda")
        cuda = gpu.load_cuda()
        assert cuda.edgexpu_cuda_linear_quant_batch_dev(fused.data_ptr(), xd.data_ptr(), h, wtype, None, m, n_out,
                                                        n_in, _stream())
        assert cuda.edgexpu_cuda_dot_quant_q8_dev(pre.data_ptr(), xq.data_ptr(), h, wtype, None, m, n_out, n_in,
                                                  _stream())
        _sync(gpu)
        np.testing.assert_array_equal(fused.cpu().numpy(), pre.cpu().numpy())
    finally:
        gpu.free_weight(h)


def test_linear_row_subrange_and_dev_path(gpu, port):
    """A handle may point at any row of a registered tensor; the device-buffer entry point gives
    the same bits as the host-buffer one."""
    torch = _torch()
    s = _synth()
    rng = np.random.default_rng(77)
    n_out, n_in, m = 333, 576, 3
    w = s.q8_0_weight(rng, n_out, n_in)
    x = s.activations(rng, m, n_in)
    h = gpu.upload_weight(w, TYPE_Q8_0, n_out, n_in)
    try:
        r0, rows = 101, 150  # odd row offset: the bulk copy start is realigned on the device
        sub = h + r0 * gpu.row_bytes(TYPE_Q8_0, n_in)
        got = gpu.linear_quant_batch(x, sub, TYPE_Q8_0, rows)
        want = port.linear(x, w[r0:r0 + rows], TYPE_Q8_0, rows)
        assert_close(got, want, port.linear_bound(x, w[r0:r0 + rows], TYPE_Q8_0, rows))
        xd = torch.from_numpy(x).cuda()
        out = torch.empty((m, rows), dtype=torch.float32, device="cuda")
        assert gpu.load_cuda().edgexpu_cuda_linear_quant_batch_dev(out.data_ptr(), xd.data_ptr(), sub, TYPE_Q8_0,
                                                                   None, m, rows, n_in, _stream())
        _sync(gpu)
        np.testing.assert_array_equal(out.cpu().numpy(), got)
        with pytest.raises(gpu.EdgexpuError, match="exceed"):
            gpu.linear_quant_batch(x, sub, TYPE_Q8_0, n_out)
    finally:
        gpu.free_weight(h)


def test_linear_deterministic(gpu):
    s = _synth()
    rng = np.random.default_rng(5)
    w = s.q4_k_weight(rng, 4096, 4096)
    x = s.activations(rng, 2, 4096)
    h = gpu.upload_weight(w, TYPE_Q4_K, 4096, 4096)
    try:
        a = gpu.linear_quant_batch(x, h, TYPE_Q4_K, 4096)
        b = gpu.linear_quant_batch(x, h, TYPE_Q4_K, 4096)
    finally:
        gpu.free_weight(h)
    np.testing.assert_array_equal(a, b)


def test_error_paths(gpu):
    host = gpu.load_host()
    x = np.ones((1, 64), np.float32)
    out = np.zeros((1, 4), np.float32)
    junk = np.zeros(4 * 68, np.uint8)
    host.edgexpu_b200_clear_error()
    host.edgexpu_cpu_linear_quant_batch(out.ctypes.data, x.ctypes.data, junk.ctypes.data, TYPE_Q8_0, None, 1, 4, 64)
    assert np.all(np.isnan(out)) and b"not a registered" in host.edgexpu_b200_last_error()
    s = _synth()
    w = s.q8_0_weight(np.random.default_rng(1), 4, 64)
    h = gpu.upload_weight(w, TYPE_Q8_0, 4, 64)
    try:
        with pytest.raises(gpu.EdgexpuError, match="type"):
            gpu.linear_quant_batch(np.ones((1, 256), np.float32), h, TYPE_Q4_K, 4)
        with pytest.raises(gpu.EdgexpuError, match="unsupported"):
            gpu.linear_quant_batch(np.ones((1, 64), np.float32), h, 7, 4)  # GGUF type 7 (Q5_1): not on this path
    finally:
        gpu.free_weight(h)


# ---- known-answer tests of the reference (gguf_quant.c:943-958, :1016-1037) --------------------


def test_reference_kats_on_gpu(gpu):
    from test_oracle import q4_k_kat_inputs, q8_0_kat_inputs

    w, x = q8_0_kat_inputs()
    h = gpu.upload_weight(w, TYPE_Q8_0, 1, 32)
    try:
        assert abs(gpu.linear_quant_batch(x, h, TYPE_Q8_0, 1)[0, 0] - 32.0) <= 0.5
    finally:
        gpu.free_weight(h)
    blk, x = q4_k_kat_inputs()
    h = gpu.upload_weight(blk, TYPE_Q4_K, 1, 256)
    try:
        tok, score = gpu.logits_greedy(h, TYPE_Q4_K, x, 1)
        assert tok == 0 and abs(score - 6.0) <= 1e-3
    finally:
        gpu.free_weight(h)


# ---- greedy logits ----------------------------------------------------------------------------


@pytest.mark.parametrize("wtype,vocab,n_embd", [(TYPE_Q8_0, 49152, 576), (TYPE_Q4_K, 128256, 4096),
                                                (TYPE_Q8_0, 777, 64), (TYPE_Q4_K, 1000, 512)])
def test_logits_greedy_matches_oracle(gpu, port, wtype, vocab, n_embd):
    s = _synth()
    rng = np.random.default_rng(vocab)
    w = s.weight(rng, wtype, vocab, n_embd)
    hidden = s.activations(rng, 1, n_embd)[0]
    tok_o, score_o, scores = port.logits(w, wtype, hidden, vocab)
    h = gpu.upload_weight(w, wtype, vocab, n_embd)
    try:
        tok, score = gpu.logits_greedy(h, wtype, hidden, vocab)
        top2 = np.argsort(scores)[-2:]
        bound = port.logits_bound(w, wtype, hidden, [tok, tok_o, *top2])
        assert abs(score - score_o) <= TOL * bound.max()
        margin = scores[top2[1]] - scores[top2[0]]
        if margin > 2 * TOL * bound.max():
            assert tok == tok_o
        else:  # near-tie: the GPU's pick must still be within tolerance of the best score
            assert scores[tok] >= score_o - 2 * TOL * bound.max()
    finally:
        gpu.free_weight(h)


def test_logits_ties_bias_and_shards(gpu, port):
    torch = _torch()
    s = _synth()
    rng = np.random.default_rng(21)
    vocab, n = 4000, 576
    w = s.q8_0_weight(rng, vocab, n)
    hidden = s.activations(rng, 1, n)[0]
    best, _, _ = port.logits(w, TYPE_Q8_0, hidden, vocab)
    w[3999] = w[best]  # exact duplicate of the winner at a higher id
    w[best + 1 if best + 1 < 3999 else 0] = w[best]
    tok_o, _, _ = port.logits(w, TYPE_Q8_0, hidden, vocab)
    assert tok_o == min(best, best + 1 if best + 1 < 3999 else 0)
    h = gpu.upload_weight(w, TYPE_Q8_0, vocab, n)
    try:
        assert gpu.logits_greedy(h, TYPE_Q8_0, hidden, vocab)[0] == tok_o
        bias = np.zeros(vocab, np.float32)
        bias[tok_o] = -np.inf
        bias[5] = np.nan
        tok_b, _, _ = port.logits(w, TYPE_Q8_0, hidden, vocab, bias)
        assert gpu.logits_greedy(h, TYPE_Q8_0, hidden, vocab, bias)[0] == tok_b
        allneg = np.full(vocab, -np.inf, np.float32)
        assert gpu.logits_greedy(h, TYPE_Q8_0, hidden, vocab, allneg)[0] == 0
        # vocab shards: the max over per-shard keys is the global greedy choice (tensor parallel)
        hd = torch.from_numpy(hidden).cuda()
        keys = torch.zeros(4, dtype=torch.int64, device="cuda")
        rb = gpu.row_bytes(TYPE_Q8_0, n)
        for i in range(4):
            r0 = i * 1000
            assert gpu.load_cuda().edgexpu_cuda_logits_argmax_dev(h + r0 * rb, TYPE_Q8_0, hd.data_ptr(), n, 1000,
                                                                  None, r0, keys[i:].data_ptr(), _stream())
        _sync(gpu)
        k = int(keys.cpu().numpy().view(np.uint64).max())
        assert gpu.key_to_id(k) == tok_o
    finally:
        gpu.free_weight(h)


@pytest.mark.parametrize("wtype,m", [(TYPE_Q4_K, 1), (TYPE_Q4_K, 5), (TYPE_Q8_0, 2)])
def test_multi_tensor_launch_equals_separate_calls(gpu, port, wtype, m):
    """q/k/v-style grouped launch: one kernel over several weight tensors sharing x."""
    torch = _torch()
    s = _synth()
    rng = np.random.default_rng(40 + m)
    n_in = 1024 if wtype == TYPE_Q4_K else 576
    shapes = [512, 128, 128] if wtype == TYPE_Q4_K else [576, 192]
    ws = [s.weight(rng, wtype, n, n_in) for n in shapes]
    hs = [gpu.upload_weight(w, wtype, n, n_in) for w, n in zip(ws, shapes)]
    try:
        x_np = s.activations(rng, m, n_in)
        x = torch.from_numpy(x_np).cuda()
        bias = [torch.from_numpy(rng.standard_normal(n).astype(np.float32)).cuda() for n in shapes]
        outs = [torch.full((m, n), float("nan"), device="cuda") for n in shapes]
        refs = [torch.full((m, n), float("nan"), device="cuda") for n in shapes]
        cuda = gpu.load_cuda()
        k = len(shapes)
        P = ctypes.c_void_p * k
        ok = cuda.edgexpu_cuda_linear_quant_multi_dev(
            k, P(*[o.data_ptr() for o in outs]), P(*hs), (ctypes.c_int * k)(*shapes), P(*[b.data_ptr() for b in bias]),
            wtype, x.data_ptr(), m, n_in, _stream())
        assert ok, cuda.edgexpu_cuda_last_error()
        for r, h, n, b in zip(refs, hs, shapes, bias):
            assert cuda.edgexpu_cuda_linear_quant_batch_dev(r.data_ptr(), x.data_ptr(), h, wtype, b.data_ptr(), m, n,
                                                            n_in, _stream())
        _sync(gpu)
        for o, r, w, n, b in zip(outs, refs, ws, shapes, bias):
            np.testing.assert_array_equal(o.cpu().numpy(), r.cpu().numpy())
            want = port.linear(x_np, w, wtype, n, b.cpu().numpy())
            assert_close(o.cpu().numpy(), want, port.linear_bound(x_np, w, wtype, n), 1e-6)
    finally:
        for h in hs:
            gpu.free_weight(h)

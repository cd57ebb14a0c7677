"""GPU parity of the tensor-core prefill GEMM (Q4_K weights x Q8_K activations, m >= 64 rows).

The GEMM splits the folded weight sc*q4 into an int8 low part and a high part and sums
L = sum l*q8 and H = sum h*q8 on the tensor cores, and the mins term summ = sum_j m_j * S_j with
dp4a on the CUDA cores; (sumi, summ) = (L + 256 H, summ) must equal the reference's int32 values
bit for bit (dot_q4_k_q8_k, gguf_dot_q8.c:711-759), and the fp32 outputs must stay within
1e-5 * sum_k |w_k x_k| of the oracle.
"""

import ctypes

import numpy as np
import pytest

from _oracle import TYPE_Q4_K
from test_gpu_parity import _stream, _sync, _torch, assert_close
from test_oracle import _synth

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def relaxed_order(gpu):
    """The GEMM serves float outputs in the relaxed float order (include/edgexpu_cuda.h); the x86
    order routes those batches to the GEMV.  Integer partials use the GEMM in both."""
    cuda = gpu.load_cuda()
    assert cuda.edgexpu_cuda_set_float_order(gpu.ORDER_RELAXED) == 1
    yield
    cuda.edgexpu_cuda_set_float_order(gpu.ORDER_X86)


def pack_scales(sc, mn):
    """Inverse of get_scale_min_k4 (gguf_quant.c:212-220): eight 6-bit (scale, min) pairs -> 12 bytes."""
    s = np.zeros(12, np.uint8)
    for j in range(4):
        s[j] = (sc[j] & 63) | ((sc[j + 4] >> 4) << 6)
        s[j + 4] = (mn[j] & 63) | ((mn[j + 4] >> 4) << 6)
        s[j + 8] = (sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4)
    return s


def uniform_q4k(n_out, n_in, sc, mn, q, d=5e-4, dmin=3e-4):
    """Q4_K rows whose every super-block has the given scales/mins and all nibbles equal to q."""
    nb = n_in // 256
    blk = np.zeros((n_out, nb, 144), np.uint8)
    blk[..., 0:2] = np.array([d], np.float16).view(np.uint8)
    blk[..., 2:4] = np.array([dmin], np.float16).view(np.uint8)
    blk[..., 4:16] = pack_scales(sc, mn)
    blk[..., 16:] = (q & 15) | ((q & 15) << 4)
    return blk.reshape(n_out, nb * 144)


def _partials(gpu, h, xq, m, n_out, n_in):
    torch = _torch()
    xq_d = torch.from_numpy(np.ascontiguousarray(xq)).cuda()
    got = torch.empty(m * n_out * (n_in // 256) * 2, dtype=torch.int32, device="cuda")
    ok = gpu.load_cuda().edgexpu_cuda_block_partials_dev(got.data_ptr(), xq_d.data_ptr(), h, TYPE_Q4_K, m, n_out, n_in,
                                                         _stream())
    assert ok, gpu.load_cuda().edgexpu_cuda_last_error()
    _sync(gpu)
    return got.cpu().numpy().reshape(m, n_out, n_in // 256, 2)


@pytest.mark.parametrize("n_out,n_in,m", [
    (128, 256, 64),     # one tile, one super-block
    (300, 1024, 64),    # ragged row tile
    (200, 512, 100),    # ragged token tile
    (257, 4096, 130),   # both ragged, 16 super-blocks, 3 token tiles
    # 16-token tiles (batches of 9..63), K split over CTAs where the row tiles alone leave SMs idle
    (128, 256, 63),     # one super-block: no split, 4 token tiles
    (300, 1024, 9),     # ragged row tile, 4 super-blocks in 2 ranges
    (257, 4096, 16),    # 16 super-blocks in 8 ranges, one full token tile
    (1000, 14336, 33),  # down-projection width: 56 super-blocks, 3 token tiles
])
def test_gemm_partials_bit_exact(gpu, port, n_out, n_in, m):
    s = _synth()
    rng = np.random.default_rng(n_out * 7 + n_in + m)
    w = s.q4_k_weight(rng, n_out, n_in)
    x = s.activations(rng, m, n_in)
    x[3] = 0.0                                  # all-zero row: zeroed Q8_K blocks
    x[5, :256] = 7.0                            # constant block: every q8 = -127
    xq = port.quantize(x, TYPE_Q4_K)
    h = gpu.upload_weight(w, TYPE_Q4_K, n_out, n_in)
    try:
        np.testing.assert_array_equal(_partials(gpu, h, xq, m, n_out, n_in), port.partials(w, xq, TYPE_Q4_K, n_in))
    finally:
        gpu.free_weight(h)


@pytest.mark.parametrize("m", [64, 16])
@pytest.mark.parametrize("sc,mn,q,lead", [
    (32, 63, 4, False),   # sc*q4 = 128: every low part is -128, q8 = -127 -> L = +128*127*256, the largest L
    (32, 63, 4, True),    # first element negated: q8 = +127 elsewhere -> L near -128*127*256
    (63, 63, 15, False),  # sc*q4 = 945: largest |sumi| (945*127*256) and |H|
    (17, 0, 15, True),    # sc*q4 = 255: high part 1, low part -1
    (63, 63, 0, False),   # zero nibbles: only the mins term
])
def test_gemm_accumulator_extremes(gpu, port, sc, mn, q, lead, m):
    """Q8_K maps the first largest |x| of a block to -127 (gguf_dot_q8.c:377-392): constant rows
    give q8 = -127 everywhere, a negated first element gives q8 = +127 everywhere else.  At m = 16 the
    16-token tiles run with the K range split."""
    n_out, n_in = 128, 1024
    w = uniform_q4k(n_out, n_in, [sc] * 8, [mn] * 8, q)
    x = np.full((m, n_in), 3.0, np.float32)
    if lead:
        x[:, ::256] = -3.0
    xq = port.quantize(x, TYPE_Q4_K)
    h = gpu.upload_weight(w, TYPE_Q4_K, n_out, n_in)
    try:
        want = port.partials(w, xq, TYPE_Q4_K, n_in)
        np.testing.assert_array_equal(_partials(gpu, h, xq, m, n_out, n_in), want)
        got = gpu.linear_quant_batch(x, h, TYPE_Q4_K, n_out)
        assert_close(got, port.linear(x, w, TYPE_Q4_K, n_out), port.linear_bound(x, w, TYPE_Q4_K, n_out))
    finally:
        gpu.free_weight(h)


@pytest.mark.parametrize("n_out,n_in,m,with_bias", [
    (4096, 4096, 64, False),     # config 3 o-projection at M = 64
    (300, 1024, 100, True),
    (1000, 14336, 70, False),    # down-projection width
    (6144, 4096, 65, True),      # fused q|k|v width, one token past a tile
    (4096, 4096, 16, False),     # config 2/4 batch 16: 16-token tile, K split in 8
    (14336, 4096, 9, True),      # gate width at the smallest routed batch
    (4096, 14336, 16, False),    # down projection at batch 16
    (300, 1024, 40, True),       # 3 token tiles, ragged rows
])
def test_gemm_linear_matches_oracle(gpu, port, n_out, n_in, m, with_bias):
    s = _synth()
    rng = np.random.default_rng(n_out + 3 * n_in + m)
    w = s.q4_k_weight(rng, n_out, n_in)
    x = s.activations(rng, m, n_in)
    bias = rng.standard_normal(n_out).astype(np.float32) if with_bias else None
    h = gpu.upload_weight(w, TYPE_Q4_K, n_out, n_in)
    try:
        got = gpu.linear_quant_batch(x, h, TYPE_Q4_K, n_out, bias)
    finally:
        gpu.free_weight(h)
    want = port.linear(x, w, TYPE_Q4_K, n_out, bias)
    bound = port.linear_bound(x, w, TYPE_Q4_K, n_out)
    assert_close(got, want, bound, 0.0 if bias is None else 1e-7 * np.abs(bias)[None, :] + 1e-6)


def test_gemm_partials_equal_gemv_partials_at_prefill_size(gpu, port):
    """Size-independent check at a config-3 batch: the GEMM's int32 partials (m = 512) equal the
    row-stream GEMV's (chunks of 4 rows, what its shared-memory tile holds at this width) exactly,
    for the down-projection width K = 14336."""
    torch = _torch()
    s = _synth()
    rng = np.random.default_rng(512)
    n_out, n_in, m = 256, 14336, 512
    w = s.q4_k_weight(rng, n_out, n_in)
    xq = port.quantize(s.activations(rng, m, n_in), TYPE_Q4_K)
    h = gpu.upload_weight(w, TYPE_Q4_K, n_out, n_in)
    try:
        big = _partials(gpu, h, xq, m, n_out, n_in)
        chunks = [_partials(gpu, h, xq[t:t + 4], 4, n_out, n_in) for t in range(0, m, 4)]
        np.testing.assert_array_equal(big, np.concatenate(chunks))
        np.testing.assert_array_equal(big[:16], port.partials(w, xq[:16], TYPE_Q4_K, n_in))
        # and the float outputs of both kernels agree to rounding
        xq_d = torch.from_numpy(xq).cuda()
        cuda = gpu.load_cuda()
        o_big = torch.empty((m, n_out), dtype=torch.float32, device="cuda")
        o_chk = torch.empty((m, n_out), dtype=torch.float32, device="cuda")
        assert cuda.edgexpu_cuda_dot_quant_q8_dev(o_big.data_ptr(), xq_d.data_ptr(), h, TYPE_Q4_K, None, m, n_out, n_in,
                                                  _stream())
        rb = gpu.act_row_bytes(TYPE_Q4_K, n_in)
        for t in range(0, m, 32):
            assert cuda.edgexpu_cuda_dot_quant_q8_dev(o_chk.data_ptr() + t * n_out * 4, xq_d.data_ptr() + t * rb, h,
                                                      TYPE_Q4_K, None, 32, n_out, n_in, _stream())
        _sync(gpu)
        a, b = o_big.cpu().numpy(), o_chk.cpu().numpy()
        assert np.max(np.abs(a - b) / (np.abs(b) + 1.0)) < 1e-4
    finally:
        gpu.free_weight(h)


def test_gemm_grouped_launch_and_determinism(gpu, port):
    torch = _torch()
    s = _synth()
    rng = np.random.default_rng(64)
    n_in, m, shapes = 1024, 96, [512, 128, 128]
    ws = [s.q4_k_weight(rng, n, n_in) for n in shapes]
    hs = [gpu.upload_weight(w, TYPE_Q4_K, n, n_in) for w, n in zip(ws, shapes)]
    try:
        x = torch.from_numpy(s.activations(rng, m, n_in)).cuda()
        outs = [torch.full((m, n), float("nan"), device="cuda") for n in shapes]
        refs = [torch.full((m, n), float("nan"), device="cuda") for n in shapes]
        cuda = gpu.load_cuda()
        k = len(shapes)
        P = ctypes.c_void_p * k
        assert cuda.edgexpu_cuda_linear_quant_multi_dev(k, P(*[o.data_ptr() for o in outs]), P(*hs),
                                                        (ctypes.c_int * k)(*shapes), None, TYPE_Q4_K, x.data_ptr(), m,
                                                        n_in, _stream())
        for r, h, n in zip(refs, hs, shapes):
            assert cuda.edgexpu_cuda_linear_quant_batch_dev(r.data_ptr(), x.data_ptr(), h, TYPE_Q4_K, None, m, n, n_in,
                                                            _stream())
        _sync(gpu)
        for o, r, w, n in zip(outs, refs, ws, shapes):
            np.testing.assert_array_equal(o.cpu().numpy(), r.cpu().numpy())
            want = port.linear(x.cpu().numpy(), w, TYPE_Q4_K, n)
            assert_close(o.cpu().numpy(), want, port.linear_bound(x.cpu().numpy(), w, TYPE_Q4_K, n))
    finally:
        for h in hs:
            gpu.free_weight(h)


# ---- the Q8_0 GEMM (gemm_q8_tc.cu) ------------------------------------------------------------------


@pytest.mark.parametrize("n_out,n_in,m,with_bias", [
    (1536, 576, 128, False),     # config 1's gate/up at its 128-token prompt (K tail: 18 blocks)
    (576, 1536, 200, True),      # down, ragged token tile
    (192, 576, 64, False),       # k/v, one token tile
    (1001, 4096, 77, True),      # ragged rows and tokens
    (130, 32, 64, False),        # one block: a chunk of one valid block
])
def test_q8_gemm_linear_matches_oracle(gpu, port, n_out, n_in, m, with_bias):
    from _oracle import TYPE_Q8_0

    s = _synth()
    rng = np.random.default_rng(n_out + 7 * n_in + m)
    w = s.q8_0_weight(rng, n_out, n_in)
    x = s.activations(rng, m, n_in)
    bias = rng.standard_normal(n_out).astype(np.float32) if with_bias else None
    h = gpu.upload_weight(w, TYPE_Q8_0, n_out, n_in)
    try:
        got = gpu.linear_quant_batch(x, h, TYPE_Q8_0, n_out, bias)
        again = gpu.linear_quant_batch(x, h, TYPE_Q8_0, n_out, bias)  # the cached repack
    finally:
        gpu.free_weight(h)
    want = port.linear(x, w, TYPE_Q8_0, n_out, bias)
    bound = port.linear_bound(x, w, TYPE_Q8_0, n_out)
    assert_close(got, want, bound, 0.0 if bias is None else 1e-7 * np.abs(bias)[None, :] + 1e-6)
    np.testing.assert_array_equal(got, again)


def test_q8_gemm_prequantized_and_grouped(gpu, port):
    """Pre-quantized Q8_0 rows (edgexpu_cuda_dot_quant_q8_dev) and a grouped q|k|v launch give the
    fp32 GEMM the same bits as the separate fp32 calls."""
    from _oracle import TYPE_Q8_0

    torch = _torch()
    s = _synth()
    rng = np.random.default_rng(99)
    n_in, m = 576, 96
    shapes = [576, 192, 192]
    ws = [s.q8_0_weight(rng, n, n_in) for n in shapes]
    x = s.activations(rng, m, n_in)
    hs = [gpu.upload_weight(w, TYPE_Q8_0, n, n_in) for w, n in zip(ws, shapes)]
    cuda = gpu.load_cuda()
    try:
        sep = [gpu.linear_quant_batch(x, h, TYPE_Q8_0, n) for h, n in zip(hs, shapes)]
        xd = torch.from_numpy(x).cuda()
        outs = [torch.full((m, n), float("nan"), device="cuda") for n in shapes]
        arr_o = (ctypes.c_void_p * 3)(*[o.data_ptr() for o in outs])
        arr_w = (ctypes.c_void_p * 3)(*hs)
        arr_n = (ctypes.c_int * 3)(*shapes)
        assert cuda.edgexpu_cuda_linear_quant_multi_dev(3, arr_o, arr_w, arr_n, None, TYPE_Q8_0, xd.data_ptr(), m, n_in,
                                                        _stream())
        xq = torch.from_numpy(port.quantize(x, TYPE_Q8_0)).cuda()
        pre = torch.full((m, shapes[0]), float("nan"), device="cuda")
        assert cuda.edgexpu_cuda_dot_quant_q8_dev(pre.data_ptr(), xq.data_ptr(), hs[0], TYPE_Q8_0, None, m, shapes[0],
                                                  n_in, _stream())
        _sync(gpu)
        for o, r in zip(outs, sep):
            np.testing.assert_array_equal(o.cpu().numpy(), r)
        np.testing.assert_array_equal(pre.cpu().numpy(), sep[0])
    finally:
        for h in hs:
            gpu.free_weight(h)

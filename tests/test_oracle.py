"""CPU tests pinning the oracle restatement (oracle/edgexpu_oracle.c) to the reference itself.

The reference has no tests/ tree; its known-answer self-tests live in
src/gguf_quant.c:934-1061 and src/cpu_kernel.c:861-972.  Those KATs are replayed here against
both the reference library (compiled from its sources by oracle/Makefile) and our restatement,
and the restatement is then pinned bit-for-bit against the reference on seeded inputs:

* activation bytes (Q8_0 AVX2+F16C path, Q8_0 scalar path, Q8_K) -- exact;
* float dots -- exact against the reference's SCALAR build, whose accumulation order the
  restatement follows; within the tolerance bound against the AVX2 build;
* per-block int32 partials -- exact, read out of the reference's own dot functions on crafted
  single-block inputs whose scales are 1.0.
"""

import numpy as np
import pytest

from _oracle import BLOCK, TYPE_Q4_0, TYPE_Q4_K, TYPE_Q5_0, TYPE_Q5_K, TYPE_Q6_K, TYPE_Q8_0, load_pkg

synth = None


def _synth():
    global synth
    if synth is None:
        load_pkg()
        import edgexpu_llm_b200.synth as s

        synth = s
    return synth


def edge_vectors(n, rng):
    """Inputs that stress rounding, ties, signs and degenerate blocks."""
    vs = []
    vs.append(np.zeros(n, np.float32))
    v = rng.standard_normal(n).astype(np.float32)
    v[::7] = 0.0
    vs.append(v)
    v = np.full(n, 1.0, np.float32)
    vs.append(v)
    v = np.full(n, -2.5, np.float32)
    vs.append(v)
    v = (rng.integers(-127, 128, n) / 127.0).astype(np.float32)  # many exact .5 rounding ties
    vs.append(v)
    v = (rng.integers(-255, 256, n) * 0.5).astype(np.float32)
    vs.append(v)
    v = rng.standard_normal(n).astype(np.float32) * 1e-6  # fp16 subnormal scales
    vs.append(v)
    v = rng.standard_normal(n).astype(np.float32) * 1e-9  # scale rounds to fp16 zero
    vs.append(v)
    v = rng.standard_normal(n).astype(np.float32) * 3e4
    vs.append(v)
    v = rng.standard_normal(n).astype(np.float32)
    v[5] = 9.0
    v[200 % n] = -9.0  # equal |max| with opposite signs: the first one sets the sign (Q8_K)
    vs.append(v)
    v = rng.standard_normal(n).astype(np.float32)
    v[3] = -7.0
    vs.append(v)
    return vs


# ---- fp16 conversions -------------------------------------------------------------------------


def test_fp16_round_nearest_even_matches_numpy(port):
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * np.float32(10.0) ** rng.integers(-9, 6, 20000),
        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e9, -1e9, 2.0 ** -24, 2.0 ** -25, 3 * 2.0 ** -26,
                  2.0 ** -14, 2.0 ** -15 * 1.5, 6.1e-5, np.inf, -np.inf], np.float32),
    ]).astype(np.float32)
    got = np.array([port.lib.eo_fp32_to_fp16(float(v)) for v in vals], np.uint16)
    want = vals.astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(got, want)


def test_fp16_to_fp32_exact(port):
    bits = np.arange(0, 65536, dtype=np.uint32).astype(np.uint16)
    want = bits.view(np.float16).astype(np.float32)
    got = np.array([port.lib.eo_fp16_to_fp32(int(b)) for b in bits], np.float32)
    finite = np.isfinite(want)
    np.testing.assert_array_equal(got[finite].view(np.uint32), want[finite].view(np.uint32))
    assert np.all(np.isnan(got[np.isnan(want)]))


# ---- the reference's own known-answer self-tests -----------------------------------------------


def test_reference_selftest_passes(ref):
    import ctypes

    buf = ctypes.create_string_buffer(256)
    assert ref.lib.edgexpu_gguf_quant_selftest(buf, 256) == 1, buf.value
    assert ref.lib.edgexpu_cpu_simd_name() == b"avx2"


def q8_0_kat_inputs():
    """gguf_quant.c:1016-1037: weight block d = fp16 1.0, qs all 1; x = all ones."""
    w = np.zeros(34, np.uint8)
    w[0:2] = np.array([0x3C00], np.uint16).view(np.uint8)
    w[2:] = 1
    return w, np.ones(32, np.float32)


def q4_k_kat_inputs():
    """gguf_quant.c:943-958: d = 1.0, first sub-block scale 1, low nibble 2 at element 0; x[0] = 3."""
    blk = np.zeros(144, np.uint8)
    blk[0:2] = np.array([0x3C00], np.uint16).view(np.uint8)
    blk[4] = 1
    blk[16] = 0x02
    x = np.zeros(256, np.float32)
    x[0] = 3.0
    return blk, x


def test_kat_q8_0_integer_dot(port, ref):
    w, x = q8_0_kat_inputs()
    xq_port = port.quantize(x, TYPE_Q8_0)[0]
    xq_ref = ref.quantize(x, TYPE_Q8_0)[0]
    np.testing.assert_array_equal(xq_port, xq_ref)
    got = port.lib.eo_dot_q8_0_q8_0(w.ctypes.data, xq_port.ctypes.data, 32)
    assert abs(got - 32.0) <= 0.5
    assert abs(ref.dot_q8(TYPE_Q8_0, w, xq_ref, 32) - 32.0) <= 0.5


def test_kat_q4_k_f32_dot(port, ref):
    blk, x = q4_k_kat_inputs()
    got = port.lib.eo_dot_q4_k_f32(blk.ctypes.data, x.ctypes.data, 256)
    assert abs(got - 6.0) <= 1e-3
    assert abs(ref.dot_f32(TYPE_Q4_K, blk, x, 256) - 6.0) <= 1e-3
    y = np.empty(256, np.float32)
    assert port.lib.eo_dequantize_row(TYPE_Q4_K, blk.ctypes.data, 256, y.ctypes.data)
    assert abs(float(np.dot(y, x)) - 6.0) <= 1e-4


# ---- activation quantizers: bit-exact ----------------------------------------------------------


@pytest.mark.parametrize("n", [32, 64, 576, 1536, 4096])
def test_quantize_q8_0_bit_exact(port, ref, n):
    rng = np.random.default_rng(n)
    for v in edge_vectors(n, rng):
        np.testing.assert_array_equal(port.quantize(v, TYPE_Q8_0), ref.quantize(v, TYPE_Q8_0))


@pytest.mark.parametrize("n", [32, 576, 1536])
def test_quantize_q8_0_scalar_path_bit_exact(port, ref_scalar, n):
    rng = np.random.default_rng(100 + n)
    for v in edge_vectors(n, rng):
        np.testing.assert_array_equal(port.quantize(v, TYPE_Q8_0, scalar=True), ref_scalar.quantize(v, TYPE_Q8_0))


def test_quantize_q8_0_paths_differ(port):
    """The x86 Release path (id = 127/amax, RNE fp16) and the generic path (id = 1/d, truncating
    fp16) give different bytes: parity is pinned to the Release build."""
    rng = np.random.default_rng(7)
    v = rng.standard_normal(4096).astype(np.float32)
    assert not np.array_equal(port.quantize(v, TYPE_Q8_0), port.quantize(v, TYPE_Q8_0, scalar=True))


@pytest.mark.parametrize("n", [256, 512, 4096, 14336])
def test_quantize_q8_k_bit_exact(port, ref, n):
    rng = np.random.default_rng(n + 1)
    for v in edge_vectors(n, rng):
        np.testing.assert_array_equal(port.quantize(v, TYPE_Q4_K), ref.quantize(v, TYPE_Q4_K))


def test_quantize_q8_k_first_max_sets_sign(port, ref):
    v = np.zeros(256, np.float32)
    v[10] = -4.0
    v[20] = 4.0
    v[30] = 1.0
    q = port.quantize(v, TYPE_Q4_K)[0]
    np.testing.assert_array_equal(q, ref.quantize(v, TYPE_Q4_K)[0])
    d = q[0:4].view(np.float32)[0]
    assert d > 0 and q[4 + 10].view(np.int8) == -127 and q[4 + 20].view(np.int8) == 127


# ---- float dots: exact vs the reference's scalar build, bounded vs its AVX2 build ---------------


@pytest.mark.parametrize("wtype,n", [(TYPE_Q8_0, 576), (TYPE_Q8_0, 1536), (TYPE_Q4_K, 4096), (TYPE_Q4_K, 1024)])
def test_dot_matches_reference(port, ref, ref_scalar, wtype, n):
    s = _synth()
    rng = np.random.default_rng(wtype * 1000 + n)
    w = s.weight(rng, wtype, 24, n)
    x = s.activations(rng, 3, n)
    xq = port.quantize(x, wtype)
    np.testing.assert_array_equal(xq, ref.quantize(x, wtype))
    fn = port.lib.eo_dot_q8_0_q8_0 if wtype == TYPE_Q8_0 else port.lib.eo_dot_q4_k_q8_k
    for t in range(3):
        for o in range(24):
            got = np.float32(fn(w[o].ctypes.data, xq[t].ctypes.data, n))
            exact = np.float32(ref_scalar.dot_q8(wtype, w[o], xq[t], n))
            assert got.view(np.uint32) == exact.view(np.uint32)
            bound = port.lib.eo_abs_bound_q8(wtype, w[o].ctypes.data, xq[t].ctypes.data, n)
            assert abs(float(got) - ref.dot_q8(wtype, w[o], xq[t], n)) <= 1e-5 * bound + 1e-30


@pytest.mark.parametrize("n", [256, 4096])
def test_dot_q4_k_f32_matches_reference(port, ref, ref_scalar, n):
    s = _synth()
    rng = np.random.default_rng(n + 5)
    w = s.q4_k_weight(rng, 16, n)
    x = s.activations(rng, 1, n)[0]
    for o in range(16):
        got = np.float32(port.lib.eo_dot_q4_k_f32(w[o].ctypes.data, x.ctypes.data, n))
        exact = np.float32(ref_scalar.dot_f32(TYPE_Q4_K, w[o], x, n))
        assert got.view(np.uint32) == exact.view(np.uint32)
        bound = port.lib.eo_abs_bound_f32(TYPE_Q4_K, w[o].ctypes.data, x.ctypes.data, n)
        assert abs(float(got) - ref.dot_f32(TYPE_Q4_K, w[o], x, n)) <= 1e-5 * bound


# ---- per-block int32 partials pinned through the reference's own dot ----------------------------


def test_partials_q8_0_pinned_by_reference(port, ref):
    """With d_w = d_x = 1.0 the reference's one-block dot returns exactly (float)ip."""
    s = _synth()
    rng = np.random.default_rng(11)
    w = s.q8_0_weight(rng, 8, 576)
    xq = port.quantize(s.activations(rng, 2, 576), TYPE_Q8_0)
    parts = port.partials(w, xq, TYPE_Q8_0, 576)
    one = np.array([0x3C00], np.uint16).view(np.uint8)
    for t in range(2):
        for o in range(8):
            for b in range(18):
                wb = w[o, 34 * b:34 * b + 34].copy()
                xb = xq[t, 34 * b:34 * b + 34].copy()
                wb[0:2] = one
                xb[0:2] = one
                assert ref.dot_q8(TYPE_Q8_0, wb, xb, 32) == float(parts[t, o, b])


def test_partials_q4_k_pinned_by_reference(port, ref_scalar):
    """d = 1, dmin = 0, Q8_K d = 1 -> the scalar reference dot is sumi; d = 0, dmin = 1 -> -summ."""
    s = _synth()
    rng = np.random.default_rng(12)
    w = s.q4_k_weight(rng, 6, 1024)
    xq = port.quantize(s.activations(rng, 2, 1024), TYPE_Q4_K)
    parts = port.partials(w, xq, TYPE_Q4_K, 1024)
    one16 = np.array([0x3C00], np.uint16).view(np.uint8)
    zero16 = np.zeros(2, np.uint8)
    one32 = np.array([1.0], np.float32).view(np.uint8)
    for t in range(2):
        for o in range(6):
            for b in range(4):
                wb = w[o, 144 * b:144 * b + 144].copy()
                xb = xq[t, 292 * b:292 * b + 292].copy()
                xb[0:4] = one32
                wb[0:2], wb[2:4] = one16, zero16
                assert ref_scalar.dot_q8(TYPE_Q4_K, wb, xb, 256) == float(parts[t, o, b, 0])
                wb[0:2], wb[2:4] = zero16, one16
                assert ref_scalar.dot_q8(TYPE_Q4_K, wb, xb, 256) == -float(parts[t, o, b, 1])


# ---- linear and logits against the reference ---------------------------------------------------


@pytest.mark.parametrize("wtype,n_out,n_in,m", [(TYPE_Q8_0, 96, 576, 4), (TYPE_Q4_K, 40, 1024, 3)])
def test_linear_quant_batch_matches_reference(port, ref, wtype, n_out, n_in, m):
    s = _synth()
    rng = np.random.default_rng(n_out + m)
    w = s.weight(rng, wtype, n_out, n_in)
    x = s.activations(rng, m, n_in)
    bias = rng.standard_normal(n_out).astype(np.float32)
    got = port.linear(x, w, wtype, n_out, bias)
    want = ref.linear(x, w, wtype, n_out, bias)
    bound = port.linear_bound(x, w, wtype, n_out)
    assert np.all(np.abs(got.astype(np.float64) - want) <= 1e-5 * bound + 1e-6 * np.abs(bias))


@pytest.mark.parametrize("wtype,n_in", [(TYPE_Q8_0, 576), (TYPE_Q4_K, 512)])
def test_logits_argmax_matches_reference(port, ref, wtype, n_in):
    s = _synth()
    rng = np.random.default_rng(n_in)
    vocab = 300
    w = s.weight(rng, wtype, vocab, n_in)
    w[200] = w[17]  # an exact tie: the lower id must win
    h = s.activations(rng, 1, n_in)[0]
    tok, score, scores = port.logits(w, wtype, h, vocab)
    rtok, rscore, rscores = ref.logits(w, wtype, h, vocab)
    assert scores[200] == scores[17]
    bound = port.logits_bound(w, wtype, h, range(vocab))
    assert np.all(np.abs(scores.astype(np.float64) - rscores) <= 1e-5 * bound)
    srt = np.sort(rscores)
    if srt[-1] - srt[-2] > 2e-5 * bound.max():
        assert tok == rtok


def test_logits_tie_prefers_lowest_id(port):
    s = _synth()
    rng = np.random.default_rng(3)
    w = s.q8_0_weight(rng, 50, 64)
    h = s.activations(rng, 1, 64)[0]
    _, _, scores = port.logits(w, TYPE_Q8_0, h, 50)
    best = int(np.argmax(scores))
    w2 = np.concatenate([w, w[best:best + 1]], axis=0)  # duplicate of the best row at id 50
    tok, _, _ = port.logits(w2, TYPE_Q8_0, h, 51)
    assert tok == best
    bias = np.zeros(51, np.float32)
    bias[:] = -np.inf
    bias[7] = np.nan
    tok, sc, _ = port.logits(w2, TYPE_Q8_0, h, 51, bias)
    assert tok == 0 and sc == -np.inf  # nothing beats -inf: the reference keeps id 0


# ---- the other GGUF weight types behind the same dispatch (Q4_0, Q5_0, Q5_K, Q6_K) --------------

OTHER_TYPES = (TYPE_Q4_0, TYPE_Q5_0, TYPE_Q5_K, TYPE_Q6_K)


@pytest.mark.parametrize("wtype", OTHER_TYPES)
@pytest.mark.parametrize("n", [256, 1536])
def test_other_types_dot_q8_matches_reference(port, ref, ref_scalar, wtype, n):
    """edgexpu_gguf_dot_quant_q8 / _q8k: bit-exact against the scalar build, bounded against AVX2."""
    s = _synth()
    rng = np.random.default_rng(wtype * 100 + n)
    w = s.weight(rng, wtype, 12, n)
    x = s.activations(rng, 2, n)
    xq = port.quantize(x, wtype)
    for t in range(2):
        for o in range(12):
            got = np.float32(port.lib.eo_dot_q8(wtype, w[o].ctypes.data, xq[t].ctypes.data, n))
            exact = np.float32(ref_scalar.dot_q8(wtype, w[o], xq[t], n))
            assert got.view(np.uint32) == exact.view(np.uint32), (t, o)
            bound = port.lib.eo_abs_bound_q8(wtype, w[o].ctypes.data, xq[t].ctypes.data, n)
            assert abs(float(got) - ref.dot_q8(wtype, w[o], xq[t], n)) <= 1e-5 * bound


@pytest.mark.parametrize("wtype", OTHER_TYPES + (TYPE_Q8_0,))
@pytest.mark.parametrize("n", [256, 1024])
def test_other_types_dot_f32_matches_reference(port, ref, ref_scalar, wtype, n):
    """edgexpu_gguf_dot_quant (fp32 activations, the logits path of the K-quants)."""
    s = _synth()
    rng = np.random.default_rng(wtype * 10 + n)
    w = s.weight(rng, wtype, 10, n)
    x = s.activations(rng, 1, n)[0]
    for o in range(10):
        got = np.float32(port.lib.eo_dot_f32(wtype, w[o].ctypes.data, x.ctypes.data, n))
        exact = np.float32(ref_scalar.dot_f32(wtype, w[o], x, n))
        assert got.view(np.uint32) == exact.view(np.uint32), o
        bound = port.lib.eo_abs_bound_f32(wtype, w[o].ctypes.data, x.ctypes.data, n)
        assert abs(float(got) - ref.dot_f32(wtype, w[o], x, n)) <= 1e-5 * bound


@pytest.mark.parametrize("wtype", OTHER_TYPES + (TYPE_Q8_0, TYPE_Q4_K))
def test_dequantize_row_matches_reference(port, ref, wtype):
    """edgexpu_gguf_dequantize (gguf_quant.c:355-411) row by row: bit-exact floats."""
    import ctypes

    s = _synth()
    rng = np.random.default_rng(wtype)
    n = 512
    w = s.weight(rng, wtype, 4, n)
    fn = ref.lib.edgexpu_gguf_dequantize
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
    for o in range(4):
        got = np.empty(n, np.float32)
        want = np.empty(n, np.float32)
        assert port.lib.eo_dequantize_row(wtype, w[o].ctypes.data, n, got.ctypes.data)
        assert fn(w[o].ctypes.data, wtype, n, want.ctypes.data, None, 0) == 1
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("wtype", (TYPE_Q4_0, TYPE_Q5_0))
def test_partials_b32_pinned_by_reference(port, ref, wtype):
    """With d_w = d_x = 1.0 the reference's one-block dot returns exactly (float)ip."""
    s = _synth()
    rng = np.random.default_rng(wtype + 40)
    bb = BLOCK[wtype][1]
    w = s.weight(rng, wtype, 6, 256)
    xq = port.quantize(s.activations(rng, 2, 256), wtype)
    parts = port.partials(w, xq, wtype, 256)
    one = np.array([0x3C00], np.uint16).view(np.uint8)
    for t in range(2):
        for o in range(6):
            for b in range(8):
                wb = w[o, bb * b:bb * b + bb].copy()
                xb = xq[t, 34 * b:34 * b + 34].copy()
                wb[0:2] = one
                xb[0:2] = one
                assert ref.dot_q8(wtype, wb, xb, 32) == float(parts[t, o, b])


def test_partials_q5_k_pinned_by_reference(port, ref_scalar):
    """As for Q4_K: d = 1, dmin = 0 gives sumi; d = 0, dmin = 1 gives -summ."""
    s = _synth()
    rng = np.random.default_rng(51)
    w = s.weight(rng, TYPE_Q5_K, 5, 512)
    xq = port.quantize(s.activations(rng, 2, 512), TYPE_Q5_K)
    parts = port.partials(w, xq, TYPE_Q5_K, 512)
    one16 = np.array([0x3C00], np.uint16).view(np.uint8)
    zero16 = np.zeros(2, np.uint8)
    one32 = np.array([1.0], np.float32).view(np.uint8)
    for t in range(2):
        for o in range(5):
            for b in range(2):
                wb = w[o, 176 * b:176 * b + 176].copy()
                xb = xq[t, 292 * b:292 * b + 292].copy()
                xb[0:4] = one32
                wb[0:2], wb[2:4] = one16, zero16
                assert ref_scalar.dot_q8(TYPE_Q5_K, wb, xb, 256) == float(parts[t, o, b, 0])
                wb[0:2], wb[2:4] = zero16, one16
                assert ref_scalar.dot_q8(TYPE_Q5_K, wb, xb, 256) == -float(parts[t, o, b, 1])


def test_partials_q6_k_pinned_by_reference(port, ref):
    """d = 1 and Q8_K d = 1 with small scales (|sumi| < 2^24, every float step exact): the AVX2
    reference dot, which forms sumi in int32 (gguf_dot_q8.c:908-963), returns exactly (float)sumi."""
    s = _synth()
    rng = np.random.default_rng(61)
    w = s.weight(rng, TYPE_Q6_K, 5, 512).reshape(5, 2, 210)
    w[:, :, 192:208] = rng.integers(-4, 5, (5, 2, 16), dtype=np.int8).view(np.uint8)
    w = w.reshape(5, 420)
    xq = port.quantize(s.activations(rng, 2, 512), TYPE_Q6_K)
    parts = port.partials(w, xq, TYPE_Q6_K, 512)
    one16 = np.array([0x3C00], np.uint16).view(np.uint8)
    one32 = np.array([1.0], np.float32).view(np.uint8)
    assert np.all(parts[..., 1] == 0)
    for t in range(2):
        for o in range(5):
            for b in range(2):
                wb = w[o, 210 * b:210 * b + 210].copy()
                xb = xq[t, 292 * b:292 * b + 292].copy()
                xb[0:4] = one32
                wb[208:210] = one16
                assert abs(int(parts[t, o, b, 0])) < (1 << 24)
                assert ref.dot_q8(TYPE_Q6_K, wb, xb, 256) == float(parts[t, o, b, 0])


@pytest.mark.parametrize("wtype", OTHER_TYPES)
def test_other_types_linear_and_logits_match_reference(port, ref, wtype):
    s = _synth()
    rng = np.random.default_rng(wtype + 7)
    n_out, n_in, m = 40, 512, 3
    w = s.weight(rng, wtype, n_out, n_in)
    x = s.activations(rng, m, n_in)
    bias = rng.standard_normal(n_out).astype(np.float32)
    got = port.linear(x, w, wtype, n_out, bias)
    want = ref.linear(x, w, wtype, n_out, bias)
    bound = port.linear_bound(x, w, wtype, n_out)
    assert np.all(np.abs(got.astype(np.float64) - want) <= 1e-5 * bound + 1e-6 * np.abs(bias))
    tok, _, scores = port.logits(w, wtype, x[0], n_out)
    rtok, _, rscores = ref.logits(w, wtype, x[0], n_out)
    lb = port.logits_bound(w, wtype, x[0], range(n_out))
    assert np.all(np.abs(scores.astype(np.float64) - rscores) <= 1e-5 * lb)
    srt = np.sort(rscores)
    if srt[-1] - srt[-2] > 2e-5 * lb.max():
        assert tok == rtok


# ---- the x86 Release build's float order: bit-identical ---------------------------------------

ALL = (TYPE_Q4_0, TYPE_Q5_0, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K)


@pytest.mark.parametrize("wtype", ALL)
@pytest.mark.parametrize("n", [256, 1536, 4096])
def test_x86_order_dots_bit_exact(port, ref, wtype, n):
    """eo_dot_q8_x86 / eo_dot_f32_x86 restate the SIMD branches' float steps: every result equals
    the reference AVX2 build's bit for bit."""
    s = _synth()
    rng = np.random.default_rng(wtype * 7 + n)
    w = s.weight(rng, wtype, 16, n)
    x = s.activations(rng, 2, n)
    x[1, ::5] = 0.0
    xq = port.quantize(x, wtype)
    for t in range(2):
        for o in range(16):
            got = np.float32(port.lib.eo_dot_q8_x86(wtype, w[o].ctypes.data, xq[t].ctypes.data, n))
            want = np.float32(ref.dot_q8(wtype, w[o], xq[t], n))
            assert got.view(np.uint32) == want.view(np.uint32), ("q8", t, o)
            got = np.float32(port.lib.eo_dot_f32_x86(wtype, w[o].ctypes.data, x[t].ctypes.data, n))
            want = np.float32(ref.dot_f32(wtype, w[o], x[t], n))
            assert got.view(np.uint32) == want.view(np.uint32), ("f32", t, o)


@pytest.mark.parametrize("wtype", ALL)
def test_x86_order_linear_bit_exact(port, ref, wtype):
    s = _synth()
    rng = np.random.default_rng(wtype + 31)
    n_out, n_in, m = 70, 1024, 5
    w = s.weight(rng, wtype, n_out, n_in)
    x = s.activations(rng, m, n_in)
    bias = rng.standard_normal(n_out).astype(np.float32)
    for b in (None, bias):
        got = port.linear(x, w, wtype, n_out, b, x86=True)
        want = ref.linear(x, w, wtype, n_out, b)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("wtype", ALL)
def test_device_recipe_matches_numpy_recipe(wtype):
    """The benchmarks' weights (synth.torch_weight, generated where they are used) follow the
    parity tests' numpy recipe: same block size, and fp16 scale fields finite and inside the
    recipe's range, so a benchmark never streams NaN or infinite block scales."""
    import torch

    s = _synth()
    n_out, n_in = 8, 1024
    g = torch.Generator()
    g.manual_seed(wtype)
    flat = s.torch_weight(wtype, n_out, n_in, g, "cpu", pad=64).numpy()
    qk, bb = BLOCK[wtype]
    nblk = n_out * n_in // qk
    assert flat.size == nblk * bb + 64 and not flat[nblk * bb:].any()
    blk = flat[: nblk * bb].reshape(nblk, bb)
    ref = s.weight(np.random.default_rng(wtype), wtype, n_out, n_in).reshape(nblk, bb)
    off, count = {TYPE_Q6_K: (208, 1), TYPE_Q4_K: (0, 2), TYPE_Q5_K: (0, 2)}.get(wtype, (0, 1))
    got = blk[:, off:off + 2 * count].copy().view(np.float16).astype(np.float32)
    want = ref[:, off:off + 2 * count].copy().view(np.float16).astype(np.float32)
    assert np.isfinite(got).all()
    lo, hi = float(want.min()), float(want.max())
    span = hi - lo
    assert got.min() >= lo - 0.1 * span and got.max() <= hi + 0.1 * span

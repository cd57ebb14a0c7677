"""The allocation-free linear entry point (edgexpu_cuda_linear_quant_batch_noalloc).

Some callers cannot allocate device memory once they are running: runtimes whose HBM budget is fixed
when the model is loaded, and decode loops that must not risk the device-wide synchronisation of
cudaMalloc/cudaFree.  This entry point needs no scratch for one or two rows and keeps the quantized
activations of larger batches in a fixed 1 MiB array compiled into the library.  The test calls it
twice in a row, with different inputs, through the C ABI and checks each result against the regular
device entry point's: bit for bit in the library's default (x86) float order, where both run the same
GEMV, and within the tolerance the other parity tests use in the relaxed order, where the regular
entry point runs Q4_K prefill batches on the tensor-core GEMM.  Cases cover the fused-quantization
batches (1, 2 rows), several GEMV passes, a prefill-sized batch and the 1 MiB limit itself; the
device's free memory must not change across the calls.  The file name sorts last so that a run
stopping at the first failure has run every other test first.
"""

import ctypes

import numpy as np
import pytest

from _oracle import TYPE_Q4_K, TYPE_Q8_0

pytestmark = pytest.mark.gpu

LIMIT = 1 << 20


def _linear(cuda, fn, torch, out_shape, x, h, wtype, m, n_out, n_in, stream):
    out = torch.full(out_shape, float("nan"), dtype=torch.float32, device="cuda")
    assert fn(out.data_ptr(), x.data_ptr(), h, wtype, None, m, n_out, n_in, stream), \
        cuda.edgexpu_cuda_last_error().decode()
    return out


CASES = [(TYPE_Q4_K, 1000, 4096, 5), (TYPE_Q8_0, 777, 1536, 3), (TYPE_Q4_K, 512, 4096, 1), (TYPE_Q8_0, 300, 576, 2),
         (TYPE_Q4_K, 256, 4096, 64), (TYPE_Q4_K, 64, 4096, LIMIT // (4096 // 256 * 292))]


@pytest.mark.parametrize("order", ["x86", "relaxed"])
@pytest.mark.parametrize("wtype,n_out,n_in,m", CASES)
def test_noalloc_matches_regular_entry_point_twice(gpu, port, wtype, n_out, n_in, m, order):
    import torch

    from test_oracle import _synth

    s = _synth()
    cuda = gpu.load_cuda()
    assert cuda.edgexpu_cuda_set_float_order(gpu.ORDER_X86 if order == "x86" else gpu.ORDER_RELAXED) == 1
    rng = np.random.default_rng(n_out + m)
    w = s.weight(rng, wtype, n_out, n_in)
    h = gpu.upload_weight(w, wtype, n_out, n_in)
    stream = torch.cuda.current_stream().cuda_stream
    buf = ctypes.create_string_buffer(512)
    try:
        xs = [torch.from_numpy(s.activations(rng, m, n_in)).cuda() for _ in range(2)]
        outs = [torch.empty((m, n_out), dtype=torch.float32, device="cuda") for _ in range(2)]
        # one call first: it looks up the array's address (and the regular path sizes its scratch)
        _linear(cuda, cuda.edgexpu_cuda_linear_quant_batch_noalloc, torch, (m, n_out), xs[0], h, wtype, m, n_out, n_in,
                stream)
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        for call in range(2):  # two calls in a row: the shared array keeps the previous contents
            o = outs[call]
            o.fill_(float("nan"))
            assert cuda.edgexpu_cuda_linear_quant_batch_noalloc(o.data_ptr(), xs[call].data_ptr(), h, wtype, None, m,
                                                                n_out, n_in, stream), cuda.edgexpu_cuda_last_error()
        assert cuda.edgexpu_cuda_stream_sync(stream, buf, 512), buf.value
        assert torch.cuda.mem_get_info()[0] == free0, "the no-alloc calls changed the device's free memory"
        for call in range(2):
            want = _linear(cuda, cuda.edgexpu_cuda_linear_quant_batch_dev, torch, (m, n_out), xs[call], h, wtype, m,
                           n_out, n_in, stream)
            assert cuda.edgexpu_cuda_stream_sync(stream, buf, 512), buf.value
            g, r = outs[call].cpu().numpy(), want.cpu().numpy()
            assert np.all(np.isfinite(g)), f"call {call}: unwritten outputs"
            if order == "x86":
                np.testing.assert_array_equal(g.view(np.uint32), r.view(np.uint32), err_msg=f"call {call}")
            else:
                bound = port.linear_bound(xs[call].cpu().numpy(), w, wtype, n_out)
                assert np.all(np.abs(g.astype(np.float64) - r) <= 1e-5 * bound), f"call {call}: out of tolerance"
    finally:
        gpu.free_weight(h)
        cuda.edgexpu_cuda_set_float_order(gpu.ORDER_X86)


def test_noalloc_rejects_batches_beyond_the_fixed_scratch(gpu):
    import torch

    from test_oracle import _synth

    cuda = gpu.load_cuda()
    n_in = 4096
    rows_fit = LIMIT // (n_in // 256 * 292)  # 224 rows of Q8_K activations
    w = _synth().q4_k_weight(np.random.default_rng(3), 8, n_in)
    h = gpu.upload_weight(w, TYPE_Q4_K, 8, n_in)
    try:
        m = rows_fit + 1
        x = torch.zeros((m, n_in), dtype=torch.float32, device="cuda")
        out = torch.zeros((m, 8), dtype=torch.float32, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        assert cuda.edgexpu_cuda_linear_quant_batch_noalloc(out.data_ptr(), x.data_ptr(), h, TYPE_Q4_K, None, m, 8, n_in,
                                                            stream) == 0
        assert b"scratch" in cuda.edgexpu_cuda_last_error()
        assert cuda.edgexpu_cuda_linear_quant_batch_noalloc(out.data_ptr(), x.data_ptr(), h, TYPE_Q4_K, None, rows_fit, 8,
                                                            n_in, stream) == 1
        buf = ctypes.create_string_buffer(512)
        assert cuda.edgexpu_cuda_stream_sync(stream, buf, 512), buf.value
    finally:
        gpu.free_weight(h)

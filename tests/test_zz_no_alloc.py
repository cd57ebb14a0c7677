"""The allocation-free linear entry point (edgexpu_cuda_linear_quant_batch_noalloc).

Some callers cannot allocate device memory once they are running: code recorded into a CUDA
graph, runtimes whose HBM budget is fixed when the model is loaded, and decode loops that must not
risk the device-wide synchronisation of cudaMalloc/cudaFree.  This entry point keeps its scratch
in a fixed 1 MiB array compiled into the library.  The test calls it twice in a row, with
different inputs, through the C ABI and checks each result against the regular device entry
point's within the tolerance the other parity tests use; it also checks the size limit.  The file
name sorts last so that a run stopping at the first failure has run every other test first.
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


@pytest.mark.parametrize("wtype,n_out,n_in,m", [(TYPE_Q4_K, 1000, 4096, 5), (TYPE_Q8_0, 777, 1536, 3)])
def test_noalloc_matches_regular_entry_point_twice(gpu, port, wtype, n_out, n_in, m):
    import torch

    from test_oracle import _synth

    s = _synth()
    cuda = gpu.load_cuda()
    rng = np.random.default_rng(n_out)
    w = s.weight(rng, wtype, n_out, n_in)
    h = gpu.upload_weight(w, wtype, n_out, n_in)
    stream = torch.cuda.current_stream().cuda_stream
    buf = ctypes.create_string_buffer(512)
    try:
        bound_tol = 1e-5
        for call in range(2):  # two calls in a row: the shared array keeps the previous contents
            x_np = s.activations(rng, m, n_in)
            x = torch.from_numpy(x_np).cuda()
            want = _linear(cuda, cuda.edgexpu_cuda_linear_quant_batch_dev, torch, (m, n_out), x, h, wtype, m, n_out,
                           n_in, stream)
            got = _linear(cuda, cuda.edgexpu_cuda_linear_quant_batch_noalloc, torch, (m, n_out), x, h, wtype, m, n_out,
                          n_in, stream)
            assert cuda.edgexpu_cuda_stream_sync(stream, buf, 512), buf.value
            bound = port.linear_bound(x_np, w, wtype, n_out)
            g, r = got.cpu().numpy().astype(np.float64), want.cpu().numpy().astype(np.float64)
            assert np.all(np.isfinite(g)), f"call {call}: unwritten outputs"
            assert np.all(np.abs(g - r) <= bound_tol * bound), f"call {call}: out of tolerance"
    finally:
        gpu.free_weight(h)


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

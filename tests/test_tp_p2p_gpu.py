"""Tensor-parallel linear with the all-reduce inside the GEMV (edgexpu_cuda_linear_quant_batch_tp_dev),
on 2, 4 and 8 GPUs: one process per GPU, CUDA IPC exchange regions, partials written over NVLink.

Checks: the summed output matches the oracle's unsharded linear within the usual bound; both ranks
hold the same bits; repeated calls (both parities of the exchange slots) give the same bits.
Each world size is skipped on boxes with fewer GPUs."""

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CASES = [(12, 4096, 4096, 1), (12, 4096, 14336, 2), (12, 1024, 2048, 5), (8, 576, 1536, 3),
         (12, 14336, 4096, 6)]  # the last: 4 rows per exchange slot, two launches


def _rank_main(rank, world, port, result_dir):
    import sys

    import torch
    import torch.distributed as dist

    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    from _oracle import load_pkg

    pkg = load_pkg()
    from edgexpu_llm_b200 import synth, tp

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.cuda.set_device(rank)
    pkg.init(rank)
    cuda = pkg.load_cuda()
    tp.connect_p2p(cuda, world, rank)
    out = {}
    for wtype, n_out, n_in, m in CASES:
        rng = np.random.default_rng(n_out + n_in + m)
        w = synth.weight(rng, wtype, n_out, n_in)
        x = synth.activations(rng, m, n_in)
        bias = rng.standard_normal(n_out).astype(np.float32)
        c0, per = tp.col_range(n_in, wtype, world, rank)
        ws = tp.shard_cols(w, n_in, wtype, world, rank)
        h = pkg.upload_weight(ws, wtype, n_out, per)
        xd = torch.from_numpy(np.ascontiguousarray(x[:, c0:c0 + per])).cuda()
        bd = torch.from_numpy(bias).cuda()
        st = torch.cuda.current_stream().cuda_stream
        runs = []
        for _ in range(3):
            o = torch.full((m, n_out), float("nan"), device="cuda")
            ok = cuda.edgexpu_cuda_linear_quant_batch_tp_dev(o.data_ptr(), xd.data_ptr(), h, wtype, bd.data_ptr(), m,
                                                             n_out, per, st)
            assert ok, cuda.edgexpu_cuda_last_error()
            runs.append(o)
        buf = __import__("ctypes").create_string_buffer(512)
        assert cuda.edgexpu_cuda_stream_sync(st, buf, 512), buf.value
        res = [r.cpu().numpy() for r in runs]
        out[(wtype, n_out, n_in, m)] = res
        pkg.free_weight(h)
    dist.barrier()
    cuda.edgexpu_cuda_tp_shutdown()
    pkg.shutdown()
    np.savez(os.path.join(result_dir, f"rank{rank}.npz"),
             **{f"{k[0]}_{k[1]}_{k[2]}_{k[3]}_{i}": v for k, vs in out.items() for i, v in enumerate(vs)})
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_linear_allreduce_in_gemv(tmp_path, port, world):
    import torch

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import random

    import torch.multiprocessing as mp

    mp.spawn(_rank_main, args=(world, random.randint(20000, 40000), str(tmp_path)), nprocs=world, join=True)
    from test_oracle import _synth
    from test_gpu_parity import assert_close

    s = _synth()
    ranks = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    for wtype, n_out, n_in, m in CASES:
        rng = np.random.default_rng(n_out + n_in + m)
        w = s.weight(rng, wtype, n_out, n_in)
        x = s.activations(rng, m, n_in)
        bias = rng.standard_normal(n_out).astype(np.float32)
        key = f"{wtype}_{n_out}_{n_in}_{m}"
        got = ranks[0][key + "_0"]
        for r in ranks:  # every call, every rank: the same bits
            for i in range(3):
                np.testing.assert_array_equal(r[key + f"_{i}"], got)
        assert_close(got, port.linear(x, w, wtype, n_out, bias), port.linear_bound(x, w, wtype, n_out),
                     1e-7 * np.abs(bias)[None, :] + 1e-6)


def _timeout_rank_main(rank, world, port, result_dir):
    """Rank 1 leaves the group between steps (it skips one tensor-parallel call, with nothing of its
    own in flight); rank 0's launch must give up waiting for rank 1's partials after its bounded wait
    (2 s), report the peer through the status word, and leave the GPU usable."""
    import ctypes
    import sys
    import time

    import torch
    import torch.distributed as dist

    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    from _oracle import load_pkg

    pkg = load_pkg()
    from edgexpu_llm_b200 import synth, tp

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.cuda.set_device(rank)
    pkg.init(rank)
    cuda = pkg.load_cuda()
    tp.connect_p2p(cuda, world, rank)
    wtype, n_out, n_in, m = 12, 1024, 4096, 1
    rng = np.random.default_rng(5)
    w = synth.weight(rng, wtype, n_out, n_in)
    x = synth.activations(rng, m, n_in)
    c0, per = tp.col_range(n_in, wtype, world, rank)
    h = pkg.upload_weight(tp.shard_cols(w, n_in, wtype, world, rank), wtype, n_out, per)
    xd = torch.from_numpy(np.ascontiguousarray(x[:, c0:c0 + per])).cuda()
    o = torch.empty((m, n_out), device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    buf = ctypes.create_string_buffer(512)
    res = {}
    # one complete step on every rank
    assert cuda.edgexpu_cuda_linear_quant_batch_tp_dev(o.data_ptr(), xd.data_ptr(), h, wtype, None, m, n_out, per, st)
    assert cuda.edgexpu_cuda_stream_sync(st, buf, 512), buf.value
    dist.barrier()
    if rank == 0:  # rank 1 does not take part in this step
        t0 = time.time()
        assert cuda.edgexpu_cuda_linear_quant_batch_tp_dev(o.data_ptr(), xd.data_ptr(), h, wtype, None, m, n_out, per, st)
        ok = cuda.edgexpu_cuda_stream_sync(st, buf, 512)
        res["seconds"] = time.time() - t0
        res["ok"] = int(ok)
        res["msg"] = buf.value.decode()
        # the context is still usable: an ordinary launch afterwards succeeds
        assert cuda.edgexpu_cuda_linear_quant_batch_dev(o.data_ptr(), xd.data_ptr(), h, wtype, None, m, n_out, per, st)
        res["after"] = int(cuda.edgexpu_cuda_stream_sync(st, buf, 512))
    dist.barrier()
    # The exchange epochs of the ranks now disagree: the group is set up again before any further step.
    pkg.free_weight(h)
    cuda.edgexpu_cuda_tp_shutdown()
    pkg.shutdown()
    if rank == 0:
        import json

        with open(os.path.join(result_dir, "timeout.json"), "w") as f:
            json.dump(res, f)
    dist.destroy_process_group()


def test_tp_peer_timeout_is_reported(tmp_path):
    import json
    import random

    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_timeout_rank_main, args=(2, random.randint(20000, 40000), str(tmp_path)), nprocs=2, join=True)
    res = json.loads((tmp_path / "timeout.json").read_text())
    assert res["ok"] == 0 and "tensor-parallel peer" in res["msg"], res
    assert 1.5 < res["seconds"] < 30, res
    assert res["after"] == 1, res

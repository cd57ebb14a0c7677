"""The device-resident model (include/edgexpu_cuda.h): the HBM budget and the GGUF loader.

* CPU: edgexpu_cuda_hbm_plan_native restates the reference's resource plan (fill_native_plan,
  src/scheduler.c:320-422) with the weight term and limit of a resident model.  Its KV, scratch
  and limit terms and its admission decision are pinned against the reference's own
  edgexpu_scheduler_estimate_native (compiled in oracle/_ref/libedgexpu_ref_runtime.so) given the
  same weight bytes and memory size.
* GPU: a synthetic GGUF file (gguf_synth) is streamed into HBM; every row of every tensor read
  back through the device dequantizer equals the oracle's dequantization of the file's bytes,
  a linear through a loaded tensor is bit-identical to the oracle's x86-order linear, and a model
  whose KV cache cannot fit is refused without allocating.
"""

import ctypes
import os

import numpy as np
import pytest

import _oracle
from _oracle import TYPE_Q4_K, TYPE_Q8_0

RUNTIME = _oracle.REPO / "oracle" / "_ref" / "libedgexpu_ref_runtime.so"


class RefProfile(ctypes.Structure):
    """edgexpu_device_profile (include/edgexpu/profiler.h:14-24; EDGEXPU_TEXT_SMALL = 64)."""

    _fields_ = [("os", ctypes.c_char * 64), ("arch", ctypes.c_char * 64), ("cpu_count", ctypes.c_int),
                ("memory_total_mb", ctypes.c_int), ("has_llama_cli", ctypes.c_int),
                ("has_rockchip_runtime", ctypes.c_int), ("has_qualcomm_runtime", ctypes.c_int),
                ("simd", ctypes.c_char * 64), ("emulated", ctypes.c_int)]


class RefPlan(ctypes.Structure):
    """edgexpu_resource_plan (include/edgexpu/scheduler.h:37-47; EDGEXPU_TEXT_MEDIUM = 256)."""

    _fields_ = [("weight_bytes", ctypes.c_size_t), ("kv_bytes", ctypes.c_size_t), ("scratch_bytes", ctypes.c_size_t),
                ("total_bytes", ctypes.c_size_t), ("limit_bytes", ctypes.c_size_t), ("file_bytes", ctypes.c_size_t),
                ("window", ctypes.c_int), ("admitted", ctypes.c_int), ("reason", ctypes.c_char * 256)]


# (file bytes, layers, kv heads, head_dim, n_embd, n_ff, heads, window, memory MB)
PLAN_CASES = [
    (142_884_864, 30, 3, 64, 576, 1536, 9, 2048, 183_359),        # config 1 on a B200
    (4_600_000_000, 32, 8, 128, 4096, 14336, 32, 8192, 183_359),  # config 4
    (4_600_000_000, 32, 8, 0, 4096, 0, 32, 1, 4_096),             # defaults: head_dim, n_ff, tiny memory
    (4_600_000_000, 32, 8, 128, 4096, 14336, 32, 1 << 20, 183_359),  # KV beyond the limit
    (10_000, 2, 2, 32, 64, 128, 2, 0, 1),                         # window < 1
]


@pytest.mark.parametrize("case", PLAN_CASES)
def test_hbm_plan_matches_reference_budget_terms(case, monkeypatch):
    if not RUNTIME.exists():
        pytest.skip("reference runtime not built (oracle/_ref)")
    monkeypatch.delenv("EDGEXPU_BUDGET_DISABLE", raising=False)
    file_bytes, layers, kv_heads, head_dim, n_embd, n_ff, heads, window, mem_mb = case
    ref = ctypes.CDLL(str(RUNTIME))
    f = ref.edgexpu_scheduler_estimate_native
    f.restype = None
    f.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int, ctypes.c_uint32, ctypes.c_uint32,
                  ctypes.c_uint32, ctypes.c_int, ctypes.POINTER(RefProfile), ctypes.POINTER(RefPlan)]
    prof = RefProfile(memory_total_mb=mem_mb)
    rp = RefPlan()
    f(file_bytes, layers, kv_heads, head_dim, n_embd, n_ff, heads, window, ctypes.byref(prof), ctypes.byref(rp))

    pkg = _oracle.load_pkg()
    cuda = pkg.load_cuda()
    plan = pkg.HbmPlan()
    got = cuda.edgexpu_cuda_hbm_plan_native(file_bytes, rp.weight_bytes, layers, kv_heads, head_dim, n_embd, n_ff,
                                            heads, window, mem_mb * 1024 * 1024, ctypes.byref(plan))
    # same weight term in: every other term and the decision must agree with the reference's plan
    assert (plan.kv_bytes, plan.scratch_bytes, plan.total_bytes, plan.limit_bytes, plan.window) == \
        (rp.kv_bytes, rp.scratch_bytes, rp.total_bytes, rp.limit_bytes, rp.window)
    assert got == plan.admitted == rp.admitted
    assert (b"exceeds" in plan.reason) == (not plan.admitted)


def test_hbm_plan_budget_disable_and_unknown_memory(monkeypatch):
    pkg = _oracle.load_pkg()
    cuda = pkg.load_cuda()
    plan = pkg.HbmPlan()
    huge = 1 << 50
    assert cuda.edgexpu_cuda_hbm_plan_native(huge, huge, 1, 1, 64, 64, 64, 1, 1, 1 << 30, ctypes.byref(plan)) == 0
    monkeypatch.setenv("EDGEXPU_BUDGET_DISABLE", "1")
    assert cuda.edgexpu_cuda_hbm_plan_native(huge, huge, 1, 1, 64, 64, 64, 1, 1, 1 << 30, ctypes.byref(plan)) == 1
    assert b"disabled" in plan.reason
    monkeypatch.delenv("EDGEXPU_BUDGET_DISABLE")
    assert cuda.edgexpu_cuda_hbm_plan_native(huge, huge, 1, 1, 64, 64, 64, 1, 1, 0, ctypes.byref(plan)) == 1
    assert b"unknown" in plan.reason


# ---- GPU: the loader ----------------------------------------------------------------------------


def _shapes():
    from edgexpu_llm_b200 import gguf_synth as gs

    q8 = gs.SMOLLM2_135M_Q8_0.with_layers(2)
    q4 = gs.LlamaShape("tiny-q4_k", 512, 2, 8, 2, 1024, 1000, TYPE_Q4_K, False)
    return [q8, q4]


def _load(pkg, path, window):
    cuda = pkg.load_cuda()
    model = ctypes.c_void_p()
    plan = pkg.HbmPlan()
    err = ctypes.create_string_buffer(512)
    ok = cuda.edgexpu_cuda_gguf_load(str(path).encode(), window, ctypes.byref(model), ctypes.byref(plan), err, 512)
    return ok, model, plan, err.value


def _tensor(cuda, model, i):
    name, dev, typ = ctypes.c_char_p(), ctypes.c_void_p(), ctypes.c_uint32()
    n_in, n_out, off, nb = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_uint64(), ctypes.c_uint64()
    assert cuda.edgexpu_cuda_gguf_tensor_at(model, i, ctypes.byref(name), ctypes.byref(dev), ctypes.byref(typ),
                                            ctypes.byref(n_in), ctypes.byref(n_out), ctypes.byref(off), ctypes.byref(nb))
    return name.value.decode(), dev.value, typ.value, n_in.value, n_out.value, off.value, nb.value


@pytest.mark.gpu
@pytest.mark.parametrize("which", [0, 1])
def test_gguf_load_every_row_bit_exact(gpu, port, tmp_path, which):
    from edgexpu_llm_b200 import gguf_synth as gs

    shape = _shapes()[which]
    path = gs.write_llama_gguf(tmp_path / f"{shape.name}.gguf", shape, seed=3)
    data = path.read_bytes()
    cuda = gpu.load_cuda()
    ok, model, plan, msg = _load(gpu, path, 256)
    assert ok, msg
    try:
        assert plan.admitted and plan.weight_bytes <= len(data) and plan.file_bytes == len(data)
        n = cuda.edgexpu_cuda_gguf_tensor_count(model)
        assert n == len(gs._tensors(shape))
        for i in range(n):
            name, dev, typ, n_in, n_out, off, nb = _tensor(cuda, model, i)
            assert cuda.edgexpu_cuda_gguf_find(model, name.encode()) == i
            raw, wtype, dims = gs.read_tensor(path, name)
            assert typ == wtype and n_in == dims[0] and nb == raw.nbytes
            assert bytes(data[off:off + nb]) == raw.tobytes()
            rows = sorted({0, n_out // 2, n_out - 1})
            for r in rows:
                got = np.full(n_in, np.nan, np.float32)
                err = ctypes.create_string_buffer(256)
                assert cuda.edgexpu_cuda_dequantize_row(dev, typ, r, n_in, got.ctypes.data, err, 256), err.value
                if typ == 0:  # F32 norm weights: the file's floats themselves
                    want = raw[r].view(np.float32).copy()
                else:
                    want = np.empty(n_in, np.float32)
                    row = np.ascontiguousarray(raw[r])
                    assert port.lib.eo_dequantize_row(typ, row.ctypes.data, n_in, want.ctypes.data)
                np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32), err_msg=f"{name} row {r}")
        # a linear through a loaded tensor: bit-identical to the oracle's x86-order linear
        name = "blk.1.ffn_down.weight"
        i = cuda.edgexpu_cuda_gguf_find(model, name.encode())
        _, dev, typ, n_in, n_out, _, _ = _tensor(cuda, model, i)
        raw, _, _ = gs.read_tensor(path, name)
        x = np.random.default_rng(5).standard_normal((2, n_in)).astype(np.float32)
        assert cuda.edgexpu_cuda_set_float_order(gpu.ORDER_X86) == 1
        got = gpu.linear_quant_batch(x, dev, typ, n_out)
        want = port.linear(x, raw, typ, n_out, None, x86=True)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    finally:
        assert cuda.edgexpu_cuda_gguf_free(model) == 1


@pytest.mark.gpu
def test_gguf_load_refuses_a_model_over_budget(gpu, tmp_path):
    import torch
    from edgexpu_llm_b200 import gguf_synth as gs

    shape = _shapes()[0]
    path = gs.write_llama_gguf(tmp_path / "m.gguf", shape, seed=1)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    ok, model, plan, msg = _load(gpu, path, 1 << 30)  # fp32 KV for 2^30 positions: far beyond HBM
    assert not ok and not plan.admitted and model.value is None
    assert b"exceeds" in msg and plan.kv_bytes == 2 * 2 * 3 * 64 * (1 << 30) * 4
    assert torch.cuda.mem_get_info()[0] == free0
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUF" + b"\0" * 60)
    ok, model, _, msg = _load(gpu, bad, 16)
    assert not ok and msg


@pytest.mark.gpu
def test_preload_feeds_the_residency_table(gpu, tmp_path):
    """edgexpu_b200_preload enters every tensor under its address in the file mapping: the
    residency lookup of the reference's load_qweight then returns the preloaded device copy."""
    import mmap

    from edgexpu_llm_b200 import gguf_synth as gs

    shape = _shapes()[1]
    path = gs.write_llama_gguf(tmp_path / "p.gguf", shape, seed=2)
    host = gpu.load_host()
    cuda = gpu.load_cuda()
    with open(path, "rb") as fh:
        mm = mmap.mmap(fh.fileno(), 0, access=mmap.ACCESS_READ)
        buf = (ctypes.c_uint8 * len(mm)).from_buffer_copy(mm)  # stands in for the session's mapping
        base = ctypes.addressof(buf)
        err = ctypes.create_string_buffer(512)
        assert host.edgexpu_b200_preload(base, len(mm), str(path).encode(), 128, err, 512), err.value
        mm.close()
    raw, wtype, dims = gs.read_tensor(path, "blk.0.attn_q.weight")
    off = bytes(buf).find(raw.tobytes())
    resident = host.edgexpu_b200_resident
    dev = resident(base + off, raw.nbytes, wtype, dims[1], dims[0], err, 512)
    assert dev, err.value
    x = np.random.default_rng(9).standard_normal((1, dims[0])).astype(np.float32)
    got = gpu.linear_quant_batch(x, dev, wtype, dims[1])
    np.testing.assert_array_equal(got.view(np.uint32),
                                  _oracle.Port().linear(x, raw, wtype, dims[1], None, x86=True).view(np.uint32))
    host.edgexpu_b200_release_range(base, len(buf))
    # released with the mapping: the address is no longer a registered tensor
    y = np.zeros((1, dims[1]), np.float32)
    assert cuda.edgexpu_cuda_linear_quant_batch(y.ctypes.data, x.ctypes.data, dev, wtype, None, 1, dims[1], dims[0],
                                                err, 512) == 0

"""CPU tests of the drop-in boundary: the libraries load, export every declared symbol, and fail
loudly (no CPU fallback) when there is no CUDA device."""

import ctypes
import pathlib
import re
import subprocess

import numpy as np
import pytest

from _oracle import REPO, load_pkg

INCLUDE = REPO / "include"
DECL = re.compile(r"^(?!static)[A-Za-z_][\w \t\*]*?\b(edgexpu_\w+)\s*\(", re.M)


def declared(header: str):
    text = (INCLUDE / header).read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(DECL.findall(text)))


def exported(lib: pathlib.Path):
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib)], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


@pytest.fixture(scope="module")
def built():
    pkg = load_pkg()
    if not (pkg.CUDA_LIB.exists() and pkg.HOST_LIB.exists()):
        subprocess.run(["make", "-s", "-C", str(pkg.PKG_DIR)], check=True)
    return pkg


def test_headers_declare_the_boundary():
    cuda = declared("edgexpu_cuda.h")
    host = declared("edgexpu_b200_host.h")
    assert "edgexpu_cuda_linear_quant_batch" in cuda and "edgexpu_cuda_logits_argmax" in cuda
    assert "edgexpu_cpu_linear_quant_batch" in host and "edgexpu_gguf_quantize_q8_k" in host
    assert "edgexpu_cuda_argmax_key_id" not in cuda  # static inline helper, not an export


@pytest.mark.parametrize("header,libattr", [("edgexpu_cuda.h", "CUDA_LIB"), ("edgexpu_b200_host.h", "HOST_LIB")])
def test_library_exports_every_declared_symbol(built, header, libattr):
    syms = exported(getattr(built, libattr))
    missing = [f for f in declared(header) if f not in syms]
    assert not missing, f"{libattr} lacks {missing}"


def test_ctypes_binding_covers_the_headers(built):
    import edgexpu_llm_b200 as pkg

    assert set(declared("edgexpu_cuda.h")) == set(pkg._CUDA_SIGS)
    assert set(declared("edgexpu_b200_host.h")) == set(pkg._HOST_SIGS)
    cuda = built.load_cuda()
    host = built.load_host()
    assert cuda.edgexpu_cuda_abi_version() == 1
    assert host.edgexpu_gguf_q8_0_nbytes(576) == 612 and host.edgexpu_gguf_q8_k_nbytes(4096) == 4672
    assert host.edgexpu_gguf_q8_k_nbytes(100) == 0
    assert host.edgexpu_gguf_can_dot_q8(8) and not host.edgexpu_gguf_can_dot_q8(12)
    assert host.edgexpu_gguf_can_dot_q8k(12) and not host.edgexpu_gguf_can_dot_q8k(8)


def _have_gpu():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


@pytest.mark.skipif(_have_gpu(), reason="checks the no-device failure path")
def test_no_device_fails_loudly(built):
    cuda = built.load_cuda()
    buf = ctypes.create_string_buffer(512)
    assert cuda.edgexpu_cuda_init(0, buf, 512) == 0
    assert buf.value  # a message, not a silent CPU fallback


@pytest.mark.skipif(_have_gpu(), reason="checks the no-device failure path")
def test_linear_without_device_writes_nan_and_sticky_error(built):
    host = built.load_host()
    host.edgexpu_b200_clear_error()
    out = np.zeros((2, 8), np.float32)
    x = np.ones((2, 64), np.float32)
    fake_weight = np.zeros(8 * 68, np.uint8)
    host.edgexpu_cpu_linear_quant_batch(out.ctypes.data, x.ctypes.data, fake_weight.ctypes.data, 8, None, 2, 8, 64)
    assert np.all(np.isnan(out))
    assert b"edgexpu_cpu_linear_quant_batch" in host.edgexpu_b200_last_error()
    # the reference's silent return on bad arguments (cpu_kernel.c:562-564) is kept
    out[:] = 1.0
    host.edgexpu_b200_clear_error()
    host.edgexpu_cpu_linear_quant_batch(out.ctypes.data, x.ctypes.data, fake_weight.ctypes.data, 8, None, 0, 8, 64)
    assert np.all(out == 1.0) and host.edgexpu_b200_last_error() == b""
    q = np.zeros(34, np.uint8)
    assert host.edgexpu_gguf_quantize_q8_0(x.ctypes.data, 32, q.ctypes.data) == 0

"""edgexpu-llm_b200: B200 (sm_100a) implementation of EdgeXPU-LLM's quantized matrix-product path.

The product is two shared libraries built by ``make -C edgexpu-llm_b200``:

* ``lib/libedgexpu_cuda.so`` -- hand-written CUDA kernels behind the C ABI of
  ``include/edgexpu_cuda.h`` (``edgexpu_cuda_*``);
* ``lib/libedgexpu_b200_host.so`` -- the C host shim of ``include/edgexpu_b200_host.h``: the
  reference's own entry points (``edgexpu_cpu_linear_quant_batch``, ``edgexpu_gguf_quantize_q8_0``
  ...) with bodies that forward to the C ABI.

This module is a thin ctypes binding over both, used by the tests, ``bench.py`` and
``__graft_entry__``.  It never computes anything itself and has no CPU fallback: if a library
is missing, :func:`load_cuda` / :func:`load_host` raise.
"""

from __future__ import annotations

import ctypes
import pathlib

PKG_DIR = pathlib.Path(__file__).resolve().parent
LIB_DIR = PKG_DIR / "lib"
CUDA_LIB = LIB_DIR / "libedgexpu_cuda.so"
HOST_LIB = LIB_DIR / "libedgexpu_b200_host.so"

TYPE_F32, TYPE_F16, TYPE_Q4_0, TYPE_Q5_0 = 0, 1, 2, 6
TYPE_Q8_0 = 8
TYPE_Q4_K = 12
TYPE_Q5_K, TYPE_Q6_K = 13, 14
QK8_0, QK_K = 32, 256
ORDER_X86, ORDER_RELAXED = 0, 1  # EDGEXPU_CUDA_ORDER_* (include/edgexpu_cuda.h)
Q8_0_BYTES, Q8_K_BYTES, Q4_K_BYTES = 34, 292, 144

_c_u8p = ctypes.POINTER(ctypes.c_uint8)
_c_f32p = ctypes.POINTER(ctypes.c_float)
_c_vp = ctypes.c_void_p
_c_sz = ctypes.c_size_t
_c_int = ctypes.c_int
_c_u32 = ctypes.c_uint32
_c_str = ctypes.c_char_p
_c_u64 = ctypes.c_uint64
_c_i64p = ctypes.POINTER(ctypes.c_int64)
_c_u64p = ctypes.POINTER(ctypes.c_uint64)


class HbmPlan(ctypes.Structure):
    """edgexpu_cuda_hbm_plan (include/edgexpu_cuda.h)."""

    _fields_ = [("weight_bytes", ctypes.c_uint64), ("kv_bytes", ctypes.c_uint64), ("scratch_bytes", ctypes.c_uint64),
                ("total_bytes", ctypes.c_uint64), ("limit_bytes", ctypes.c_uint64), ("file_bytes", ctypes.c_uint64),
                ("window", ctypes.c_int), ("admitted", ctypes.c_int), ("reason", ctypes.c_char * 256)]


_CUDA_SIGS = {
    "edgexpu_cuda_abi_version": (_c_int, []),
    "edgexpu_cuda_set_float_order": (_c_int, [_c_int]),
    "edgexpu_cuda_float_order": (_c_int, []),
    "edgexpu_cuda_init": (_c_int, [_c_int, _c_str, _c_sz]),
    "edgexpu_cuda_shutdown": (_c_int, []),
    "edgexpu_cuda_last_error": (_c_str, []),
    "edgexpu_cuda_upload_weight": (_c_int, [_c_vp, _c_sz, _c_u32, _c_int, _c_int, ctypes.POINTER(_c_vp), _c_str, _c_sz]),
    "edgexpu_cuda_register_weight": (_c_int, [_c_vp, _c_sz, _c_u32, _c_int, _c_int, _c_str, _c_sz]),
    "edgexpu_cuda_free_weight": (_c_int, [_c_vp]),
    "edgexpu_cuda_quantize_q8_0": (_c_int, [_c_vp, _c_int, _c_vp, _c_str, _c_sz]),
    "edgexpu_cuda_quantize_q8_k": (_c_int, [_c_vp, _c_int, _c_vp, _c_str, _c_sz]),
    "edgexpu_cuda_linear_quant_batch": (
        _c_int, [_c_vp, _c_vp, _c_vp, _c_u32, _c_vp, _c_int, _c_int, _c_int, _c_str, _c_sz]),
    "edgexpu_cuda_logits_argmax": (
        _c_int, [_c_vp, _c_u32, _c_vp, _c_int, _c_int, _c_vp, ctypes.POINTER(_c_u32), _c_f32p, _c_str, _c_sz]),
    "edgexpu_cuda_quantize_dev": (_c_int, [_c_u32, _c_vp, _c_int, _c_int, _c_vp, _c_vp]),
    "edgexpu_cuda_linear_quant_batch_dev": (_c_int, [_c_vp, _c_vp, _c_vp, _c_u32, _c_vp, _c_int, _c_int, _c_int, _c_vp]),
    "edgexpu_cuda_linear_quant_multi_dev": (
        _c_int, [_c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_u32, _c_vp, _c_int, _c_int, _c_vp]),
    "edgexpu_cuda_linear_quant_batch_noalloc": (
        _c_int, [_c_vp, _c_vp, _c_vp, _c_u32, _c_vp, _c_int, _c_int, _c_int, _c_vp]),
    "edgexpu_cuda_dot_quant_q8_dev": (_c_int, [_c_vp, _c_vp, _c_vp, _c_u32, _c_vp, _c_int, _c_int, _c_int, _c_vp]),
    "edgexpu_cuda_logits_argmax_dev": (_c_int, [_c_vp, _c_u32, _c_vp, _c_int, _c_int, _c_vp, ctypes.c_int64, _c_vp, _c_vp]),
    "edgexpu_cuda_block_partials_dev": (_c_int, [_c_vp, _c_vp, _c_vp, _c_u32, _c_int, _c_int, _c_int, _c_vp]),
    "edgexpu_cuda_dot_quant": (_c_int, [_c_u32, _c_vp, _c_vp, _c_int, _c_int, _c_f32p, _c_str, _c_sz]),
    "edgexpu_cuda_dequantize_row": (_c_int, [_c_vp, _c_u32, ctypes.c_int64, _c_int, _c_vp, _c_str, _c_sz]),
    "edgexpu_cuda_dequantize_rows_dev": (_c_int, [_c_vp, _c_vp, _c_u32, _c_vp, _c_int, _c_int, _c_vp]),
    "edgexpu_cuda_reserve": (_c_int, [_c_int, _c_int, _c_str, _c_sz]),
    "edgexpu_cuda_stream_sync": (_c_int, [_c_vp, _c_str, _c_sz]),
    "edgexpu_cuda_tp_init": (_c_int, [_c_int, _c_int, _c_vp, _c_str, _c_sz]),
    "edgexpu_cuda_tp_connect": (_c_int, [_c_vp, _c_str, _c_sz]),
    "edgexpu_cuda_tp_shutdown": (_c_int, []),
    "edgexpu_cuda_linear_quant_batch_tp_dev": (_c_int, [_c_vp, _c_vp, _c_vp, _c_u32, _c_vp, _c_int, _c_int, _c_int,
                                                        _c_vp]),
    "edgexpu_cuda_sample_softmax": (_c_int, [_c_vp, _c_int, ctypes.c_float, _c_u64p, ctypes.POINTER(_c_u32), _c_str,
                                             _c_sz]),
    "edgexpu_cuda_logits_sample": (_c_int, [_c_vp, _c_u32, _c_vp, _c_int, _c_int, _c_vp, ctypes.c_float, ctypes.c_float,
                                            _c_u64p, ctypes.POINTER(_c_u32), _c_str, _c_sz]),
    "edgexpu_cuda_hbm_plan_native": (_c_int, [_c_u64, _c_u64, _c_u32, _c_u32, _c_int, _c_u32, _c_u32, _c_u32, _c_int,
                                              _c_u64, ctypes.POINTER(HbmPlan)]),
    "edgexpu_cuda_gguf_load": (_c_int, [_c_str, _c_int, ctypes.POINTER(_c_vp), ctypes.POINTER(HbmPlan), _c_str, _c_sz]),
    "edgexpu_cuda_gguf_tensor_count": (_c_int, [_c_vp]),
    "edgexpu_cuda_gguf_tensor_at": (_c_int, [_c_vp, _c_int, ctypes.POINTER(_c_str), ctypes.POINTER(_c_vp),
                                             ctypes.POINTER(_c_u32), _c_i64p, _c_i64p, _c_u64p, _c_u64p]),
    "edgexpu_cuda_gguf_find": (_c_int, [_c_vp, _c_str]),
    "edgexpu_cuda_gguf_meta": (_c_int, [_c_vp, _c_str, _c_u64p, ctypes.POINTER(ctypes.c_double),
                                        ctypes.POINTER(_c_str)]),
    "edgexpu_cuda_gguf_free": (_c_int, [_c_vp]),
    "edgexpu_cuda_llama_open": (_c_int, [_c_str, _c_int, ctypes.POINTER(_c_vp), _c_str, _c_sz]),
    "edgexpu_cuda_llama_forward": (_c_int, [_c_vp, _c_vp, _c_int, _c_int, ctypes.c_float, ctypes.c_float, _c_u64p,
                                            ctypes.POINTER(_c_u32), _c_vp, _c_str, _c_sz]),
    "edgexpu_cuda_llama_close": (_c_int, [_c_vp]),
}

_HOST_SIGS = {
    "edgexpu_b200_logits_sample": (_c_int, [_c_vp, _c_u32, _c_vp, _c_int, _c_int, _c_vp, ctypes.c_float, ctypes.c_float,
                                            _c_u64p, ctypes.POINTER(_c_u32), _c_str, _c_sz]),
    "edgexpu_b200_preload": (_c_int, [_c_vp, _c_sz, _c_str, _c_int, _c_str, _c_sz]),
    "edgexpu_cpu_linear_quant": (None, [_c_vp, _c_vp, _c_vp, _c_u32, _c_vp, _c_int, _c_int]),
    "edgexpu_cpu_linear_quant_batch": (None, [_c_vp, _c_vp, _c_vp, _c_u32, _c_vp, _c_int, _c_int, _c_int]),
    "edgexpu_gguf_q8_0_nbytes": (_c_sz, [_c_int]),
    "edgexpu_gguf_quantize_q8_0": (_c_int, [_c_vp, _c_int, _c_vp]),
    "edgexpu_gguf_can_dot_q8": (_c_int, [_c_u32]),
    "edgexpu_gguf_q8_k_nbytes": (_c_sz, [_c_int]),
    "edgexpu_gguf_quantize_q8_k": (_c_int, [_c_vp, _c_int, _c_vp]),
    "edgexpu_gguf_can_dot_q8k": (_c_int, [_c_u32]),
    "edgexpu_gguf_dot_quant_q8": (ctypes.c_float, [_c_u32, _c_vp, _c_vp, _c_int]),
    "edgexpu_gguf_dot_quant_q8k": (ctypes.c_float, [_c_u32, _c_vp, _c_vp, _c_int]),
    "edgexpu_gguf_dot_quant": (ctypes.c_float, [_c_u32, _c_vp, _c_vp, _c_int]),
    "edgexpu_b200_init": (_c_int, [_c_int, _c_str, _c_sz]),
    "edgexpu_b200_shutdown": (None, []),
    "edgexpu_b200_resident": (_c_vp, [_c_vp, _c_sz, _c_u32, _c_int, _c_int, _c_str, _c_sz]),
    "edgexpu_b200_release_range": (None, [_c_vp, _c_sz]),
    "edgexpu_b200_last_error": (_c_str, []),
    "edgexpu_b200_clear_error": (None, []),
    "edgexpu_b200_logits_greedy": (_c_int, [_c_vp, _c_u32, _c_vp, _c_int, _c_int, _c_vp, ctypes.POINTER(_c_u32), _c_str, _c_sz]),
}

_libs: dict[str, ctypes.CDLL] = {}


def _bind(path: pathlib.Path, sigs: dict) -> ctypes.CDLL:
    if not path.exists():
        raise ImportError(f"{path} is missing: build it with `make -C {PKG_DIR}` (no CPU fallback exists)")
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def load_cuda() -> ctypes.CDLL:
    """The CUDA C ABI (raises ImportError if the library has not been built)."""
    if "cuda" not in _libs:
        _libs["cuda"] = _bind(CUDA_LIB, _CUDA_SIGS)
    return _libs["cuda"]


def load_host() -> ctypes.CDLL:
    """The C host shim with the reference's entry-point names."""
    if "host" not in _libs:
        load_cuda()
        _libs["host"] = _bind(HOST_LIB, _HOST_SIGS)
    return _libs["host"]


class EdgexpuError(RuntimeError):
    pass


def _err_buf():
    return ctypes.create_string_buffer(512)


def _check(ok: int, buf=None) -> None:
    if not ok:
        msg = buf.value.decode() if buf is not None and buf.value else load_cuda().edgexpu_cuda_last_error().decode()
        raise EdgexpuError(msg)


# GGUF type id -> (elements per block, bytes per block), gguf_quant.c:69-106.
BLOCKS = {TYPE_F32: (1, 4), TYPE_F16: (1, 2), TYPE_Q4_0: (32, 18), TYPE_Q5_0: (32, 22), TYPE_Q8_0: (32, 34),
          TYPE_Q4_K: (256, 144), TYPE_Q5_K: (256, 176), TYPE_Q6_K: (256, 210)}
Q8_0_ACT_TYPES = (TYPE_Q8_0, TYPE_Q5_0, TYPE_Q4_0)  # edgexpu_gguf_can_dot_q8; the K-quants use Q8_K


def row_bytes(wtype: int, n: int) -> int:
    if wtype not in BLOCKS:
        raise ValueError(f"unsupported type {wtype}")
    qk, bb = BLOCKS[wtype]
    return (n // qk) * bb


def act_row_bytes(wtype: int, n: int) -> int:
    return (n // QK8_0) * Q8_0_BYTES if wtype in Q8_0_ACT_TYPES else (n // QK_K) * Q8_K_BYTES


def init(device: int = 0) -> None:
    buf = _err_buf()
    _check(load_cuda().edgexpu_cuda_init(device, buf, 512), buf)


def shutdown() -> None:
    load_cuda().edgexpu_cuda_shutdown()


def _ptr(a) -> int:
    """Address of a numpy array (host) or torch tensor (device or host)."""
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


def upload_weight(w_bytes, wtype: int, n_out: int, n_in: int) -> int:
    """Upload a packed GGUF tensor (numpy uint8) once; returns the device handle (int)."""
    import numpy as np

    w_bytes = np.ascontiguousarray(w_bytes, dtype=np.uint8)
    h = _c_vp()
    buf = _err_buf()
    _check(load_cuda().edgexpu_cuda_upload_weight(w_bytes.ctypes.data, w_bytes.nbytes, wtype, n_out, n_in,
                                                  ctypes.byref(h), buf, 512), buf)
    return int(h.value)


def register_weight(dev_tensor, wtype: int, n_out: int, n_in: int) -> int:
    """Register caller-owned device memory (a torch uint8 CUDA tensor with >= 16 spare bytes)."""
    buf = _err_buf()
    _check(load_cuda().edgexpu_cuda_register_weight(dev_tensor.data_ptr(), dev_tensor.numel(), wtype, n_out, n_in,
                                                    buf, 512), buf)
    return int(dev_tensor.data_ptr())


def free_weight(handle: int) -> None:
    load_cuda().edgexpu_cuda_free_weight(handle)


def quantize(x, wtype: int):
    """Quantize one fp32 row on the GPU through the host-buffer C ABI (returns numpy uint8)."""
    import numpy as np

    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(act_row_bytes(wtype, x.size), np.uint8)
    buf = _err_buf()
    fn = load_cuda().edgexpu_cuda_quantize_q8_0 if wtype in Q8_0_ACT_TYPES else load_cuda().edgexpu_cuda_quantize_q8_k
    _check(fn(x.ctypes.data, x.size, out.ctypes.data, buf, 512), buf)
    return out


def linear_quant_batch(x, handle: int, wtype: int, n_out: int, bias=None):
    """out[m][n_out] through the reference-named host shim ``edgexpu_cpu_linear_quant_batch``."""
    import numpy as np

    host = load_host()
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None, :]
    m, n_in = x.shape
    out = np.empty((m, n_out), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    host.edgexpu_b200_clear_error()
    host.edgexpu_cpu_linear_quant_batch(out.ctypes.data, x.ctypes.data, handle, wtype,
                                        None if b is None else b.ctypes.data, m, n_out, n_in)
    err = host.edgexpu_b200_last_error()
    if err:
        raise EdgexpuError(err.decode())
    return out


def logits_greedy(handle: int, wtype: int, hidden, vocab: int, bias=None):
    """(token_id, best_score) through the C ABI's synchronous greedy-logits call."""
    import numpy as np

    h = np.ascontiguousarray(hidden, dtype=np.float32).ravel()
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    tok = _c_u32()
    score = ctypes.c_float()
    buf = _err_buf()
    _check(load_cuda().edgexpu_cuda_logits_argmax(handle, wtype, h.ctypes.data, h.size, vocab,
                                                  None if b is None else b.ctypes.data, ctypes.byref(tok),
                                                  ctypes.byref(score), buf, 512), buf)
    return int(tok.value), float(score.value)


def key_to_id(key: int) -> int:
    return 0 if key == 0 else 0xFFFFFFFF - (key & 0xFFFFFFFF)

"""ctypes bindings of the oracle libraries (test infrastructure, never the product).

* ``oracle/liboracle_port.so`` -- our C restatement of the reference path (always buildable).
* ``oracle/_ref/libedgexpu_ref_avx2.so`` / ``_scalar.so`` -- the reference's own sources compiled
  by ``oracle/Makefile``; present in the development container and shipped prebuilt to GPU boxes.
"""

from __future__ import annotations

import ctypes
import importlib.util
import os
import pathlib
import subprocess
import sys

import numpy as np

REPO = pathlib.Path(__file__).resolve().parent.parent
ORACLE_DIR = REPO / "oracle"
PORT_LIB = ORACLE_DIR / "liboracle_port.so"
REF_AVX2 = ORACLE_DIR / "_ref" / "libedgexpu_ref_avx2.so"
REF_SCALAR = ORACLE_DIR / "_ref" / "libedgexpu_ref_scalar.so"
# The reference checkout (development container only): $EDGEXPU_REFERENCE, else a sibling directory
# of this repository named "reference".
REFERENCE = pathlib.Path(os.environ.get("EDGEXPU_REFERENCE", str(REPO.parent / "reference")))
REF_SRC = REFERENCE / "src"

TYPE_Q4_0, TYPE_Q5_0, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K = 2, 6, 8, 12, 13, 14
ALL_TYPES = (TYPE_Q4_0, TYPE_Q5_0, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K)
B32_TYPES = (TYPE_Q4_0, TYPE_Q5_0, TYPE_Q8_0)  # Q8_0 activations (can_dot_q8)
BLOCK = {TYPE_Q4_0: (32, 18), TYPE_Q5_0: (32, 22), TYPE_Q8_0: (32, 34), TYPE_Q4_K: (256, 144),
         TYPE_Q5_K: (256, 176), TYPE_Q6_K: (256, 210)}


def act_is_q8_0(wtype: int) -> bool:
    return wtype in B32_TYPES


_vp, _int, _u32, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_size_t


def load_pkg():
    """Import the package directory ``edgexpu-llm_b200`` as module ``edgexpu_llm_b200``."""
    name = "edgexpu_llm_b200"
    if name in sys.modules:
        return sys.modules[name]
    root = REPO / "edgexpu-llm_b200"
    spec = importlib.util.spec_from_file_location(name, root / "__init__.py", submodule_search_locations=[str(root)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def ensure_port() -> pathlib.Path:
    if not PORT_LIB.exists():
        subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), "port"], check=True)
    return PORT_LIB


def ensure_ref() -> bool:
    if REF_AVX2.exists() and REF_SCALAR.exists():
        return True
    if REF_SRC.exists():
        subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), "ref", f"REF={REFERENCE}"], check=True)
        return REF_AVX2.exists()
    return False


class Port:
    """Our restatement (oracle/edgexpu_oracle.c)."""

    def __init__(self):
        lib = ctypes.CDLL(str(ensure_port()))
        sig = {
            "eo_fp32_to_fp16": (ctypes.c_uint16, [ctypes.c_float]),
            "eo_fp32_to_fp16_trunc": (ctypes.c_uint16, [ctypes.c_float]),
            "eo_fp16_to_fp32": (ctypes.c_float, [ctypes.c_uint16]),
            "eo_quantize_q8_0": (_int, [_vp, _int, _vp]),
            "eo_quantize_q8_0_scalar": (_int, [_vp, _int, _vp]),
            "eo_quantize_q8_k": (_int, [_vp, _int, _vp]),
            "eo_partials_q8_0": (_int, [_vp, _vp, _int, _vp]),
            "eo_partials_q4_k": (_int, [_vp, _vp, _int, _vp, _vp]),
            "eo_partials_b32": (_int, [_u32, _vp, _vp, _int, _vp]),
            "eo_partials_k": (_int, [_u32, _vp, _vp, _int, _vp, _vp]),
            "eo_dot_q8": (ctypes.c_float, [_u32, _vp, _vp, _int]),
            "eo_dot_f32": (ctypes.c_float, [_u32, _vp, _vp, _int]),
            "eo_dot_q8_x86": (ctypes.c_float, [_u32, _vp, _vp, _int]),
            "eo_dot_f32_x86": (ctypes.c_float, [_u32, _vp, _vp, _int]),
            "eo_linear_quant_batch_x86": (_int, [_vp, _vp, _vp, _u32, _vp, _int, _int, _int]),
            "eo_logits_argmax_x86": (_int, [_vp, _u32, _vp, _int, _int, _vp, ctypes.POINTER(_u32),
                                            ctypes.POINTER(ctypes.c_float), _vp]),
            "eo_dot_q8_0_q8_0": (ctypes.c_float, [_vp, _vp, _int]),
            "eo_dot_q4_k_q8_k": (ctypes.c_float, [_vp, _vp, _int]),
            "eo_dot_q4_k_f32": (ctypes.c_float, [_vp, _vp, _int]),
            "eo_dot_q8_0_f32": (ctypes.c_float, [_vp, _vp, _int]),
            "eo_abs_bound_q8": (ctypes.c_double, [_u32, _vp, _vp, _int]),
            "eo_abs_bound_f32": (ctypes.c_double, [_u32, _vp, _vp, _int]),
            "eo_dequantize_row": (_int, [_u32, _vp, _int, _vp]),
            "eo_linear_quant_batch": (_int, [_vp, _vp, _vp, _u32, _vp, _int, _int, _int]),
            "eo_linear_quant_batch_bound": (_int, [_vp, _vp, _vp, _u32, _int, _int, _int]),
            "eo_logits_argmax": (_int, [_vp, _u32, _vp, _int, _int, _vp, ctypes.POINTER(_u32),
                                        ctypes.POINTER(ctypes.c_float), _vp]),
        }
        for k, (r, a) in sig.items():
            f = getattr(lib, k)
            f.restype, f.argtypes = r, a
        self.lib = lib

    def quantize(self, x: np.ndarray, wtype: int, scalar: bool = False) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        if x.ndim == 1:
            x = x[None]
        rows = []
        for r in x:
            if act_is_q8_0(wtype):
                out = np.empty(r.size // 32 * 34, np.uint8)
                fn = self.lib.eo_quantize_q8_0_scalar if scalar else self.lib.eo_quantize_q8_0
            else:
                out = np.empty(r.size // 256 * 292, np.uint8)
                fn = self.lib.eo_quantize_q8_k
            assert fn(r.ctypes.data, r.size, out.ctypes.data) == 1
            rows.append(out)
        return np.stack(rows)

    def partials(self, w: np.ndarray, xq: np.ndarray, wtype: int, n_in: int) -> np.ndarray:
        """[m][n_out][nb] (32-element types) or [m][n_out][nb][2] (K-quants) int32 per-block partials."""
        w = np.ascontiguousarray(w, np.uint8)
        xq = np.ascontiguousarray(xq, np.uint8)
        n_out, m = w.shape[0], xq.shape[0]
        if act_is_q8_0(wtype):
            nb = n_in // 32
            out = np.empty((m, n_out, nb), np.int32)
            for t in range(m):
                for o in range(n_out):
                    assert self.lib.eo_partials_b32(wtype, w[o].ctypes.data, xq[t].ctypes.data, n_in,
                                                    out[t, o].ctypes.data)
            return out
        nb = n_in // 256
        out = np.empty((m, n_out, nb, 2), np.int32)
        si = np.empty(nb, np.int32)
        sm = np.empty(nb, np.int32)
        for t in range(m):
            for o in range(n_out):
                assert self.lib.eo_partials_k(wtype, w[o].ctypes.data, xq[t].ctypes.data, n_in, si.ctypes.data,
                                              sm.ctypes.data)
                out[t, o, :, 0] = si
                out[t, o, :, 1] = sm
        return out

    def linear(self, x, w, wtype, n_out, bias=None, x86=False):
        """x86=True: the reference x86 build's float order (bit-identical), else its scalar order."""
        x = np.ascontiguousarray(x, np.float32)
        if x.ndim == 1:
            x = x[None]
        w = np.ascontiguousarray(w, np.uint8)
        m, n_in = x.shape
        out = np.empty((m, n_out), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        fn = self.lib.eo_linear_quant_batch_x86 if x86 else self.lib.eo_linear_quant_batch
        assert fn(out.ctypes.data, x.ctypes.data, w.ctypes.data, wtype, None if b is None else b.ctypes.data, m,
                  n_out, n_in) == 1
        return out

    def linear_bound(self, x, w, wtype, n_out):
        x = np.ascontiguousarray(x, np.float32)
        if x.ndim == 1:
            x = x[None]
        w = np.ascontiguousarray(w, np.uint8)
        m, n_in = x.shape
        out = np.empty((m, n_out), np.float64)
        assert self.lib.eo_linear_quant_batch_bound(out.ctypes.data, x.ctypes.data, w.ctypes.data, wtype,
                                                    m, n_out, n_in) == 1
        return out

    def logits(self, w, wtype, hidden, vocab, bias=None, x86=False):
        w = np.ascontiguousarray(w, np.uint8)
        h = np.ascontiguousarray(hidden, np.float32).ravel()
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        tok = _u32()
        sc = ctypes.c_float()
        scores = np.empty(vocab, np.float32)
        fn = self.lib.eo_logits_argmax_x86 if x86 else self.lib.eo_logits_argmax
        assert fn(w.ctypes.data, wtype, h.ctypes.data, h.size, vocab,
                                         None if b is None else b.ctypes.data, ctypes.byref(tok),
                                         ctypes.byref(sc), scores.ctypes.data) == 1
        return int(tok.value), float(sc.value), scores

    def logits_bound(self, w, wtype, hidden, rows):
        """Per-row tolerance bound of the logits dot (quantized hidden for the Q8_0-activation types,
        fp32 for the K-quants)."""
        w = np.ascontiguousarray(w, np.uint8)
        h = np.ascontiguousarray(hidden, np.float32).ravel()
        if act_is_q8_0(wtype):
            hq = self.quantize(h, TYPE_Q8_0)[0]
            return np.array([self.lib.eo_abs_bound_q8(wtype, w[r].ctypes.data, hq.ctypes.data, h.size) for r in rows])
        return np.array([self.lib.eo_abs_bound_f32(wtype, w[r].ctypes.data, h.ctypes.data, h.size) for r in rows])


class Ref:
    """The reference's own hot-path sources, compiled by oracle/Makefile."""

    def __init__(self, path: pathlib.Path):
        lib = ctypes.CDLL(str(path))
        sig = {
            "edgexpu_gguf_quantize_q8_0": (_int, [_vp, _int, _vp]),
            "edgexpu_gguf_quantize_q8_k": (_int, [_vp, _int, _vp]),
            "edgexpu_gguf_dot_quant_q8": (ctypes.c_float, [_u32, _vp, _vp, _int]),
            "edgexpu_gguf_dot_quant_q8k": (ctypes.c_float, [_u32, _vp, _vp, _int]),
            "edgexpu_gguf_dot_quant": (ctypes.c_float, [_u32, _vp, _vp, _int]),
            "edgexpu_cpu_linear_quant_batch": (None, [_vp, _vp, _vp, _u32, _vp, _int, _int, _int]),
            "edgexpu_gguf_quant_selftest": (_int, [ctypes.c_char_p, _sz]),
            "edgexpu_cpu_simd_name": (ctypes.c_char_p, []),
        }
        for k, (r, a) in sig.items():
            f = getattr(lib, k)
            f.restype, f.argtypes = r, a
        self.lib = lib

    def quantize(self, x, wtype):
        x = np.ascontiguousarray(x, np.float32)
        if x.ndim == 1:
            x = x[None]
        rows = []
        for r in x:
            if act_is_q8_0(wtype):
                out = np.empty(r.size // 32 * 34, np.uint8)
                assert self.lib.edgexpu_gguf_quantize_q8_0(r.ctypes.data, r.size, out.ctypes.data) == 1
            else:
                out = np.empty(r.size // 256 * 292, np.uint8)
                assert self.lib.edgexpu_gguf_quantize_q8_k(r.ctypes.data, r.size, out.ctypes.data) == 1
            rows.append(out)
        return np.stack(rows)

    def dot_q8(self, wtype, wrow, xq, n):
        wrow = np.ascontiguousarray(wrow, np.uint8)
        xq = np.ascontiguousarray(xq, np.uint8)
        fn = self.lib.edgexpu_gguf_dot_quant_q8 if act_is_q8_0(wtype) else self.lib.edgexpu_gguf_dot_quant_q8k
        return fn(wtype, wrow.ctypes.data, xq.ctypes.data, n)

    def dot_f32(self, wtype, wrow, x, n):
        wrow = np.ascontiguousarray(wrow, np.uint8)
        x = np.ascontiguousarray(x, np.float32)
        return self.lib.edgexpu_gguf_dot_quant(wtype, wrow.ctypes.data, x.ctypes.data, n)

    def linear(self, x, w, wtype, n_out, bias=None):
        x = np.ascontiguousarray(x, np.float32)
        if x.ndim == 1:
            x = x[None]
        w = np.ascontiguousarray(w, np.uint8)
        m, n_in = x.shape
        out = np.full((m, n_out), np.nan, np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self.lib.edgexpu_cpu_linear_quant_batch(out.ctypes.data, x.ctypes.data, w.ctypes.data, wtype,
                                                None if b is None else b.ctypes.data, m, n_out, n_in)
        return out

    def logits(self, w, wtype, hidden, vocab, bias=None):
        """Greedy argmax restated over the reference's own per-row dots (native.c:2355-2397)."""
        w = np.ascontiguousarray(w, np.uint8)
        h = np.ascontiguousarray(hidden, np.float32).ravel()
        n = h.size
        if act_is_q8_0(wtype):
            hq = self.quantize(h, TYPE_Q8_0)[0]
            scores = np.array([self.dot_q8(wtype, w[i], hq, n) for i in range(vocab)], np.float32)
        else:
            scores = np.array([self.dot_f32(wtype, w[i], h, n) for i in range(vocab)], np.float32)
        if bias is not None:
            scores = scores + np.asarray(bias, np.float32)
        best, bs = 0, -np.inf
        for i, s in enumerate(scores):
            if s > bs:
                best, bs = i, s
        return best, float(bs), scores

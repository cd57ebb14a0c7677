"""End-to-end greedy decode through the reference's own layer loop, token-identical to the reference.

Two builds of the same reference runtime (src/native.c and the rest of src/, compiled from the
reference's sources) run the same seeded synthetic GGUF model and prompt:

* oracle/_ref/libedgexpu_ref_runtime.so -- the reference unchanged: every quantized matrix product
  and the greedy logits on the CPU (x86 Release flags);
* integration/_build/libedgexpu_native_b200.so -- the reference with integration/edgexpu_b200.patch
  and the C host shim dropped in: weights resident in HBM, every linear and the greedy logits on the
  B200, the rest of the layer loop (norms, RoPE, attention, SwiGLU, KV cache) unchanged on the CPU.

Both are driven by integration/greedy_driver.c through the reference's public session API:
prefill of the prompt ids, then greedy steps (edgexpu_native_generate_next, temperature 0).  The bar
is the reference's own (``greedy_ids=`` of its verify scripts): identical token ids at every step.
The test also reports each step's top-2 logit margin (the oracle's logits on the reference's hidden
state), so a mismatch can be told from a near-tie.

Configurations (BASELINE): 1 = SmolLM2-135M-shaped, all Q8_0, 128 prompt + 128 greedy tokens, full
size; 4 = Llama-3-8B-shaped, all Q4_K, 512 prompt + 256 greedy tokens, with 4 of its 32 layers (full
width and vocabulary) to keep the CPU reference run short.
"""

import ctypes
import pathlib

import numpy as np
import pytest

from _oracle import REPO

pytestmark = pytest.mark.gpu

REF_RUNTIME = REPO / "oracle" / "_ref" / "libedgexpu_ref_runtime.so"
B200_RUNTIME = REPO / "integration" / "_build" / "libedgexpu_native_b200.so"


def _bind(path: pathlib.Path):
    if not path.exists():
        pytest.fail(f"{path} is missing: build it (oracle/Makefile `ref`, integration/Makefile)")
    lib = ctypes.CDLL(str(path))
    f = lib.edgexpu_greedy_run
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                  ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
    return lib


def greedy(lib, path, prompt, n_new, n_embd, hidden=False):
    ids = np.zeros(n_new, np.uint32)
    hid = np.zeros((n_new, n_embd), np.float32) if hidden else None
    secs = np.zeros(2)
    err = ctypes.create_string_buffer(1024)
    made = lib.edgexpu_greedy_run(str(path).encode(), prompt.ctypes.data, prompt.size, n_new, ids.ctypes.data,
                                  None if hid is None else hid.ctypes.data, n_embd, secs.ctypes.data, err, 1024)
    assert made == n_new, err.value.decode(errors="replace")
    return ids, hid, secs


def margins(port, path, shape, hid):
    from edgexpu_llm_b200 import gguf_synth as gs

    w, wtype, _ = gs.read_tensor(path, "token_embd.weight" if shape.tied else "output.weight")
    out = []
    for h in hid:
        _, _, scores = port.logits(w, wtype, h, shape.vocab)
        s = np.sort(scores)
        out.append(float(s[-1] - s[-2]))
    return np.array(out)


CASES = [("smollm2_135m_q8_0", 0, 128, 128), ("llama3_8b_q4_k_4l", 4, 512, 256)]


@pytest.mark.parametrize("name,layers,n_prompt,n_new", CASES)
def test_greedy_ids_identical_to_reference(gpu, port, tmp_path, name, layers, n_prompt, n_new):
    from edgexpu_llm_b200 import gguf_synth as gs

    shape = gs.SMOLLM2_135M_Q8_0 if name.startswith("smollm2") else gs.LLAMA3_8B_Q4_K
    if layers:
        shape = shape.with_layers(layers)
    path = gs.write_llama_gguf(tmp_path / f"{name}.gguf", shape, seed=0)
    prompt = gs.prompt_ids(shape, n_prompt, seed=0)
    ref = _bind(REF_RUNTIME)
    b200 = _bind(B200_RUNTIME)
    ids_ref, hid_ref, t_ref = greedy(ref, path, prompt, n_new, shape.n_embd, hidden=True)
    ids_gpu, hid_gpu, t_gpu = greedy(b200, path, prompt, n_new, shape.n_embd, hidden=True)
    mg = margins(port, path, shape, hid_ref)
    rel = np.abs(hid_gpu - hid_ref).max(axis=1) / np.abs(hid_ref).max(axis=1)
    print(f"\n{name}: prefill {n_prompt} tokens ref {t_ref[0]:.3f} s / b200 {t_gpu[0]:.3f} s; "
          f"decode {n_new} tokens ref {t_ref[1]:.3f} s ({n_new / t_ref[1]:.1f} tok/s) / b200 {t_gpu[1]:.3f} s "
          f"({n_new / t_gpu[1]:.1f} tok/s); min top-2 margin {mg.min():.3e}; "
          f"max hidden-state rel. diff {rel.max():.2e}")
    bad = np.flatnonzero(ids_ref != ids_gpu)
    assert bad.size == 0, (f"first differing step {bad[0]}: ref {ids_ref[bad[0]]} b200 {ids_gpu[bad[0]]}, "
                           f"top-2 margin there {mg[bad[0]]:.3e}, hidden rel. diff {rel[bad[0]]:.2e}")
    assert np.all(mg > 0), "an exact tie in the reference's logits"


def test_model_reload_releases_resident_weights(gpu, tmp_path):
    """Two models loaded one after the other (the second may be mapped at the first one's
    addresses): the residency table is released on unmap, so the second run uses its own weights."""
    from edgexpu_llm_b200 import gguf_synth as gs

    shape = gs.SMOLLM2_135M_Q8_0.with_layers(2)
    p0 = gs.write_llama_gguf(tmp_path / "a.gguf", shape, seed=0)
    p1 = gs.write_llama_gguf(tmp_path / "b.gguf", shape, seed=1)
    prompt = gs.prompt_ids(shape, 16, seed=0)
    ref, b200 = _bind(REF_RUNTIME), _bind(B200_RUNTIME)
    for p in (p0, p1, p0):
        want, _, _ = greedy(ref, p, prompt, 8, shape.n_embd)
        got, _, _ = greedy(b200, p, prompt, 8, shape.n_embd)
        np.testing.assert_array_equal(got, want)

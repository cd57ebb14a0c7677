"""Seeded synthetic GGUF model files for the end-to-end greedy decode through the reference's own
layer loop (``src/native.c``), with random-init weights of a named architecture's shape.

The file follows the GGUF v3 layout that the reference's parser reads (``src/gguf.c:359-610``):
magic ``GGUF``, version 3, tensor count, metadata count; metadata as (key, type, value); tensor
infos as (name, n_dims, dims with dims[0] = the row length, type, offset); the data section starts
at the next 32-byte boundary and every tensor starts 32-byte aligned inside it.

Metadata written (``llama`` architecture, the keys ``apply_gguf_u32_key`` and the f32 branch of
``edgexpu_gguf_load`` consume): block count, context length, embedding length, feed-forward
length, head counts, RMS epsilon, RoPE frequency base; ``tokenizer.ggml.model = "gpt2"`` with a
vocabulary of distinct placeholder pieces (the vocabulary size is the logits width,
``native.c:2309``), no merges, and an end-of-sequence id outside the vocabulary so greedy decoding
never stops early (``native.c:2643-2649``).  Prompts are token ids, set directly.

Weights follow the benchmark recipes of ``synth.py`` (Q8_0: d ~ U(1e-4, 2e-3), qs ~ U{-127..127};
Q4_K: d, dmin ~ U(1e-4, 1e-3), uniform scale and quant bytes); norm weights are fp32 1 + N(0, 0.02).
"""

from __future__ import annotations

import dataclasses
import pathlib
import struct

import numpy as np

from . import synth

GGUF_U32, GGUF_F32, GGUF_STRING, GGUF_ARRAY = 4, 6, 8, 9
TYPE_F32 = 0
ALIGN = 32


@dataclasses.dataclass(frozen=True)
class LlamaShape:
    """A llama-architecture decoder (the reference's ``llama`` plugin, ``src/arch/llama.c``)."""

    name: str
    n_embd: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    n_ff: int
    vocab: int
    wtype: int                  # GGUF type of every projection and of the embedding
    tied: bool                  # logits from token_embd (no output.weight)
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0
    context: int = 2048

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_heads

    def with_layers(self, n_layers: int) -> "LlamaShape":
        return dataclasses.replace(self, n_layers=n_layers, name=f"{self.name}-{n_layers}l")

    def weight_bytes_per_token(self) -> int:
        """Bytes of quantized weights one decode token streams (every projection + the logits)."""
        rb = synth.row_bytes
        kv = self.n_kv_heads * self.head_dim
        layer = (rb(self.wtype, self.n_embd) * (2 * self.n_embd + 2 * kv + 2 * self.n_ff)
                 + rb(self.wtype, self.n_ff) * self.n_embd)
        return self.n_layers * layer + rb(self.wtype, self.n_embd) * self.vocab


# Configuration 1: SmolLM2-135M-shaped, all Q8_0, tied embeddings, RoPE theta 1e5.
SMOLLM2_135M_Q8_0 = LlamaShape("smollm2-135m-q8_0", 576, 30, 9, 3, 1536, 49152, synth.TYPE_Q8_0, True,
                               rope_theta=1e5)
# Configuration 4: Llama-3-8B-shaped, all Q4_K, separate output.weight; RoPE theta 5e5 (not given by
# the configuration; Llama 3's value).
LLAMA3_8B_Q4_K = LlamaShape("llama3-8b-q4_k", 4096, 32, 32, 8, 14336, 128256, synth.TYPE_Q4_K, False,
                            rope_theta=5e5)


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv_u32(key: str, v: int) -> bytes:
    return _str(key) + struct.pack("<II", GGUF_U32, v)


def _kv_f32(key: str, v: float) -> bytes:
    return _str(key) + struct.pack("<If", GGUF_F32, v)


def _kv_str(key: str, v: str) -> bytes:
    return _str(key) + struct.pack("<I", GGUF_STRING) + _str(v)


def _kv_str_array(key: str, items) -> bytes:
    parts = [_str(key), struct.pack("<IIQ", GGUF_ARRAY, GGUF_STRING, len(items))]
    parts.extend(_str(s) for s in items)
    return b"".join(parts)


def _tensors(shape: LlamaShape):
    """(name, n_in, n_out, type) of every tensor of the model, in file order."""
    kv = shape.n_kv_heads * shape.head_dim
    out = [("token_embd.weight", shape.n_embd, shape.vocab, shape.wtype)]
    for i in range(shape.n_layers):
        p = f"blk.{i}."
        out += [(p + "attn_norm.weight", shape.n_embd, 1, TYPE_F32),
                (p + "ffn_norm.weight", shape.n_embd, 1, TYPE_F32),
                (p + "attn_q.weight", shape.n_embd, shape.n_embd, shape.wtype),
                (p + "attn_k.weight", shape.n_embd, kv, shape.wtype),
                (p + "attn_v.weight", shape.n_embd, kv, shape.wtype),
                (p + "attn_output.weight", shape.n_embd, shape.n_embd, shape.wtype),
                (p + "ffn_gate.weight", shape.n_embd, shape.n_ff, shape.wtype),
                (p + "ffn_up.weight", shape.n_embd, shape.n_ff, shape.wtype),
                (p + "ffn_down.weight", shape.n_ff, shape.n_embd, shape.wtype)]
    out.append(("output_norm.weight", shape.n_embd, 1, TYPE_F32))
    if not shape.tied:
        out.append(("output.weight", shape.n_embd, shape.vocab, shape.wtype))
    return out


def _tensor_bytes(rng: np.random.Generator, n_in: int, n_out: int, wtype: int) -> np.ndarray:
    if wtype == TYPE_F32:
        return (1.0 + 0.02 * rng.standard_normal(n_in * n_out)).astype(np.float32).view(np.uint8)
    rows = []
    chunk = max(1, (64 << 20) // max(1, synth.row_bytes(wtype, n_in)))  # bound the temporary size
    for r0 in range(0, n_out, chunk):
        rows.append(synth.weight(rng, wtype, min(chunk, n_out - r0), n_in).reshape(-1))
    return np.concatenate(rows)


def write_llama_gguf(path, shape: LlamaShape, seed: int = 0) -> pathlib.Path:
    """Write a random-init GGUF file of `shape` to `path` (seeded) and return the path."""
    path = pathlib.Path(path)
    rng = np.random.default_rng(seed)
    tensors = _tensors(shape)
    arch = "llama"
    meta = [
        _kv_str("general.architecture", arch),
        _kv_str("general.name", shape.name),
        _kv_u32(f"{arch}.block_count", shape.n_layers),
        _kv_u32(f"{arch}.context_length", shape.context),
        _kv_u32(f"{arch}.embedding_length", shape.n_embd),
        _kv_u32(f"{arch}.feed_forward_length", shape.n_ff),
        _kv_u32(f"{arch}.attention.head_count", shape.n_heads),
        _kv_u32(f"{arch}.attention.head_count_kv", shape.n_kv_heads),
        _kv_f32(f"{arch}.attention.layer_norm_rms_epsilon", shape.rms_eps),
        _kv_f32(f"{arch}.rope.freq_base", shape.rope_theta),
        _kv_str("tokenizer.ggml.model", "gpt2"),
        _kv_str_array("tokenizer.ggml.tokens", [f"<t{i}>" for i in range(shape.vocab)]),
        _kv_u32("tokenizer.ggml.bos_token_id", shape.vocab + 1),
        _kv_u32("tokenizer.ggml.eos_token_id", shape.vocab + 2),
    ]
    infos, offsets, off = [], [], 0
    for name, n_in, n_out, wtype in tensors:
        nbytes = synth.row_bytes(wtype, n_in) * n_out if wtype != TYPE_F32 else 4 * n_in * n_out
        dims = (n_in,) if n_out == 1 else (n_in, n_out)
        infos.append(_str(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims) +
                     struct.pack("<IQ", wtype, off))
        offsets.append((off, nbytes))
        off = (off + nbytes + ALIGN - 1) // ALIGN * ALIGN
    header = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(meta)) + b"".join(meta) + b"".join(infos)
    pad = (-len(header)) % ALIGN
    with open(path, "wb") as f:
        f.write(header + b"\0" * pad)
        pos = 0
        for (name, n_in, n_out, wtype), (o, nbytes) in zip(tensors, offsets):
            if o > pos:
                f.write(b"\0" * (o - pos))
            data = _tensor_bytes(rng, n_in, n_out, wtype)
            assert data.nbytes == nbytes, name
            f.write(data.tobytes())
            pos = o + nbytes
    return path


def prompt_ids(shape: LlamaShape, n: int, seed: int = 0) -> np.ndarray:
    """`n` uniform random token ids of the vocabulary (the configurations' prompts)."""
    return np.random.default_rng(seed + 1).integers(0, shape.vocab, n, dtype=np.uint32)


def _skip_value(buf: memoryview, pos: int, vtype: int) -> int:
    scalar = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}
    if vtype == GGUF_STRING:
        (n,) = struct.unpack_from("<Q", buf, pos)
        return pos + 8 + n
    if vtype == GGUF_ARRAY:
        etype, count = struct.unpack_from("<IQ", buf, pos)
        pos += 12
        if etype == GGUF_STRING:
            for _ in range(count):
                (n,) = struct.unpack_from("<Q", buf, pos)
                pos += 8 + n
            return pos
        return pos + count * scalar[etype]
    return pos + scalar[vtype]


def read_tensor(path, name: str) -> tuple[np.ndarray, int, tuple]:
    """(raw bytes, GGUF type, dims) of tensor `name` of a GGUF v3 file (the reader of
    ``src/gguf.c:359-610`` restated, for tests that need a model's tensors)."""
    data = pathlib.Path(path).read_bytes()
    buf = memoryview(data)
    assert data[:4] == b"GGUF"
    _, n_tensors, n_kv = struct.unpack_from("<IQQ", buf, 4)
    pos = 24
    for _ in range(n_kv):
        (n,) = struct.unpack_from("<Q", buf, pos)
        pos += 8 + n
        (vtype,) = struct.unpack_from("<I", buf, pos)
        pos = _skip_value(buf, pos + 4, vtype)
    found = None
    for _ in range(n_tensors):
        (n,) = struct.unpack_from("<Q", buf, pos)
        tname = bytes(buf[pos + 8:pos + 8 + n]).decode()
        pos += 8 + n
        (nd,) = struct.unpack_from("<I", buf, pos)
        dims = struct.unpack_from(f"<{nd}Q", buf, pos + 4)
        wtype, off = struct.unpack_from("<IQ", buf, pos + 4 + 8 * nd)
        pos += 4 + 8 * nd + 12
        if tname == name:
            found = (wtype, off, dims)
    assert found is not None, name
    wtype, off, dims = found
    base = (pos + ALIGN - 1) // ALIGN * ALIGN + off
    n_in = dims[0]
    rows = int(np.prod(dims[1:])) if len(dims) > 1 else 1
    nbytes = (synth.row_bytes(wtype, n_in) if wtype != TYPE_F32 else 4 * n_in) * rows
    return np.frombuffer(data, np.uint8, nbytes, base).reshape(rows, -1), wtype, dims

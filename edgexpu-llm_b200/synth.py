"""Seeded synthetic GGUF blocks following the recipes of the benchmark configurations.

* Q8_0 weight block (34 B): fp16 d ~ U(1e-4, 2e-3), 32 int8 qs ~ U{-127..127}.
* Q4_K super-block (144 B): fp16 d, dmin ~ U(1e-4, 1e-3); 12 scale bytes whose eight 6-bit
  (scale, min) pairs are ~ U{0..63}; 128 bytes of nibbles ~ U{0..15}.  The 6-bit fields of the
  packing (get_scale_min_k4, gguf_quant.c:212-220) are a bijection of the 96 scale bits, so
  uniform random scale bytes give uniform independent (scale, min) pairs.
* Q4_0 (18 B) / Q5_0 (22 B): fp16 d ~ U(1e-4, 2e-3) as for Q8_0; high bits and nibbles uniform.
* Q5_K (176 B): the Q4_K recipe, plus 32 bytes of uniform high bits.
* Q6_K (210 B): 128 + 64 bytes of uniform low/high quant bits, int8 scales ~ U{-128..127}, fp16
  d ~ U(1e-4, 1e-3).
  (The benchmark configurations name only Q8_0 and Q4_K; these recipes follow their value ranges.)
* Activations: fp32 ~ N(0, 1).

The numpy versions are used for parity tests; the torch versions generate the multi-GB
benchmark tensors directly in HBM.
"""

from __future__ import annotations

import numpy as np

Q8_0_BYTES, Q4_K_BYTES = 34, 144
TYPE_Q4_0, TYPE_Q5_0, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K = 2, 6, 8, 12, 13, 14
BLOCK = {TYPE_Q4_0: (32, 18), TYPE_Q5_0: (32, 22), TYPE_Q8_0: (32, 34), TYPE_Q4_K: (256, 144),
         TYPE_Q5_K: (256, 176), TYPE_Q6_K: (256, 210)}


def row_bytes(wtype: int, n: int) -> int:
    """Bytes of one packed row of n elements (edgexpu_gguf_row_bytes, gguf_quant.c:468-480)."""
    qk, bb = BLOCK[wtype]
    return n // qk * bb


def _fp16_bits(v: np.ndarray) -> np.ndarray:
    return v.astype(np.float16).view(np.uint8).reshape(v.shape + (2,))


def q8_0_weight(rng: np.random.Generator, n_out: int, n_in: int) -> np.ndarray:
    nb = n_in // 32
    blk = np.empty((n_out, nb, Q8_0_BYTES), np.uint8)
    blk[..., 0:2] = _fp16_bits(rng.uniform(1e-4, 2e-3, (n_out, nb)))
    blk[..., 2:] = rng.integers(-127, 128, (n_out, nb, 32), dtype=np.int8).view(np.uint8)
    return blk.reshape(n_out, nb * Q8_0_BYTES)


def q4_k_weight(rng: np.random.Generator, n_out: int, n_in: int) -> np.ndarray:
    nb = n_in // 256
    blk = rng.integers(0, 256, (n_out, nb, Q4_K_BYTES), dtype=np.uint8)
    blk[..., 0:2] = _fp16_bits(rng.uniform(1e-4, 1e-3, (n_out, nb)))
    blk[..., 2:4] = _fp16_bits(rng.uniform(1e-4, 1e-3, (n_out, nb)))
    return blk.reshape(n_out, nb * Q4_K_BYTES)


def _blocks(rng: np.random.Generator, wtype: int, n_out: int, n_in: int) -> np.ndarray:
    qk, bb = BLOCK[wtype]
    return rng.integers(0, 256, (n_out, n_in // qk, bb), dtype=np.uint8)


def q4_0_weight(rng: np.random.Generator, n_out: int, n_in: int) -> np.ndarray:
    blk = _blocks(rng, TYPE_Q4_0, n_out, n_in)
    blk[..., 0:2] = _fp16_bits(rng.uniform(1e-4, 2e-3, blk.shape[:2]))
    return blk.reshape(n_out, -1)


def q5_0_weight(rng: np.random.Generator, n_out: int, n_in: int) -> np.ndarray:
    blk = _blocks(rng, TYPE_Q5_0, n_out, n_in)
    blk[..., 0:2] = _fp16_bits(rng.uniform(1e-4, 2e-3, blk.shape[:2]))
    return blk.reshape(n_out, -1)


def q5_k_weight(rng: np.random.Generator, n_out: int, n_in: int) -> np.ndarray:
    blk = _blocks(rng, TYPE_Q5_K, n_out, n_in)
    blk[..., 0:2] = _fp16_bits(rng.uniform(1e-4, 1e-3, blk.shape[:2]))
    blk[..., 2:4] = _fp16_bits(rng.uniform(1e-4, 1e-3, blk.shape[:2]))
    return blk.reshape(n_out, -1)


def q6_k_weight(rng: np.random.Generator, n_out: int, n_in: int) -> np.ndarray:
    blk = _blocks(rng, TYPE_Q6_K, n_out, n_in)
    blk[..., 208:210] = _fp16_bits(rng.uniform(1e-4, 1e-3, blk.shape[:2]))
    return blk.reshape(n_out, -1)


_MAKERS = {TYPE_Q4_0: q4_0_weight, TYPE_Q5_0: q5_0_weight, TYPE_Q5_K: q5_k_weight, TYPE_Q6_K: q6_k_weight}


def weight(rng: np.random.Generator, wtype: int, n_out: int, n_in: int) -> np.ndarray:
    if wtype == TYPE_Q8_0:
        return q8_0_weight(rng, n_out, n_in)
    if wtype == TYPE_Q4_K:
        return q4_k_weight(rng, n_out, n_in)
    return _MAKERS[wtype](rng, n_out, n_in)


def activations(rng: np.random.Generator, m: int, n: int) -> np.ndarray:
    return rng.standard_normal((m, n)).astype(np.float32)


def torch_weight(wtype: int, n_out: int, n_in: int, generator, device, pad: int = 256):
    """Same recipe generated on the device; returns a flat uint8 tensor with `pad` spare bytes."""
    import torch

    qk, bb = BLOCK[wtype]
    nblk = n_out * (n_in // qk)
    flat = torch.empty(nblk * bb + pad, dtype=torch.uint8, device=device)
    flat[nblk * bb:] = 0
    blk = flat[: nblk * bb].view(nblk, bb)
    if wtype == TYPE_Q8_0:
        blk[:, 2:] = torch.randint(-127, 128, (nblk, 32), dtype=torch.int8, device=device,
                                   generator=generator).view(torch.uint8)
        d = torch.empty(nblk, dtype=torch.float32, device=device).uniform_(1e-4, 2e-3, generator=generator)
        blk[:, 0:2] = d.to(torch.float16).view(torch.uint8).view(nblk, 2)
    elif wtype == TYPE_Q4_K:
        blk[:, 4:] = torch.randint(0, 256, (nblk, bb - 4), dtype=torch.uint8, device=device, generator=generator)
        dd = torch.empty(nblk, 2, dtype=torch.float32, device=device).uniform_(1e-4, 1e-3, generator=generator)
        blk[:, 0:4] = dd.to(torch.float16).view(torch.uint8).view(nblk, 4)
    else:  # uniform bytes, then the fp16 fields of the numpy recipe above
        off, count, lo, hi = _FP16_FIELDS[wtype]
        blk[:] = torch.randint(0, 256, (nblk, bb), dtype=torch.uint8, device=device, generator=generator)
        dd = torch.empty(nblk, count, dtype=torch.float32, device=device).uniform_(lo, hi, generator=generator)
        blk[:, off:off + 2 * count] = dd.to(torch.float16).view(torch.uint8).view(nblk, 2 * count)
    return flat


# (byte offset, number of consecutive fp16 fields, uniform range) per block of the other types
_FP16_FIELDS = {TYPE_Q4_0: (0, 1, 1e-4, 2e-3), TYPE_Q5_0: (0, 1, 1e-4, 2e-3), TYPE_Q5_K: (0, 2, 1e-4, 1e-3),
                TYPE_Q6_K: (208, 1, 1e-4, 1e-3)}

"""Tensor-parallel sharding of the quantized matrix products (one process per GPU).

The reference is single-process (OpenMP over output rows only); this module adds the
multi-GPU layout of the configuration-4 decode:

* q/k/v/gate/up and the logits weight shard by OUTPUT ROWS: each rank holds rows
  [r*N/W, (r+1)*N/W) -- a contiguous byte range of the GGUF tensor -- sees the full activation,
  and produces its slice of the output; nothing is exchanged.
* o/down shard by INPUT COLUMNS at super-block (Q4_K: 256) or block (Q8_0: 32) granularity, so
  activation quantization never straddles ranks and stays bit-exact; each rank produces a partial
  fp32 output and the partials are summed with one all-reduce.
* the greedy token: each rank reduces its vocab rows to one 64-bit key (order-preserving score
  bits high, 0xFFFFFFFF - id low), and a MAX all-reduce over ranks gives the global choice with
  the reference's lowest-id tie rule (native.c:2380).  Keys are unsigned; collectives reduce
  signed int64, so the sign bit is flipped before and after the reduction.

The helpers work on numpy byte arrays (host GGUF data) and torch tensors (device buffers);
the collective calls go through torch.distributed (NCCL on GPUs, gloo in CPU tests).
"""

from __future__ import annotations

import numpy as np

BLOCK = {8: (32, 34), 12: (256, 144)}  # type -> (elements per block, bytes per block)
SIGN64 = -(2 ** 63)


def row_range(n_rows: int, world: int, rank: int) -> tuple[int, int]:
    if n_rows % world:
        raise ValueError(f"{n_rows} rows do not split evenly over {world} ranks")
    per = n_rows // world
    return rank * per, per


def shard_rows(w: np.ndarray, world: int, rank: int) -> np.ndarray:
    """Rows [r*N/W, (r+1)*N/W) of a [N][row_bytes] GGUF tensor (a contiguous byte range)."""
    r0, per = row_range(w.shape[0], world, rank)
    return np.ascontiguousarray(w[r0:r0 + per])


def col_range(n_in: int, wtype: int, world: int, rank: int) -> tuple[int, int]:
    qk, _ = BLOCK[wtype]
    nb = n_in // qk
    if nb % world:
        raise ValueError(f"{nb} blocks of {qk} do not split evenly over {world} ranks")
    per = nb // world
    return rank * per * qk, per * qk


def shard_cols(w: np.ndarray, n_in: int, wtype: int, world: int, rank: int) -> np.ndarray:
    """Input columns [c0, c0 + n_in/W) of every row, as a new [N][n_in/W row bytes] tensor."""
    qk, bb = BLOCK[wtype]
    c0, cn = col_range(n_in, wtype, world, rank)
    blk = w.reshape(w.shape[0], n_in // qk, bb)
    return np.ascontiguousarray(blk[:, c0 // qk:(c0 + cn) // qk]).reshape(w.shape[0], -1)


def to_signed_key(keys):
    """uint64 argmax keys (held in int64 storage) -> int64 values with the same order."""
    return keys ^ SIGN64 if not isinstance(keys, np.ndarray) else (keys.view(np.uint64) ^ np.uint64(1 << 63)).view(np.int64)


def from_signed_key(keys):
    return to_signed_key(keys)


def allreduce_partial_(t, group=None):
    """Sum of the column-sharded partial outputs (in place)."""
    import torch.distributed as dist

    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return t


def allreduce_argmax_(keys, group=None):
    """Global greedy key: MAX over ranks of the per-shard keys (int64 tensor, in place)."""
    import torch.distributed as dist

    keys.bitwise_xor_(SIGN64)
    dist.all_reduce(keys, op=dist.ReduceOp.MAX, group=group)
    keys.bitwise_xor_(SIGN64)
    return keys


def key_id(key: int) -> int:
    key &= (1 << 64) - 1
    return 0 if key == 0 else 0xFFFFFFFF - (key & 0xFFFFFFFF)


def make_key(score: float, token: int) -> int:
    """Host-side packing of one (score, id) pair, identical to the device's argmax_key()."""
    import math
    import struct

    if math.isnan(score) or score == -math.inf:
        return 0
    u = struct.unpack("<I", struct.pack("<f", score))[0]
    u = (~u & 0xFFFFFFFF) if (u & 0x80000000) else (u | 0x80000000)
    return (u << 32) | (0xFFFFFFFF - token)


def key_as_int64(key: int) -> int:
    """Unsigned 64-bit key -> the int64 with the same bits (for int64 tensor storage)."""
    return key - (1 << 64) if key >= (1 << 63) else key


def connect_p2p(cuda_lib, world: int, rank: int, group=None) -> None:
    """Set up the in-GEMV all-reduce of column-sharded projections: allocate this rank's exchange
    region, exchange the CUDA IPC handles over torch.distributed and open the peers' regions.
    After this, ``edgexpu_cuda_linear_quant_batch_tp_dev`` returns the summed output on every
    rank (no separate collective)."""
    import ctypes

    import torch.distributed as dist

    err = ctypes.create_string_buffer(512)
    handle = (ctypes.c_uint8 * 64)()
    if not cuda_lib.edgexpu_cuda_tp_init(world, rank, handle, err, 512):
        raise RuntimeError(err.value.decode())
    handles = [None] * world
    dist.all_gather_object(handles, bytes(handle), group=group)
    blob = b"".join(handles)
    if not cuda_lib.edgexpu_cuda_tp_connect(blob, err, 512):
        raise RuntimeError(err.value.decode())
    dist.barrier(group=group)

#!/usr/bin/env python3
"""Throughput of EdgeXPU-LLM's quantized matrix-product hot path on B200.

Metric: Q4_K / Q8_0 GEMV HBM GB/s -- algorithmic bytes (packed weights plus
activations in, quantized activations, outputs) per second, whole job.

Workloads (``--workload``):

* ``llama3_8b_q4k_decode`` (default): one step = every quantized matrix product of one
  Llama-3-8B-shaped decode token at batch ``--batch`` (default 1) -- 32 layers x {q 4096x4096,
  k 1024x4096, v 1024x4096, o 4096x4096, gate 14336x4096, up 14336x4096, down 4096x14336} plus
  the greedy logits over output.weight 128256x4096 with the fp32 hidden state (native.c:2355-2397).
  These are configuration 2's GEMV shapes in configuration 4's per-token arrangement:
  4,221,370,368 bytes of random-init Q4_K weights resident in HBM (far larger than L2, so no
  flush is needed between steps).  Each projection quantizes its activation (Q8_K) first.
  With N > 1 GPUs the path is tensor-parallel: q/k/v/gate/up and the logits shard by rows,
  o/down by input columns, followed by an NCCL fp32 all-reduce; the greedy token is an NCCL
  max-reduction of packed (score, id) keys.  Total work is fixed, so scaling is "strong".
* ``smollm2_q8_0_decode``: configuration 1's weight stream (30 layers of SmolLM2-135M-shaped
  Q8_0 projections + the tied 49152x576 Q8_0 logits), replicas only at N > 1.
* ``native_greedy``: configurations 1 and 4 end to end -- greedy decode tok/s through the reference's
  own layer loop (src/native.c) with the B200 path dropped in (integration/_build/
  libedgexpu_native_b200.so: every linear and the greedy logits on the GPU, weights resident in HBM,
  the rest of the loop on the host), on a seeded synthetic GGUF model (``--model smollm2``: SmolLM2-
  135M-shaped Q8_0, or ``llama3``: Llama-3-8B-shaped Q4_K, ``--layers`` to shorten it), ``--prompt``
  prompt ids, then ``--steps`` greedy tokens; the reference arm runs the unchanged reference runtime
  (oracle/_ref/libedgexpu_ref_runtime.so) on the same file.  The line also states whether the token
  ids of both are identical.  N > 1: independent replicas, one per GPU.
* ``device_decode``: configurations 1 and 4 decoded whole on the device (edgexpu_cuda_llama_*: every
  layer op, the KV cache and the greedy logits in HBM, token-identical to the reference): the
  prompt, then ``--warmup`` untimed and ``--steps`` timed greedy tokens, one public-API call per
  token (its id in, the next id out).  cpu_baseline: the unchanged reference runtime on a bounded
  sample of the same decode, whose ids are compared with the device's.  N > 1: replicas.
* ``llama3_8b_q4k_prefill``: configuration 3 -- one step = every quantized projection of the
  32 Llama-3-8B-shaped layers (``--layers`` fewer for small profiling cases) for a prompt of
  ``--batch`` tokens (default 2048), run by the tensor-core GEMM (tcgen05 kind::i8).  Metric:
  useful int8 TOPS (2 * M * N * K per projection); the tensor roofline is 2 x the measured bf16
  peak (B200's dense int8 rate is twice bf16).
* ``gemv``: one product per step, ``--shape n_out,n_in`` at ``--batch`` rows of weight type
  ``--wtype`` (configurations 0 and 2 name Q8_0 and Q4_K; Q4_0, Q5_0, Q5_K and Q6_K run on the
  same shapes), each step over the next of several weight copies that together exceed L2.  The
  line adds the kernel alone (activations pre-quantized) as the roofline.  No reference arm.

Arms: ``--impl ours`` (default) times the CUDA path; ``--impl reference`` times the reference's
own CPU implementation (oracle/_ref, compiled from the reference sources) on this host's cores.
"""

from __future__ import annotations

import argparse
import ctypes
import datetime
import importlib.util
import json
import os
import pathlib
import statistics
import subprocess
import sys
import time

ROOT = pathlib.Path(__file__).resolve().parent
PKG_DIR = ROOT / "edgexpu-llm_b200"
REF_LIB = ROOT / "oracle" / "_ref" / "libedgexpu_ref_avx2.so"
REF_DRIVER = ROOT / "oracle" / "_ref" / "libedgexpu_ref_driver.so"
PEAKS = ROOT / "MEASURED_PEAKS.json"
TRAFFIC = ROOT / "profiles" / "traffic.json"

TYPE_Q4_0, TYPE_Q5_0, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K = 2, 6, 8, 12, 13, 14
# GGUF weight types of the gemv workload: type id, (block elements, block bytes), arithmetic
WTYPES = {"q4_0": TYPE_Q4_0, "q5_0": TYPE_Q5_0, "q8_0": TYPE_Q8_0, "q4_k": TYPE_Q4_K, "q5_k": TYPE_Q5_K,
          "q6_k": TYPE_Q6_K}
BLOCKS = {TYPE_Q4_0: (32, 18), TYPE_Q5_0: (32, 22), TYPE_Q8_0: (32, 34), TYPE_Q4_K: (256, 144),
          TYPE_Q5_K: (256, 176), TYPE_Q6_K: (256, 210)}
DTYPES = {TYPE_Q4_0: "u4 x i8 -> i32 -> f32", TYPE_Q5_0: "u5 x i8 -> i32 -> f32", TYPE_Q8_0: "i8 x i8 -> i32 -> f32",
          TYPE_Q4_K: "u4/i8 x i8 -> i32 -> f32", TYPE_Q5_K: "u5/i8 x i8 -> i32 -> f32",
          TYPE_Q6_K: "u6/i8 x i8 -> i32 -> f32"}
GROUP_WITH_PREV = {"attn_k", "attn_v", "ffn_up"}  # read the same activations as the projection before
FALLBACK_HBM_GBS = 6650.0

WORKLOADS = {
    "llama3_8b_q4k_decode": {
        "type": TYPE_Q4_K, "layers": 32, "hidden": 4096,
        "proj": [("attn_q", 4096, 4096, "row"), ("attn_k", 1024, 4096, "row"), ("attn_v", 1024, 4096, "row"),
                 ("attn_output", 4096, 4096, "col"), ("ffn_gate", 14336, 4096, "row"),
                 ("ffn_up", 14336, 4096, "row"), ("ffn_down", 4096, 14336, "col")],
        "vocab": 128256, "tp": True,
    },
    "smollm2_q8_0_decode": {
        "type": TYPE_Q8_0, "layers": 30, "hidden": 576,
        "proj": [("attn_q", 576, 576, "row"), ("attn_k", 192, 576, "row"), ("attn_v", 192, 576, "row"),
                 ("attn_output", 576, 576, "row"), ("ffn_gate", 1536, 576, "row"), ("ffn_up", 1536, 576, "row"),
                 ("ffn_down", 576, 1536, "row")],
        "vocab": 49152, "tp": False,
    },
}


def load_pkg():
    name = "edgexpu_llm_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, PKG_DIR / "__init__.py", submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def row_bytes(t, n):
    qk, bb = BLOCKS[t]
    return n // qk * bb


def act_bytes(t, n):
    """Bytes of one quantized activation row: Q8_0 blocks for the 32-element types, Q8_K for the K-quants."""
    return n // 32 * 34 if BLOCKS[t][0] == 32 else n // 256 * 292


def linear_alg_bytes(t, n_out, n_in, m):
    """Algorithmic bytes of one linear: the weight once, plus per activation row its fp32 input
    (4K), its quantized form and its fp32 output (4N)."""
    return n_out * row_bytes(t, n_in) + m * (4 * n_in + act_bytes(t, n_in) + 4 * n_out)


# Library routing constants, for counting the kernels a call launches (the gpu_launches claim):
# rowstream_kernel.cuh (activation tile budget, rows per launch, prologue quantization), launch.h
# (tensor-core thresholds, tensor-parallel exchange slot), gemm_tc.cu (row tile, K split).
PROLOGUE_QUANT_MAX_M, ROWSTREAM_MAX_M, ACT_BUDGET = 2, 16, 96 * 1024
TC_MIN_M, TC_SMALL_MIN_M, TC_BM, TP_SLOT_BYTES = 64, 9, 128, 512 * 1024


def rowstream_max_m(t, k):
    """Activation rows one row-stream launch takes (rowstream_max_m)."""
    if BLOCKS[t][0] == 32:  # Q8_0 activations: 32 int8 + an fp32 scale per block
        per = 36 * (k // 32)
    else:  # Q8_K activations per 128-element unit: bytes, int32 and int16 sums, half a scale
        u = k // 128
        per = ((144 * u + (u // 2) * 4 + 15) & ~15) + 16 * u
    return min(ROWSTREAM_MAX_M, ACT_BUDGET // (per + 64))


def tc_split_ranges(m, n_rows, k, sm_count):
    """K ranges of a Q4_K tensor-core launch (tc_split): more than one adds the reduction kernel."""
    nb = k // 256
    bn = 16 if m < TC_MIN_M else 128
    base = -(-n_rows // TC_BM) * -(-m // bn)
    n_ks = 1
    if bn == 16 and base < 2 * sm_count:
        n_ks = max(1, min(-(-2 * sm_count // base), nb // 2))
    sb_per = -(-nb // n_ks)
    return -(-nb // sb_per)


def linear_launches(t, m, k, n_outs, relaxed, sm_count, tp_col=False):
    """Kernels of one linear call over the tensors `n_outs` sharing their activations, routed as the
    library routes it (run_linear_dev, edgexpu_cuda_linear_quant_multi_dev, the tensor-parallel
    linear): tensor-core GEMMs for relaxed-order Q4_K batches of 9+ and Q8_0 batches of 64+,
    otherwise the row-stream GEMV in chunks of rows, behind one quantize launch unless the GEMV
    quantizes in its own prologue."""
    if not tp_col and relaxed and t == TYPE_Q4_K and m >= TC_SMALL_MIN_M:
        return 1 + sum(1 + (tc_split_ranges(m, n, k, sm_count) > 1) for n in n_outs)
    if not tp_col and relaxed and t == TYPE_Q8_0 and m >= TC_MIN_M:
        return 2 * len(n_outs)
    chunk = rowstream_max_m(t, k)
    if tp_col:
        chunk = min(chunk, TP_SLOT_BYTES // 8 // n_outs[0], m)
        return -(-m // chunk) + (0 if chunk <= PROLOGUE_QUANT_MAX_M else 1)
    return -(-m // chunk) + (0 if m <= PROLOGUE_QUANT_MAX_M else 1)


def logits_alg_bytes(t, vocab, n_embd):
    extra = act_bytes(t, n_embd) if t == TYPE_Q8_0 else 0
    return vocab * row_bytes(t, n_embd) + 4 * n_embd + extra + 8


def shard_shapes(wl, world, rank):
    """Per-rank (label, n_out, n_in, kind) of one layer, plus the vocab rows [v0, v0+nv)."""
    out = []
    for label, n_out, n_in, kind in wl["proj"]:
        if world > 1 and wl["tp"]:
            if kind == "row":
                out.append((label, n_out // world, n_in, kind))
            else:
                out.append((label, n_out, n_in // world, kind))
        else:
            out.append((label, n_out, n_in, kind))
    nv = wl["vocab"] // world if (world > 1 and wl["tp"]) else wl["vocab"]
    return out, rank * nv if (world > 1 and wl["tp"]) else 0, nv


def step_bytes(wl, m):
    """Algorithmic bytes of one full (unsharded) step."""
    t = wl["type"]
    per_layer = sum(linear_alg_bytes(t, n_out, n_in, m) for _, n_out, n_in, _ in wl["proj"])
    return wl["layers"] * per_layer + m * logits_alg_bytes(t, wl["vocab"], wl["hidden"])


# ---- clocks -------------------------------------------------------------------------------------

CLOCK_FIELDS = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                "clocks_event_reasons.sw_power_cap")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    def __init__(self, index: int):
        self.cmd = ["nvidia-smi", f"--id={index}", f"--query-gpu={CLOCK_FIELDS}", "--format=csv,noheader,nounits",
                    "-lms", "100"]
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(self.cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self, t0: float, t1: float):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        self.proc.terminate()
        out = self.proc.communicate(timeout=10)[0]
        sms, maxes, reasons = [], [], set()
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                sm, mx = float(f[1]), float(f[2])
            except ValueError:
                continue
            if not (t0 <= ts <= t1):
                continue
            sms.append(sm)
            maxes.append(mx)
            for name, val in zip(REASONS, f[4:8]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": max(maxes) if maxes else None,
                "reasons": sorted(reasons), "samples": len(sms)}


# ---- distributed plumbing -----------------------------------------------------------------------


def traffic_per_launch(alg_bytes):
    """DRAM bytes per row-stream launch: the DRAM/algorithmic byte ratio that ncu measured on a
    capturable case (profiles/traffic.json) applied to this launch's algorithmic bytes."""
    try:
        rs = json.loads(TRAFFIC.read_text())["rowstream"]
        return int(round(alg_bytes * rs["dram_bytes_per_launch"] / rs["alg_bytes_per_launch"]))
    except (OSError, ValueError, KeyError):
        return None


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def peak_hbm():
    try:
        return float(json.loads(PEAKS.read_text())["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


# ---- the reference's CPU implementation (baseline arm) ------------------------------------------


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


class RefCPU:
    def __init__(self):
        if not (REF_LIB.exists() and REF_DRIVER.exists()):
            raise FileNotFoundError("oracle/_ref not built")
        # The reference's OpenMP loops run on every host core (torchrun exports OMP_NUM_THREADS=1;
        # the reference honours the variable instead of probing, cpu_kernel.c:53-57).  libgomp reads
        # it when it loads, i.e. at the CDLL below.
        os.environ["OMP_NUM_THREADS"] = str(host_threads())
        self.lib = ctypes.CDLL(str(REF_LIB))
        self.drv = ctypes.CDLL(str(REF_DRIVER))
        vp, i, u = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32
        self.lib.edgexpu_cpu_linear_quant_batch.argtypes = [vp, vp, vp, u, vp, i, i, i]
        self.lib.edgexpu_cpu_linear_quant_batch.restype = None
        self.drv.eoref_logits_greedy.argtypes = [vp, u, vp, i, i, vp, ctypes.POINTER(u), ctypes.POINTER(ctypes.c_float)]
        self.drv.eoref_logits_greedy.restype = i

    def linear(self, out, x, w, t, m, n_out, n_in):
        self.lib.edgexpu_cpu_linear_quant_batch(out.ctypes.data, x.ctypes.data, w.ctypes.data, t, None, m, n_out, n_in)

    def logits(self, w, t, h, n_embd, vocab):
        tok = ctypes.c_uint32()
        sc = ctypes.c_float()
        assert self.drv.eoref_logits_greedy(w.ctypes.data, t, h.ctypes.data, n_embd, vocab, None, ctypes.byref(tok),
                                            ctypes.byref(sc)) == 1
        return tok.value


def host_weight(rng, t, n_out, n_in):
    import numpy as np

    rb = row_bytes(t, n_in)
    w = np.frombuffer(rng.bytes(n_out * rb), np.uint8).reshape(n_out, rb).copy()
    if t == TYPE_Q8_0:
        blk = w.reshape(n_out, -1, 34)
        blk[..., 0:2] = rng.uniform(1e-4, 2e-3, blk.shape[:2]).astype(np.float16).view(np.uint8).reshape(blk.shape[:2] + (2,))
        qs = blk[..., 2:].view(np.int8)
        qs[qs == -128] = -127
    else:
        blk = w.reshape(n_out, -1, 144)
        blk[..., 0:4] = rng.uniform(1e-4, 1e-3, blk.shape[:2] + (2,)).astype(np.float16).view(np.uint8).reshape(blk.shape[:2] + (4,))
    return w


class CpuWorkload:
    """The workload (or a whole-layer sample of it) in host memory, run by the reference's CPU code."""

    def __init__(self, wl, m, layers, vocab_rows):
        import numpy as np

        self.ref = RefCPU()
        rng = np.random.default_rng(0)
        self.wl, self.m, self.t = wl, m, wl["type"]
        self.weights = [(host_weight(rng, self.t, n_out, n_in), n_out, n_in)
                        for _ in range(layers) for _, n_out, n_in, _k in wl["proj"]]
        self.vocab_rows = vocab_rows
        self.lw = host_weight(rng, self.t, vocab_rows, wl["hidden"])
        self.xs = {n_in: rng.standard_normal((m, n_in)).astype(np.float32) for _, _, n_in, _ in wl["proj"]}
        self.outs = {n_out: np.empty((m, n_out), np.float32) for _, n_out, _, _ in wl["proj"]}
        self.h = rng.standard_normal(wl["hidden"]).astype(np.float32)
        self.nbytes = (sum(linear_alg_bytes(self.t, n_out, n_in, m) for _, n_out, n_in in self.weights)
                       + m * logits_alg_bytes(self.t, vocab_rows, wl["hidden"]))
        self.threads = int(os.environ["OMP_NUM_THREADS"])

    def step(self):
        for w, n_out, n_in in self.weights:
            self.ref.linear(self.outs[n_out], self.xs[n_in], w, self.t, self.m, n_out, n_in)
        for _ in range(self.m):
            self.ref.logits(self.lw, self.t, self.h, self.wl["hidden"], self.vocab_rows)


def cpu_run(wl, m, layers, vocab_rows, min_seconds, min_reps):
    """Reference CPU GB/s on a sample, median over reps lasting >= min_seconds in total."""
    w = CpuWorkload(wl, m, layers, vocab_rows)
    w.step()  # the first call runs the reference's OpenMP thread probe (cpu_kernel.c:28-177)
    times = []
    t_start = time.perf_counter()
    while len(times) < min_reps or time.perf_counter() - t_start < min_seconds:
        t0 = time.perf_counter()
        w.step()
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    return w.nbytes / sec / 1e9, sec, w.nbytes, w.threads


def ref_sample_layers(wl, m, budget_bytes=5e9):
    """Whole layers (with their share of the logits rows) per reference step: the whole step when it is
    at most ~5 GB of algorithmic bytes (the decode workloads at batch 1), so that the reference arm times
    the same work as ours and a --steps K run still ends within minutes."""
    per_layer = step_bytes(wl, m) / wl["layers"]
    return max(1, min(wl["layers"], int(budget_bytes // per_layer)))


def run_reference(args, wl):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    m = args.batch
    layers = args.ref_layers or ref_sample_layers(wl, m)
    vocab_rows = wl["vocab"] * layers // wl["layers"]
    try:
        w = CpuWorkload(wl, m, layers, vocab_rows)
    except FileNotFoundError as e:
        print(json.dumps({"impl": "reference", "unavailable": f"reference CPU build missing: {e}"}))
        return
    for _ in range(max(1, args.warmup)):  # the first one also runs the reference's thread probe
        w.step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        w.step()
    sec = (time.perf_counter() - t0) / args.steps
    gbs = w.nbytes / sec / 1e9
    sample = (f"{'all' if layers == wl['layers'] else layers} of {wl['layers']} layers + {vocab_rows} of "
              f"{wl['vocab']} logits rows per step ({w.nbytes} algorithmic bytes), reference AVX2 build with OpenMP")
    line = {
        "metric": f"{'Q4_K' if wl['type'] == TYPE_Q4_K else 'Q8_0'} GEMV HBM GB/s ({args.workload}, batch {m})",
        "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True,
        "scaling": "strong" if wl["tp"] else "weak", "vs_baseline": None,
        "dtype": "u4/i8 x i8 -> i32 -> f32" if wl["type"] == TYPE_Q4_K else "i8 x i8 -> i32 -> f32",
        "data": "synthetic (seeded random-init GGUF blocks)", "impl": "reference",
        "config": {"workload": args.workload, "batch": m, "parallelism": f"cpu ({w.threads} threads)"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": w.threads, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---- our CUDA path ------------------------------------------------------------------------------


def set_float_order(cuda, args):
    order = 0 if args.float_order == "x86" else 1  # EDGEXPU_CUDA_ORDER_X86 / _RELAXED
    if not cuda.edgexpu_cuda_set_float_order(order):
        raise RuntimeError(cuda.edgexpu_cuda_last_error().decode())


def run_ours(args, wl):
    import numpy as np
    import torch
    import torch.distributed as dist

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    pkg = load_pkg()
    from edgexpu_llm_b200 import synth

    cuda = pkg.load_cuda()
    host = pkg.load_host()
    pkg.init(local)
    set_float_order(cuda, args)
    dev = torch.device("cuda", local)
    t = wl["type"]
    m = args.batch
    tp = world > 1 and wl["tp"]
    shapes, v0, nv = shard_shapes(wl, world, rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000 + rank)

    # Weights: generated in HBM with the seeded recipe and registered with the library.
    layers = []
    for _ in range(wl["layers"]):
        lay = []
        for label, n_out, n_in, kind in shapes:
            buf = synth.torch_weight(t, n_out, n_in, gen, dev)
            h = pkg.register_weight(buf, t, n_out, n_in)
            lay.append((label, n_out, n_in, kind, buf, h))
        layers.append(lay)
    # Launch groups of one layer: projections that read the same activations go in one launch
    # (q|k|v and gate|up); o and down each follow their own input.
    groups = []
    for i, (label, n_out, n_in, kind) in enumerate(shapes):
        if groups and label in GROUP_WITH_PREV and shapes[groups[-1][-1]][3] == "row" and kind == "row":
            groups[-1].append(i)
        else:
            groups.append([i])
    P = ctypes.c_void_p * 4
    I4 = ctypes.c_int * 4
    group_args = []  # per layer, per group: ctypes arrays for the multi-tensor call
    for lay in layers:
        ga = []
        for grp in groups:
            ga.append((len(grp), P(), P(*[lay[i][5] for i in grp]), I4(*[lay[i][1] for i in grp]), grp))
        group_args.append(ga)
    lbuf = synth.torch_weight(t, nv, wl["hidden"], gen, dev)
    lh = pkg.register_weight(lbuf, t, nv, wl["hidden"])

    # Activations / outputs (fixed random inputs; in the model these come from the host layer ops).
    ins = {}
    for _, n_out, n_in, _k in shapes:
        if n_in not in ins:
            ins[n_in] = torch.randn((m, n_in), generator=gen, device=dev, dtype=torch.float32)
    outs = {label: torch.empty((m, n_out), device=dev, dtype=torch.float32) for label, n_out, _, _ in shapes}
    for ga in group_args:
        for n_t, out_arr, _w, _n, grp in ga:
            for j, i in enumerate(grp):
                out_arr[j] = outs[shapes[i][0]].data_ptr()
    hidden = torch.randn(wl["hidden"], generator=gen, device=dev, dtype=torch.float32)
    keys = torch.zeros(max(1, m), device=dev, dtype=torch.int64)
    sign = torch.tensor(-(2 ** 63), device=dev, dtype=torch.int64)
    buf = ctypes.create_string_buffer(512)
    for n_in in ins:
        assert cuda.edgexpu_cuda_reserve(m, n_in, buf, 512), buf.value
    p2p = tp and args.collective == "p2p"
    if p2p:
        from edgexpu_llm_b200 import tp as tpmod

        tpmod.connect_p2p(cuda, world, rank)

    def enqueue_gemvs(st, collectives):
        for lay, ga in zip(layers, group_args):
            for n_t, out_arr, w_arr, n_arr, grp in ga:
                label, n_out, n_in, kind = shapes[grp[0]]
                if n_t == 1 and p2p and kind == "col":  # GEMV with its all-reduce over NVLink, one launch
                    ok = cuda.edgexpu_cuda_linear_quant_batch_tp_dev(out_arr[0], ins[n_in].data_ptr(), w_arr[0], t, None,
                                                                     m, n_out, n_in, st)
                elif n_t == 1:
                    ok = cuda.edgexpu_cuda_linear_quant_batch_dev(out_arr[0], ins[n_in].data_ptr(), w_arr[0], t, None, m,
                                                                  n_out, n_in, st)
                else:
                    ok = cuda.edgexpu_cuda_linear_quant_multi_dev(n_t, out_arr, w_arr, n_arr, None, t,
                                                                  ins[n_in].data_ptr(), m, n_in, st)
                if not ok:
                    raise RuntimeError(cuda.edgexpu_cuda_last_error().decode())
                if collectives and tp and kind == "col" and not p2p:
                    dist.all_reduce(outs[label])

    def enqueue_step():
        st = torch.cuda.current_stream().cuda_stream
        enqueue_gemvs(st, True)
        for i in range(m):
            if not cuda.edgexpu_cuda_logits_argmax_dev(lh, t, hidden.data_ptr(), wl["hidden"], nv, None, v0,
                                                       keys[i:].data_ptr(), st):
                raise RuntimeError(cuda.edgexpu_cuda_last_error().decode())
        if tp:
            keys.bitwise_xor_(sign)  # uint64 order -> int64 order for the max-reduction
            dist.all_reduce(keys, op=dist.ReduceOp.MAX)
            keys.bitwise_xor_(sign)

    # Eager warm-up (sizes scratch, sets kernel attributes), then capture one step in a graph.
    enqueue_step()
    torch.cuda.synchronize()
    graph = None
    cap_stream = torch.cuda.Stream(device=dev)
    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=cap_stream):
            enqueue_step()
        torch.cuda.synchronize()
    except Exception as e:  # noqa: BLE001 -- fall back to eager launches, reported in config
        graph = None
        print(f"[bench] graph capture failed ({e}); timing eager launches", file=sys.stderr)
        torch.cuda.synchronize()

    def one_step():
        if graph is not None:
            graph.replay()
        else:
            enqueue_step()

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_load0 = time.time()
    ev0.record()
    for _ in range(args.steps):
        one_step()
    ev1.record()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        dist.barrier()
    # Keep the same load running (untimed) until clocks have been sampled for >= 2 s.
    extended = False
    while time.time() - t_load0 < 2.0:
        extended = True
        for _ in range(max(1, args.steps)):
            one_step()
        torch.cuda.synchronize()
    t_load1 = time.time()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop(t_load0, t_load1)
    clocks["window"] = ("timed region extended by identical untimed steps to 2 s of sampling"
                        if extended else "timed region")

    ms_t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    total_bytes = step_bytes(wl, m) * (1 if tp else world)
    value_gbs = total_bytes * args.steps / (ms_max / 1e3) / 1e9

    # Roofline of the dominant kernel (the row-stream GEMV): the step's GEMV launches alone (no
    # collectives, no logits) captured in one graph and timed with events on its stream.
    g_k = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_k, stream=cap_stream):
        enqueue_gemvs(torch.cuda.current_stream().cuda_stream, False)
    for _ in range(3):
        g_k.replay()
    torch.cuda.synchronize()
    ka, kb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k_reps = max(3, min(args.steps, 20))
    ka.record()
    for _ in range(k_reps):
        g_k.replay()
    kb.record()
    torch.cuda.synchronize()
    kern_s = ka.elapsed_time(kb) / 1e3 / k_reps
    kern_launches = wl["layers"] * len(groups)
    kern_bytes = wl["layers"] * sum(linear_alg_bytes(t, n_out, n_in, m) for _, n_out, n_in, _k in shapes)
    achieved = kern_bytes / kern_s / 1e9
    del g_k
    peak, peak_kind = peak_hbm()
    traffic = traffic_per_launch(kern_bytes / kern_launches)

    def time_order(order):
        """The same device step and kernel-only graph timed in another float order (untimed otherwise)."""
        assert cuda.edgexpu_cuda_set_float_order(order) == 1
        g_s, g_g = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_s, stream=cap_stream):
            enqueue_step()
        with torch.cuda.graph(g_g, stream=cap_stream):
            enqueue_gemvs(torch.cuda.current_stream().cuda_stream, False)
        for _ in range(max(3, args.warmup)):
            g_s.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            g_s.replay()
        e1.record()
        torch.cuda.synchronize()
        t_ms = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t_ms, op=dist.ReduceOp.MAX)
        e0.record()
        for _ in range(k_reps):
            g_g.replay()
        e1.record()
        torch.cuda.synchronize()
        k_s = e0.elapsed_time(e1) / 1e3 / k_reps
        del g_s, g_g
        set_float_order(cuda, args)
        step_ms = float(t_ms.item()) / args.steps
        return {"value": round(total_bytes / (step_ms / 1e3) / 1e9, 2), "ms_per_step": round(step_ms, 4),
                "roofline_frac": round(kern_bytes / k_s / 1e9 / peak, 4), "avg_launch_us": round(k_s / kern_launches * 1e6, 3)}

    other_order = None
    if args.compare_orders:
        other = "x86" if args.float_order == "relaxed" else "relaxed"
        other_order = {"float_order": other, **time_order(0 if other == "x86" else 1)}

    # Tensor-parallel check (untimed): the all-reduce the step performs for a column-sharded projection
    # must give every rank the same bits and equal the sum of the ranks' own partial products (each from
    # the single-GPU GEMV, which the parity tests pin to the reference) within 1e-5 of sum |w x|.
    tp_check = None
    if tp:
        label, n_out, n_in, _k = next(sh for sh in shapes if sh[3] == "col")
        i = next(k for k, sh in enumerate(shapes) if sh[0] == label)
        h_c = layers[0][i][5]
        st = torch.cuda.current_stream().cuda_stream
        got = torch.empty((m, n_out), device=dev, dtype=torch.float32)
        part = torch.empty((m, n_out), device=dev, dtype=torch.float32)
        if p2p:
            ok = cuda.edgexpu_cuda_linear_quant_batch_tp_dev(got.data_ptr(), ins[n_in].data_ptr(), h_c, t, None, m, n_out,
                                                             n_in, st)
        else:
            ok = cuda.edgexpu_cuda_linear_quant_batch_dev(got.data_ptr(), ins[n_in].data_ptr(), h_c, t, None, m, n_out,
                                                          n_in, st)
        ok = ok and cuda.edgexpu_cuda_linear_quant_batch_dev(part.data_ptr(), ins[n_in].data_ptr(), h_c, t, None, m,
                                                             n_out, n_in, st)
        if not ok:
            raise RuntimeError(cuda.edgexpu_cuda_last_error().decode())
        if not cuda.edgexpu_cuda_stream_sync(st, buf, 512):
            raise RuntimeError(buf.value.decode())
        if not p2p:
            dist.all_reduce(got)
        parts = [torch.empty_like(part) for _ in range(world)]
        gots = [torch.empty_like(got) for _ in range(world)]
        dist.all_gather(parts, part)
        dist.all_gather(gots, got)
        want = sum(pp.double() for pp in parts)
        bound = sum(pp.double().abs() for pp in parts)
        rel = float(((got.double() - want).abs() / (bound + 1e-30)).max())
        same = all(torch.equal(g.view(torch.int32), got.view(torch.int32)) for g in gots)
        keys_all = [torch.empty_like(keys) for _ in range(world)]
        dist.all_gather(keys_all, keys)
        keys_same = all(torch.equal(k, keys) for k in keys_all)
        tp_check = {"projection": label, "identical_on_all_ranks": bool(same), "greedy_key_identical": bool(keys_same),
                    "max_err_vs_sum_of_partials": rel, "ok": bool(same and keys_same and rel <= 1e-5)}
        if not tp_check["ok"]:
            raise RuntimeError(f"tensor-parallel check failed: {tp_check}")

    # End to end through the reference-named host shim: host buffers, H2D/D2H inside the timed region.
    hx = {n_in: ins[n_in].cpu().numpy() for n_in in ins}
    hout = {label: np.empty((m, n_out), np.float32) for label, n_out, _, _ in shapes}
    hh = hidden.cpu().numpy()
    tok = ctypes.c_uint32()
    h2d = d2h = 0
    for _, n_out, n_in, kind in shapes:
        h2d += 4 * m * n_in * wl["layers"]
        d2h += (4 * m * n_out + 4) * wl["layers"]
        if tp and kind == "col":
            h2d += 4 * m * n_out * wl["layers"]
            d2h += 4 * m * n_out * wl["layers"]
    h2d += 4 * wl["hidden"] * m
    d2h += 12 * m
    red = {label: torch.empty((m, n_out), device=dev, dtype=torch.float32) for label, n_out, _, k in shapes if k == "col"}

    def e2e_step():
        for lay in layers:
            for label, n_out, n_in, kind, _b, h in lay:
                o = hout[label]
                host.edgexpu_cpu_linear_quant_batch(o.ctypes.data, hx[n_in].ctypes.data, h, t, None, m, n_out, n_in)
                if tp and kind == "col":
                    r = red[label]
                    r.copy_(torch.from_numpy(o))
                    dist.all_reduce(r)
                    o[...] = r.cpu().numpy()
        for _ in range(m):
            ok = host.edgexpu_b200_logits_greedy(lh, t, hh.ctypes.data, wl["hidden"], nv, None, ctypes.byref(tok),
                                                 buf, 512)
            if not ok:
                raise RuntimeError(buf.value.decode())
        err = host.edgexpu_b200_last_error()
        if err:
            raise RuntimeError(err.decode())

    host.edgexpu_b200_clear_error()
    for _ in range(max(1, min(args.warmup, 3))):
        e2e_step()
    if world > 1:
        dist.barrier()
    e_steps = max(1, min(args.steps, 10))
    t0 = time.perf_counter()
    for _ in range(e_steps):
        e2e_step()
    e2e_s = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
    e2e_gbs = total_bytes * e_steps / float(e2e_s.item()) / 1e9

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cl = max(1, wl["layers"] // 8)
            gbs_cpu, sec_cpu, nb_cpu, threads = cpu_run(wl, m, cl, wl["vocab"] * cl // wl["layers"], 10.0, 3)
            cpu_baseline = {"value": round(gbs_cpu, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
                            "sample": f"{cl} of {wl['layers']} layers + {wl['vocab'] * cl // wl['layers']} logits rows "
                                      f"({nb_cpu} bytes) per rep, median of reps over >= 10 s, reference AVX2 build "
                                      f"(oracle/_ref) with OpenMP"}
        except FileNotFoundError as e:
            cpu_baseline = {"value": None, "unit": "GB/s", "cores": 0, "kind": "reference", "sample": f"unavailable: {e}"}

    # the kernels of every group's call as the library routes it, plus one logits kernel per token
    relaxed = args.float_order == "relaxed"
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    tc_small = t == TYPE_Q4_K and relaxed and 9 <= m < 64
    launches_per_step = wl["layers"] * sum(
        linear_launches(t, m, shapes[grp[0]][2], [shapes[i][1] for i in grp], relaxed, sms,
                        tp_col=p2p and len(grp) == 1 and shapes[grp[0]][3] == "col") for grp in groups) + m
    line = {
        "metric": f"{'Q4_K' if t == TYPE_Q4_K else 'Q8_0'} GEMV HBM GB/s ({args.workload}, batch {m})",
        "value": round(value_gbs, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
        "scaling": "strong" if tp else "weak", "vs_baseline": None,
        "dtype": "u4/i8 x i8 -> i32 -> f32" if t == TYPE_Q4_K else "i8 x i8 -> i32 -> f32",
        "data": "synthetic (seeded random-init GGUF blocks generated in HBM)",
        "config": {"workload": args.workload, "batch": m,
                   "parallelism": f"tp{world}" if tp else (f"replicas{world}" if world > 1 else "single"),
                   "bytes_per_step": total_bytes, "l2": "inputs larger than L2 (weights streamed once per step)",
                   "graph": graph is not None, "tokens_per_s_gemv_only": round(args.steps / (ms_max / 1e3) * m, 2),
                   "float_order": args.float_order, "other_float_order": other_order, "tp_check": tp_check,
                   "collective": ("o/down all-reduce inside the GEMV over NVLink (P2P stores), argmax via NCCL"
                                  if p2p else ("NCCL all-reduce after o/down, NCCL argmax" if tp else "none"))},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "kernel": ("gemm_q4k_tc, 16-token tiles with split K (+ activation packing, split reduction)"
                                if tc_small else "rowstream GEMV (Q4_K x Q8_K)" if t == TYPE_Q4_K
                                else "rowstream GEMV (Q8_0 x Q8_0)"),
                     "launches": kern_launches, "avg_launch_us": round(kern_s / kern_launches * 1e6, 3),
                     "peak_source": f"{peak_kind} hbm_gbs"},
        "cpu_baseline": cpu_baseline,
        "e2e": {"value": round(e2e_gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "edgexpu_cpu_linear_quant_batch + edgexpu_b200_logits_greedy (host buffers)"},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    graph = None
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()  # no rank unmaps its exchange region while a peer may still write to it
    pkg.shutdown()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_gemv(args):
    """Configurations 0 and 2: one GEMV per step (activation quantization included) over the
    next of `copies` weight copies, so the weights streamed per step always come from HBM."""
    import math

    import numpy as np
    import torch

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    pkg = load_pkg()
    from edgexpu_llm_b200 import synth

    cuda, host = pkg.load_cuda(), pkg.load_host()
    pkg.init(local)
    set_float_order(cuda, args)
    dev = torch.device("cuda", local)
    t = WTYPES[args.wtype]
    n_out, n_in = (int(v) for v in args.shape.split(","))
    m = args.batch
    wb = n_out * row_bytes(t, n_in)
    copies = max(2, math.ceil(args.rotate_bytes / wb))
    gen = torch.Generator(device=dev)
    gen.manual_seed(7 + rank)
    wbuf = synth.torch_weight(t, n_out * copies, n_in, gen, dev)
    h0 = pkg.register_weight(wbuf, t, n_out * copies, n_in)
    x = torch.randn((m, n_in), generator=gen, device=dev, dtype=torch.float32)
    out = torch.empty((m, n_out), device=dev, dtype=torch.float32)
    buf = ctypes.create_string_buffer(512)
    assert cuda.edgexpu_cuda_reserve(m, n_in, buf, 512), buf.value

    def enqueue(k0, k):
        st = torch.cuda.current_stream().cuda_stream
        for i in range(k0, k0 + k):
            if not cuda.edgexpu_cuda_linear_quant_batch_dev(out.data_ptr(), x.data_ptr(), h0 + (i % copies) * wb, t,
                                                            None, m, n_out, n_in, st):
                raise RuntimeError(cuda.edgexpu_cuda_last_error().decode())

    enqueue(0, 1)
    torch.cuda.synchronize()
    cap = torch.cuda.Stream(device=dev)
    g_warm, g_timed = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_warm, stream=cap):
        enqueue(0, max(1, args.warmup))
    with torch.cuda.graph(g_timed, stream=cap):
        enqueue(max(1, args.warmup), args.steps)
    g_warm.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_load0 = time.time()
    ev0.record()
    g_timed.replay()
    ev1.record()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    extended = False
    while time.time() - t_load0 < 2.0:
        extended = True
        g_timed.replay()
        torch.cuda.synchronize()
    clocks = sampler.stop(t_load0, time.time())
    clocks["window"] = ("timed region extended by identical untimed steps to 2 s of sampling"
                        if extended else "timed region")
    nbytes = linear_alg_bytes(t, n_out, n_in, m)
    value = nbytes * args.steps / (ms / 1e3) / 1e9

    # GEMV kernel alone (activations pre-quantized): a graph of launches over the weight copies,
    # timed with events on its stream (single event pairs are too coarse for microsecond kernels).
    st = torch.cuda.current_stream().cuda_stream
    xq = torch.empty(m * act_bytes(t, n_in) + 64, dtype=torch.uint8, device=dev)
    assert cuda.edgexpu_cuda_quantize_dev(t, x.data_ptr(), m, n_in, xq.data_ptr(), st)
    torch.cuda.synchronize()
    n_k = max(args.steps, copies)
    g_k = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_k, stream=cap):
        sk = torch.cuda.current_stream().cuda_stream
        for i in range(n_k):
            assert cuda.edgexpu_cuda_dot_quant_q8_dev(out.data_ptr(), xq.data_ptr(), h0 + (i % copies) * wb, t, None, m,
                                                      n_out, n_in, sk)
    g_k.replay()
    torch.cuda.synchronize()
    ka, kb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ka.record()
    g_k.replay()
    kb.record()
    torch.cuda.synchronize()
    kern_ms = ka.elapsed_time(kb) / n_k
    del g_k
    kbytes = wb + m * (act_bytes(t, n_in) + 4 * n_out)
    achieved = kbytes / (kern_ms / 1e3) / 1e9
    peak, peak_kind = peak_hbm()

    # End to end through the reference-named host shim.
    hx = x.cpu().numpy()
    hout = np.empty((m, n_out), np.float32)
    host.edgexpu_b200_clear_error()

    def e2e(i):
        host.edgexpu_cpu_linear_quant_batch(hout.ctypes.data, hx.ctypes.data, h0 + (i % copies) * wb, t, None, m, n_out,
                                            n_in)

    for i in range(3):
        e2e(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        e2e(i)
    e2e_s = time.perf_counter() - t0
    err = host.edgexpu_b200_last_error()
    if err:
        raise RuntimeError(err.decode())
    line = {
        "metric": f"{args.wtype.upper()} GEMV HBM GB/s ({n_out}x{n_in}, batch {m})",
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": DTYPES[t],
        "data": "synthetic (seeded random-init GGUF blocks generated in HBM)",
        "config": {"workload": "gemv", "type": args.wtype, "n_out": n_out, "n_in": n_in, "batch": m,
                   "weight_copies": copies, "l2": f"rotating {copies} weight copies ({copies * wb} bytes) > L2",
                   "parallelism": "single", "float_order": args.float_order},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic_per_launch(nbytes), "kernel_us": round(kern_ms * 1e3, 3),
                     "peak_source": f"{peak_kind} hbm_gbs"},
        "cpu_baseline": None,
        "e2e": {"value": round(nbytes * args.steps / e2e_s / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": 4 * m * n_in, "d2h_bytes_per_step": 4 * m * n_out + 4,
                "path": "edgexpu_cpu_linear_quant_batch (host buffers)"},
        "gpu_launches": args.steps * linear_launches(t, m, n_in, [n_out], args.float_order == "relaxed",
                                                     torch.cuda.get_device_properties(dev).multi_processor_count),
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    del g_warm, g_timed
    torch.cuda.synchronize()
    pkg.shutdown()


# ---- configuration 3: prefill GEMM ------------------------------------------------------------

PREFILL = WORKLOADS["llama3_8b_q4k_decode"]
TENSOR_I8_SPEC_TOPS = 4500.0


def prefill_ops(m, layers):
    return 2.0 * m * layers * sum(n_out * n_in for _, n_out, n_in, _k in PREFILL["proj"])


def peak_i8():
    try:
        pk = json.loads(PEAKS.read_text())
        if pk.get("bf16_tflops"):
            return 2.0 * float(pk["bf16_tflops"]), "2 x measured bf16_tflops (MEASURED_PEAKS.json)"
    except (OSError, ValueError):
        pass
    return 2.0 * 1590.0, "2 x fallback bf16 1590 TFLOP/s"


class CpuPrefill:
    """One layer's seven projections at m tokens through the reference's CPU linear."""

    def __init__(self, m):
        import numpy as np

        self.ref = RefCPU()
        rng = np.random.default_rng(0)
        self.m = m
        self.ws = [(host_weight(rng, TYPE_Q4_K, n_out, n_in), n_out, n_in) for _, n_out, n_in, _k in PREFILL["proj"]]
        self.xs = {n_in: rng.standard_normal((m, n_in)).astype(np.float32) for _, _, n_in in self.ws}
        self.outs = {n_out: np.empty((m, n_out), np.float32) for _, n_out, _ in self.ws}
        self.ops = prefill_ops(m, 1)
        self.threads = int(os.environ["OMP_NUM_THREADS"])

    def step(self):
        for w, n_out, n_in in self.ws:
            self.ref.linear(self.outs[n_out], self.xs[n_in], w, TYPE_Q4_K, self.m, n_out, n_in)


def cpu_prefill(m, min_seconds, min_reps):
    """Reference CPU TOPS on the one-layer sample, median over reps lasting >= min_seconds."""
    w = CpuPrefill(m)
    w.step()  # the first call runs the reference's OpenMP thread probe (cpu_kernel.c:28-177)
    times = []
    t_start = time.perf_counter()
    while len(times) < min_reps or time.perf_counter() - t_start < min_seconds:
        t0 = time.perf_counter()
        w.step()
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    return w.ops / sec / 1e12, sec, w.threads


def run_prefill_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    m = min(args.batch, 64)
    try:
        w = CpuPrefill(m)
    except FileNotFoundError as e:
        print(json.dumps({"impl": "reference", "unavailable": f"reference CPU build missing: {e}"}))
        return
    for _ in range(max(1, args.warmup)):
        w.step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        w.step()
    sec = (time.perf_counter() - t0) / args.steps
    tops = w.ops / sec / 1e12
    sample = (f"one layer's seven projections at {m} of {args.batch} prompt tokens per step "
              f"({w.ops:.3e} useful ops), reference AVX2 build with OpenMP")
    print(json.dumps({
        "metric": f"Q4_K prefill GEMM useful int8 TOPS (llama3_8b_q4k_prefill, M {args.batch})",
        "value": round(tops, 4), "unit": "TOPS", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "u4/i8 x i8 -> i32 -> f32", "data": "synthetic (seeded random-init GGUF blocks)",
        "impl": "reference", "config": {"workload": "llama3_8b_q4k_prefill", "batch": args.batch,
                                        "parallelism": f"cpu ({w.threads} threads)"},
        "cpu_baseline": {"value": round(tops, 4), "unit": "TOPS", "cores": w.threads, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": round(tops, 4), "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_prefill(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    pkg = load_pkg()
    from edgexpu_llm_b200 import synth

    WT = TYPE_Q8_0 if args.wtype == "q8_0" else TYPE_Q4_K
    tname = "Q8_0" if WT == TYPE_Q8_0 else "Q4_K"

    cuda = pkg.load_cuda()
    host = pkg.load_host()
    pkg.init(local)
    # This workload is the tensor-core GEMM, which serves float outputs in the relaxed order (the
    # x86 order routes prefill batches to the GEMV).
    args.float_order = "relaxed"
    set_float_order(cuda, args)
    dev = torch.device("cuda", local)
    m = args.batch
    shapes = PREFILL["proj"]
    L = args.layers or PREFILL["layers"]
    gen = torch.Generator(device=dev)
    gen.manual_seed(3000 + rank)
    layers = []
    for _ in range(L):
        lay = []
        for label, n_out, n_in, _k in shapes:
            buf = synth.torch_weight(WT, n_out, n_in, gen, dev)
            lay.append((label, n_out, n_in, buf, pkg.register_weight(buf, WT, n_out, n_in)))
        layers.append(lay)
    ins = {n_in: torch.randn((m, n_in), generator=gen, device=dev) for _, _, n_in, _k in shapes}
    outs = {label: torch.empty((m, n_out), device=dev) for label, n_out, _, _k in shapes}
    groups = [[0, 1, 2], [3], [4, 5], [6]]  # q|k|v and gate|up share their activations
    P = ctypes.c_void_p * 4
    I4 = ctypes.c_int * 4
    calls = []
    for lay in layers:
        for grp in groups:
            calls.append((len(grp), P(*[outs[lay[i][0]].data_ptr() for i in grp]), P(*[lay[i][4] for i in grp]),
                          I4(*[lay[i][1] for i in grp]), lay[grp[0]][2]))
    buf = ctypes.create_string_buffer(512)
    for n_in in ins:
        assert cuda.edgexpu_cuda_reserve(m, n_in, buf, 512), buf.value

    def enqueue_step():
        st = torch.cuda.current_stream().cuda_stream
        for n_t, o_arr, w_arr, n_arr, n_in in calls:
            if n_t == 1:
                ok = cuda.edgexpu_cuda_linear_quant_batch_dev(o_arr[0], ins[n_in].data_ptr(), w_arr[0], WT, None,
                                                              m, n_arr[0], n_in, st)
            else:
                ok = cuda.edgexpu_cuda_linear_quant_multi_dev(n_t, o_arr, w_arr, n_arr, None, WT,
                                                              ins[n_in].data_ptr(), m, n_in, st)
            if not ok:
                raise RuntimeError(cuda.edgexpu_cuda_last_error().decode())

    def check_status():
        if not cuda.edgexpu_cuda_stream_sync(torch.cuda.current_stream().cuda_stream, buf, 512):
            raise RuntimeError(buf.value.decode())

    enqueue_step()
    torch.cuda.synchronize()
    check_status()
    graph = torch.cuda.CUDAGraph()
    cap_stream = torch.cuda.Stream(device=dev)
    with torch.cuda.graph(graph, stream=cap_stream):
        enqueue_step()
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_load0 = time.time()
    ev0.record()
    for _ in range(args.steps):
        graph.replay()
    ev1.record()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    extended = False
    while time.time() - t_load0 < 2.0:
        extended = True
        graph.replay()
        torch.cuda.synchronize()
    t_load1 = time.time()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop(t_load0, t_load1)
    clocks["window"] = ("timed region extended by identical untimed steps to 2 s of sampling"
                        if extended else "timed region")
    check_status()
    ms_t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    ops = prefill_ops(m, L)
    tops = ops * world * args.steps / (ms_max / 1e3) / 1e12

    # Per projection: the GEMM (with its activation packing) of one layer's shape, replayed from a CUDA
    # graph of 5 calls (no host launch cost in the figure), events on the stream.
    per_proj = {}
    for i, (label, n_out, n_in, _k) in enumerate(shapes):
        o = outs[label]
        reps = 5
        g_p = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_p, stream=cap_stream):
            st_c = torch.cuda.current_stream().cuda_stream
            for j in range(reps):
                if not cuda.edgexpu_cuda_linear_quant_batch_dev(o.data_ptr(), ins[n_in].data_ptr(), layers[j % L][i][4],
                                                                WT, None, m, n_out, n_in, st_c):
                    raise RuntimeError(cuda.edgexpu_cuda_last_error().decode())
        for _ in range(2):
            g_p.replay()
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        g_p.replay()
        a1.record()
        torch.cuda.synchronize()
        del g_p
        us = a0.elapsed_time(a1) / reps * 1e3
        per_proj[label] = {"us": round(us, 1), "tops": round(2.0 * m * n_out * n_in / (us * 1e-6) / 1e12, 1)}
    check_status()
    peak, peak_src = peak_i8()

    # End to end through the reference-named host shim (host buffers, copies inside the timed region).
    hx = {n_in: ins[n_in].cpu().numpy() for n_in in ins}
    hout = {label: np.empty((m, n_out), np.float32) for label, n_out, _, _k in shapes}
    h2d = sum(4 * m * n_in for _, _, n_in, _k in shapes) * L
    d2h = sum(4 * m * n_out for _, n_out, _, _k in shapes) * L

    def e2e_step():
        for lay in layers:
            for label, n_out, n_in, _b, h in lay:
                host.edgexpu_cpu_linear_quant_batch(hout[label].ctypes.data, hx[n_in].ctypes.data, h, WT, None,
                                                    m, n_out, n_in)
        err = host.edgexpu_b200_last_error()
        if err:
            raise RuntimeError(err.decode())

    host.edgexpu_b200_clear_error()
    e2e_step()
    if world > 1:
        dist.barrier()
    e_steps = max(1, min(args.steps, 3))
    t0 = time.perf_counter()
    for _ in range(e_steps):
        e2e_step()
    e2e_s = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
    e2e_tops = ops * world * e_steps / float(e2e_s.item()) / 1e12

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and WT == TYPE_Q4_K:
        try:
            ct, csec, threads = cpu_prefill(64, 10.0, 3)
            cpu_baseline = {"value": round(ct, 4), "unit": "TOPS", "cores": threads, "kind": "reference",
                            "sample": f"one layer's seven projections at 64 of {m} tokens per rep ({csec:.3f} s), "
                                      f"median over >= 10 s, reference AVX2 build (oracle/_ref) with OpenMP"}
        except FileNotFoundError as e:
            cpu_baseline = {"value": None, "unit": "TOPS", "cores": 0, "kind": "reference", "sample": f"unavailable: {e}"}

    line = {
        "metric": f"{tname} prefill GEMM useful int8 TOPS (llama3_8b_q4k_prefill, M {m})",
        "value": round(tops, 2), "unit": "TOPS", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_max / args.steps, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "i8 x i8 -> i32 -> f32" if WT == TYPE_Q8_0 else "u4/i8 x i8 -> i32 -> f32",
        "data": "synthetic (seeded random-init GGUF blocks generated in HBM)",
        "config": {"workload": "llama3_8b_q4k_prefill", "weight_type": tname, "batch": m, "layers": L,
                   "parallelism": f"replicas{world}" if world > 1 else "single", "ops_per_step": ops,
                   "prompt_tokens_per_s": round(m * world * args.steps / (ms_max / 1e3) * L / PREFILL["layers"], 1),
                   "graph": True, "l2": "weights larger than L2, streamed once per step", "per_projection": per_proj,
                   "spec_frac": round(tops / world / TENSOR_I8_SPEC_TOPS, 4)},
        "roofline": {"bound": "tensor", "achieved": round(tops / world, 1), "peak": round(peak, 1), "unit": "TOP/s",
                     "frac": round(tops / world / peak, 4), "traffic": None,
                     "kernel": ("gemm_q8_tc" if WT == TYPE_Q8_0 else "gemm_q4k_tc") + " (tcgen05 kind::i8) incl. its activation packing",
                     "peak_source": peak_src,
                     "note": ("exact integer path runs 2 int8 MMA passes per useful MAC (sc*q4 needs 10 bits)"
                              if WT == TYPE_Q4_K else "one int8 MMA of K = 32 per Q8_0 block into its own "
                              "accumulator; the per-block scaling on the CUDA cores binds")},
        "cpu_baseline": cpu_baseline,
        "e2e": {"value": round(e2e_tops, 2), "unit": "TOPS", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "edgexpu_cpu_linear_quant_batch (host buffers), one call per projection"},
        "gpu_launches": L * args.steps * sum(
            linear_launches(WT, m, shapes[grp[0]][2], [shapes[i][1] for i in grp], True,
                            torch.cuda.get_device_properties(dev).multi_processor_count) for grp in groups),
        "clocks": clocks,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graph
    torch.cuda.synchronize()
    pkg.shutdown()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ---- end to end through the reference's layer loop ---------------------------------------------

NATIVE_B200 = ROOT / "integration" / "_build" / "libedgexpu_native_b200.so"
NATIVE_REF = ROOT / "oracle" / "_ref" / "libedgexpu_ref_runtime.so"


def _bind_greedy(path):
    lib = ctypes.CDLL(str(path))
    f = lib.edgexpu_greedy_run
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                  ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
    return f


def _greedy(fn, path, prompt, n_new):
    import numpy as np

    ids = np.zeros(n_new, np.uint32)
    secs = np.zeros(2)
    err = ctypes.create_string_buffer(1024)
    made = fn(str(path).encode(), prompt.ctypes.data, prompt.size, n_new, ids.ctypes.data, None, 0, secs.ctypes.data,
              err, 1024)
    if made != n_new:
        raise RuntimeError(err.value.decode(errors="replace"))
    return ids, secs


def run_native(args):
    import tempfile

    world, rank, local = dist_env()
    os.environ["EDGEXPU_B200_DEVICE"] = str(local)
    pkg = load_pkg()
    from edgexpu_llm_b200 import gguf_synth as gs

    shape = gs.SMOLLM2_135M_Q8_0 if args.model == "smollm2" else gs.LLAMA3_8B_Q4_K
    if args.layers:
        shape = shape.with_layers(args.layers)
    n_prompt = args.prompt or (128 if args.model == "smollm2" else 512)
    n_new = args.steps
    is_ref = args.impl == "reference"
    if is_ref and rank != 0:
        return
    with tempfile.TemporaryDirectory() as td:
        path = gs.write_llama_gguf(pathlib.Path(td) / f"{shape.name}.gguf", shape, seed=0)
        prompt = gs.prompt_ids(shape, n_prompt, seed=0)
        ref_fn = _bind_greedy(NATIVE_REF) if NATIVE_REF.exists() else None
        if is_ref:
            if ref_fn is None:
                print(json.dumps({"impl": "reference", "unavailable": f"{NATIVE_REF} not built"}))
                return
            _greedy(ref_fn, path, prompt, min(n_new, max(1, args.warmup)))  # warm-up (thread probe, page cache)
            ids, secs = _greedy(ref_fn, path, prompt, n_new)
        else:
            pkg.load_cuda()
            if not pkg.load_cuda().edgexpu_cuda_set_float_order(0 if args.float_order == "x86" else 1):
                raise RuntimeError("set_float_order")
            fn = _bind_greedy(NATIVE_B200)
            _greedy(fn, path, prompt, min(n_new, max(1, args.warmup)))  # warm-up (first uploads, kernel attributes)
            ids, secs = _greedy(fn, path, prompt, n_new)
        tok_s = n_new / secs[1]
        ref_line = None
        if not is_ref and rank == 0 and world == 1 and ref_fn is not None and not args.no_cpu_baseline:
            r_ids, r_secs = _greedy(ref_fn, path, prompt, n_new)
            ref_line = {"value": round(n_new / r_secs[1], 3), "unit": "tok/s", "cores": host_threads(), "kind": "reference",
                        "sample": f"the same {n_prompt}-token prompt and {n_new} greedy tokens through the unchanged "
                                  f"reference runtime (oracle/_ref, AVX2 + OpenMP); prefill {r_secs[0]:.3f} s",
                        "greedy_ids_identical": bool((r_ids == ids).all())}
    wb = shape.weight_bytes_per_token()
    tot = torch_all_sum(tok_s, world) if (world > 1 and not is_ref) else tok_s
    peak, peak_kind = peak_hbm()
    line = {
        "metric": f"decode tok/s through the reference's layer loop ({shape.name}, batch 1)",
        "value": round(tot, 3), "unit": "tok/s", "n_gpus": 1 if is_ref else world, "steps": n_new,
        "warmup": args.warmup, "ms_per_step": round(secs[1] / n_new * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "i8 x i8 -> i32 -> f32" if shape.wtype == 8 else "u4/i8 x i8 -> i32 -> f32",
        "data": "synthetic (seeded random-init GGUF model, uniform random prompt ids)",
        "config": {"workload": "native_greedy", "model": shape.name, "layers": shape.n_layers, "prompt": n_prompt,
                   "greedy_tokens": n_new, "prefill_s": round(float(secs[0]), 4),
                   "parallelism": f"replicas{world}" if world > 1 else "single",
                   "float_order": None if is_ref else args.float_order,
                   "path": "reference runtime, unchanged, CPU" if is_ref else
                           "reference runtime + integration/edgexpu_b200.patch + host shim, linear and logits on B200"},
        "e2e": {"value": round(tot, 3), "unit": "tok/s", "h2d_bytes_per_step": 0 if is_ref else
                4 * shape.n_layers * (4 * shape.n_embd + shape.n_ff) + 4 * shape.n_embd,
                "d2h_bytes_per_step": 0 if is_ref else
                4 * shape.n_layers * (2 * shape.n_embd + 2 * shape.n_kv_heads * shape.head_dim + 2 * shape.n_ff) + 8},
    }
    if is_ref:
        line["impl"] = "reference"
        line["cpu_baseline"] = {"value": round(tok_s, 3), "unit": "tok/s", "cores": host_threads(), "kind": "reference",
                                "sample": f"{n_new} greedy tokens after a {n_prompt}-token prompt"}
    else:
        line["roofline"] = {"bound": "hbm", "achieved": round(wb / (secs[1] / n_new) / 1e9, 1), "peak": peak,
                            "unit": "GB/s", "frac": round(wb / (secs[1] / n_new) / 1e9 / peak, 4),
                            "note": "weight bytes per token / wall time per token: the host layer loop and one "
                                    "synchronous call per projection bound this path, not the kernels",
                            "peak_source": f"{peak_kind} hbm_gbs"}
        line["config"]["l2"] = "no flush: the weights of one token exceed L2 for llama3 and fit it for smollm2"
        line["cpu_baseline"] = ref_line
        # per synchronous call (7 projections per layer at batch 1, then the logits): the input pull, the
        # GEMV (it quantizes its own activations) and the finish kernel
        line["gpu_launches"] = n_new * (7 * shape.n_layers + 1) * 3
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_device_decode(args):
    import tempfile

    import numpy as np

    world, rank, local = dist_env()
    pkg = load_pkg()
    from edgexpu_llm_b200 import gguf_synth as gs

    shape = gs.SMOLLM2_135M_Q8_0 if args.model == "smollm2" else gs.LLAMA3_8B_Q4_K
    if args.layers:
        shape = shape.with_layers(args.layers)
    n_prompt = args.prompt or (128 if args.model == "smollm2" else 512)
    is_ref = args.impl == "reference"
    if is_ref and rank != 0:
        return
    ref_fn = _bind_greedy(NATIVE_REF) if NATIVE_REF.exists() else None
    with tempfile.TemporaryDirectory() as td:
        path = gs.write_llama_gguf(pathlib.Path(td) / f"{shape.name}.gguf", shape, seed=0)
        prompt = gs.prompt_ids(shape, n_prompt, seed=0)
        sample_n = min(args.steps, args.ref_tokens)
        if is_ref:
            if ref_fn is None:
                print(json.dumps({"impl": "reference", "unavailable": f"{NATIVE_REF} not built"}))
                return
            _greedy(ref_fn, path, prompt, 1)  # warm-up (thread probe, page cache)
            ids, secs = _greedy(ref_fn, path, prompt, sample_n)
            tok_s = sample_n / secs[1]
            line = {"metric": f"decode tok/s ({shape.name}, batch 1)", "value": round(tok_s, 3), "unit": "tok/s",
                    "n_gpus": 1, "steps": sample_n, "warmup": 1, "ms_per_step": round(secs[1] / sample_n * 1e3, 4),
                    "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 layer ops, int8 dots",
                    "data": "synthetic (seeded random-init GGUF model, uniform random prompt ids)",
                    "config": {"workload": "device_decode", "model": shape.name, "layers": shape.n_layers,
                               "prompt": n_prompt, "greedy_tokens": sample_n, "prefill_s": round(float(secs[0]), 4)},
                    "impl": "reference",
                    "cpu_baseline": {"value": round(tok_s, 3), "unit": "tok/s", "cores": host_threads(),
                                     "kind": "reference", "sample": f"{sample_n} greedy tokens after a {n_prompt}-token "
                                                                   "prompt (unchanged reference runtime)"},
                    "e2e": {"value": round(tok_s, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
            print(json.dumps(line), flush=True)
            return
        pkg.init(local)
        cuda = pkg.load_cuda()
        assert cuda.edgexpu_cuda_set_float_order(pkg.ORDER_X86) == 1
        window = n_prompt + args.warmup + args.steps + 1
        sess = ctypes.c_void_p()
        err = ctypes.create_string_buffer(1024)
        t_open = time.perf_counter()
        if not cuda.edgexpu_cuda_llama_open(str(path).encode(), window, ctypes.byref(sess), err, 1024):
            raise RuntimeError(err.value.decode())
        t_open = time.perf_counter() - t_open
        nxt = ctypes.c_uint32()
        ids = []

        def step(toks, pos):
            if not cuda.edgexpu_cuda_llama_forward(sess, toks.ctypes.data, toks.size, pos, 0.0, 1.0, None,
                                                   ctypes.byref(nxt), None, err, 1024):
                raise RuntimeError(err.value.decode())
            ids.append(nxt.value)
            return np.array([nxt.value], np.uint32)

        try:
            t0 = time.perf_counter()
            tok = step(prompt, 0)
            prefill_s = time.perf_counter() - t0
            pos = n_prompt
            for _ in range(args.warmup):
                tok = step(tok, pos)
                pos += 1
            sampler = ClockSampler(local)
            sampler.start()
            time.sleep(0.3)
            t_w0 = time.time()
            t0 = time.perf_counter()
            for _ in range(args.steps):
                tok = step(tok, pos)
                pos += 1
            dt = time.perf_counter() - t0
            t_w1 = time.time()
            clocks = sampler.stop(t_w0, t_w1)
        finally:
            cuda.edgexpu_cuda_llama_close(sess)
        tok_s = args.steps / dt
        ref_line = None
        if rank == 0 and world == 1 and ref_fn is not None and not args.no_cpu_baseline:
            r_ids, r_secs = _greedy(ref_fn, path, prompt, sample_n)
            ref_line = {"value": round(sample_n / r_secs[1], 3), "unit": "tok/s", "cores": host_threads(),
                        "kind": "reference",
                        "sample": f"{sample_n} greedy tokens after the same {n_prompt}-token prompt through the unchanged "
                                  f"reference runtime (oracle/_ref, AVX2 + OpenMP); prefill {r_secs[0]:.3f} s",
                        "greedy_ids_identical": bool((np.asarray(ids[:sample_n], np.uint32) == r_ids).all())}
    wb = shape.weight_bytes_per_token()
    tot = torch_all_sum(tok_s, world) if world > 1 else tok_s
    peak, peak_kind = peak_hbm()
    per_tok = dt / args.steps
    line = {
        "metric": f"decode tok/s ({shape.name}, batch 1)", "value": round(tot, 3), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_tok * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 layer ops, int8 x int8 -> i32 -> f32 dots",
        "data": "synthetic (seeded random-init GGUF model, uniform random prompt ids)",
        "config": {"workload": "device_decode", "model": shape.name, "layers": shape.n_layers, "prompt": n_prompt,
                   "greedy_tokens": args.steps, "prefill_s": round(prefill_s, 4), "open_s": round(t_open, 3),
                   "parallelism": f"replicas{world}" if world > 1 else "single", "float_order": "x86",
                   "l2": "no flush: the weights of one token exceed L2 for llama3 and fit it for smollm2",
                   "path": "edgexpu_cuda_llama_forward: one call per token, all layer ops on the B200"},
        "e2e": {"value": round(tot, 3), "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 8},
        "roofline": {"bound": "hbm", "achieved": round(wb / per_tok / 1e9, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(wb / per_tok / 1e9 / peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
                     "note": "weight bytes per token / wall time per token (each token's call waits for its id)"},
        "cpu_baseline": ref_line,
        # per token: the step word, the embedding row, per layer 2 norms + 4 GEMVs + RoPE/scores + softmax/V +
        # SwiGLU, the output norm, and the greedy logits GEMV
        "gpu_launches": args.steps * (9 * shape.n_layers + 4),
        "clocks": clocks,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)


def torch_all_sum(v, world):
    import torch
    import torch.distributed as dist

    if not dist.is_initialized():
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t)
    return float(t.item())


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["gemv", "llama3_8b_q4k_prefill", "native_greedy",
                                                              "device_decode"],
                    default="llama3_8b_q4k_decode")
    ap.add_argument("--wtype", choices=sorted(WTYPES), default="q4_k",
                    help="gemv workload: weight type; prefill workload: q4_k or q8_0")
    ap.add_argument("--shape", default="14336,4096", help="gemv workload: n_out,n_in")
    ap.add_argument("--rotate-bytes", type=float, default=512e6, help="gemv workload: total bytes of weight copies")
    ap.add_argument("--batch", type=int, default=0, help="tokens per step (default 1 for decode, 2048 for prefill)")
    ap.add_argument("--layers", type=int, default=0, help="prefill workload: layers per step (0 = all 32)")
    ap.add_argument("--ref-layers", type=int, default=0,
                    help="reference arm: layers per step (0 = a sample of about 0.6 GB per step)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--model", choices=["smollm2", "llama3"], default="smollm2", help="native_greedy workload: model")
    ap.add_argument("--prompt", type=int, default=0, help="native_greedy workload: prompt ids (128 / 512 by model)")
    ap.add_argument("--ref-tokens", type=int, default=16, help="device_decode workload: tokens of the CPU reference sample")
    ap.add_argument("--float-order", choices=["x86", "relaxed"], default="relaxed",
                    help="relaxed: the GEMV's own summation order, within 1e-5 * sum|w x| of the reference; x86: float "
                         "outputs bit-identical to the reference's x86 build (the library's default order, the one "
                         "the token-identical decode needs).  The decode line also reports the other order's times.")
    ap.add_argument("--no-compare-orders", dest="compare_orders", action="store_false",
                    help="decode workloads: do not time the step in the other float order as well")
    ap.add_argument("--collective", choices=["p2p", "nccl"], default="p2p",
                    help="tensor parallel: all-reduce of o/down inside the GEMV over NVLink (p2p) or NCCL after it")
    args = ap.parse_args()
    if args.batch <= 0:
        args.batch = 2048 if args.workload == "llama3_8b_q4k_prefill" else 1
    if args.workload == "llama3_8b_q4k_prefill":
        if args.wtype not in ("q4_k", "q8_0"):
            ap.error("the prefill workload runs the Q4_K and Q8_0 tensor-core GEMMs: --wtype q4_k or q8_0")
        (run_prefill_reference if args.impl == "reference" else run_prefill)(args)
        return
    if args.workload == "device_decode":
        run_device_decode(args)
        return
    if args.workload == "native_greedy":
        if args.float_order == "relaxed" and "--float-order" not in sys.argv:
            args.float_order = "x86"  # the token-identical order is this workload's point
        run_native(args)
        return
    if args.workload == "gemv":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the gemv workload has no reference arm; "
                                                                  "use the decode workloads"}))
            return
        run_gemv(args)
        return
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, wl)
    else:
        run_ours(args, wl)


if __name__ == "__main__":
    main()

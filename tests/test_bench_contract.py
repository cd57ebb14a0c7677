"""CPU checks of bench.py's accounting: the algorithmic bytes behind every roofline figure.

* Block sizes of every weight type equal the package's table (synth.BLOCK, the GGUF layouts of
  gguf_quant.c:468-480).
* One Llama-3-8B decode step streams 4,221,370,368 bytes of Q4_K weights at batch 1 (32 layers of
  q, k, v, o, gate, up, down plus the 128256-row output.weight), the per-token figure the
  configuration states.  At batch b the projections' weights count once and b * (4K + 292K/256 +
  4N) of activations and outputs per projection are added; the step makes one greedy-logits call
  per token (the reference samples each sequence on its own, native.c:2355-2397), so the
  output.weight, the fp32 hidden state and the 8-byte key count b times.
* The command line refuses what it cannot measure, without touching a GPU.
"""

import importlib.util
import json
import subprocess
import sys

import pytest

import _oracle

ROOT = _oracle.REPO


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _synth():
    _oracle.load_pkg()
    import edgexpu_llm_b200.synth as s

    return s


def test_block_sizes_match_the_package():
    b, s = _bench(), _synth()
    assert set(b.BLOCKS) == set(s.BLOCK)
    for t in b.WTYPES.values():
        for n in (256, 4096, 14336):
            assert b.row_bytes(t, n) == s.row_bytes(t, n)
        assert b.act_bytes(t, 4096) == (4096 // 32 * 34 if s.BLOCK[t][0] == 32 else 4096 // 256 * 292)


def test_decode_step_bytes():
    b = _bench()
    wl = b.WORKLOADS["llama3_8b_q4k_decode"]
    t = wl["type"]
    layers = wl["layers"] * sum(n_out * b.row_bytes(t, n_in) for _, n_out, n_in, _k in wl["proj"])
    logits = wl["vocab"] * b.row_bytes(t, wl["hidden"])
    assert layers + logits == 4_221_370_368
    for m in (1, 16):
        acts = wl["layers"] * sum(m * (4 * n_in + b.act_bytes(t, n_in) + 4 * n_out) for _, n_out, n_in, _k in wl["proj"])
        assert b.step_bytes(wl, m) == layers + acts + m * (logits + 4 * wl["hidden"] + 8)
    assert b.step_bytes(wl, 16) == 8_844_656_768  # the batch-16 step: 6.64 ms = 1333 GB/s


def test_tensor_parallel_shards_cover_the_step():
    b = _bench()
    wl = b.WORKLOADS["llama3_8b_q4k_decode"]
    t = wl["type"]
    full, _, vocab = b.shard_shapes(wl, 1, 0)
    for world in (2, 4, 8):
        total = 0
        rows = 0
        for rank in range(world):
            shapes, v0, nv = b.shard_shapes(wl, world, rank)
            assert v0 == rank * nv
            rows += nv
            total += sum(n_out * b.row_bytes(t, n_in) for _, n_out, n_in, _k in shapes)
        assert rows == vocab
        assert total == sum(n_out * b.row_bytes(t, n_in) for _, n_out, n_in, _k in full)


def _run(*args):
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True, timeout=120)


def test_prefill_refuses_other_weight_types():
    r = _run("--workload", "llama3_8b_q4k_prefill", "--wtype", "q6_k")
    assert r.returncode == 2 and "q4_k or q8_0" in r.stderr


@pytest.mark.parametrize("wtype", ["q4_0", "q6_k"])
def test_gemv_reference_arm_is_unavailable(wtype):
    r = _run("--impl", "reference", "--workload", "gemv", "--wtype", wtype)
    assert r.returncode == 0
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and "unavailable" in line


def test_launch_counts_follow_the_library_routing():
    """linear_launches restates the library's routing (capi.cu run_linear_dev and the grouped call,
    tp_p2p.cu's linear, gemm_tc.cu tc_split) on 148 SMs; the cases below were traced by hand."""
    b = _bench()
    Q4K, Q80, SM = b.TYPE_Q4_K, b.TYPE_Q8_0, 148
    # batch 1: the GEMV quantizes in its prologue, one launch per call (the headline's 129 per token)
    assert b.linear_launches(Q4K, 1, 4096, [4096, 1024, 1024], True, SM) == 1
    assert b.linear_launches(Q4K, 1, 14336, [4096], True, SM, tp_col=True) == 1
    wl = b.WORKLOADS["llama3_8b_q4k_decode"]
    assert wl["layers"] * 4 + 1 == 129
    # batch 16, relaxed: one packing, then per tensor a K-split GEMM and its reduction
    assert b.linear_launches(Q4K, 16, 4096, [4096, 1024, 1024], True, SM) == 7
    assert b.linear_launches(Q4K, 16, 4096, [14336, 14336], True, SM) == 5
    assert b.linear_launches(Q4K, 16, 14336, [4096], True, SM) == 3
    # prefill: 128-token tiles cover the SMs, no split
    assert b.linear_launches(Q4K, 2048, 4096, [14336], True, SM) == 2
    assert b.tc_split_ranges(2048, 14336, 4096, SM) == 1
    # x86 order: quantize once, then GEMV chunks of rows (16 at K = 4096, 5 at K = 14336)
    assert b.rowstream_max_m(Q4K, 4096) == 16 and b.rowstream_max_m(Q4K, 14336) == 5
    assert b.linear_launches(Q4K, 16, 4096, [4096], False, SM) == 2
    assert b.linear_launches(Q4K, 16, 14336, [4096], False, SM) == 5
    # Q8_0: configuration 0's GEMV, and the tensor-core GEMM from 64 rows (packing + GEMM)
    assert b.linear_launches(Q80, 1, 576, [1536], True, SM) == 1
    assert b.linear_launches(Q80, 4, 576, [1536], True, SM) == 2
    assert b.linear_launches(Q80, 64, 4096, [4096, 1024], True, SM) == 4


def test_prefill_layer_launch_counts():
    """One prefill layer: Q4_K packs once per group (4) and runs one GEMM per tensor (7); Q8_0 packs
    per tensor (7 x 2)."""
    b = _bench()
    shapes, groups = b.PREFILL["proj"], [[0, 1, 2], [3], [4, 5], [6]]

    def per_layer(wt, m):
        return sum(b.linear_launches(wt, m, shapes[g[0]][2], [shapes[i][1] for i in g], True, 148) for g in groups)

    assert per_layer(b.TYPE_Q4_K, 2048) == 11
    assert per_layer(b.TYPE_Q8_0, 2048) == 14

"""The benchmark's host-side pieces (no GPU): the algorithmic byte and FLOP counts the
roofline uses, the synthetic workloads, and the reference arm's JSON line."""

import json
import subprocess
import sys

import torch

import bench
from conftest import ROOT


def test_decode_counts_match_the_reference_bench_model():
    # cfg2: T = 32 x 4096 cached tokens, H = 128 (the reference bench's model, bench.py:80-81).
    t = 32 * 4096
    assert bench.decode_bytes(t, 32, 128) == (t * 576 + 32 * 128 * 576 + 32 * 128 * 512) * 2
    assert abs(bench.decode_bytes(t, 32, 128) / 1e6 - 159.9) < 0.1
    assert abs(bench.decode_flops(t, 128) / 1e9 - 36.5) < 0.1


def test_layer_counts_for_the_deepseek_layer_step():
    flops, nbytes = bench.layer_counts(16, 8192)
    # 374 MB of weights and 155 MB of cache (plus q / out / x) per GPU.
    assert 525e6 < nbytes < 535e6
    assert flops > bench.decode_flops(16 * 8193, 128)


def test_workloads_have_the_baseline_shapes():
    cpu = torch.device("cpu")
    q, kv, lens, bt = bench.make_workload(bench.CONFIGS["cfg2"], cpu, seed=1)
    assert q.shape == (32, 128, 576) and kv.shape == (2048, 64, 576) and q.dtype == torch.bfloat16
    assert bool((lens == 4096).all()) and bt.shape == (32, 64)
    assert sorted(bt.flatten().tolist()) == list(range(2048)), "every page used once"
    small_ragged = dict(bench.CONFIGS["cfg4"], batch=24, seqlen=2000)  # cfg4's generator, small
    q, kv, lens, bt = bench.make_workload(small_ragged, cpu, seed=1000)
    assert q.shape[0] == 24 and int(lens.min()) >= 1 and int(lens.max()) <= 2000
    need = (lens + 63) // 64
    used = torch.cat([bt[b, : int(n)] for b, n in enumerate(need)])
    assert used.numel() == kv.shape[0] and used.unique().numel() == used.numel(), "pages without replacement"


def test_sharded_workload_partitions_the_global_batch():
    cpu = torch.device("cpu")
    cfg = dict(bench.CONFIGS["cfg4"], batch=40, seqlen=3000)
    total = 0
    for rank in range(4):
        q, kv, lens, bt, job_tokens, job_batch = bench.make_sharded_workload(cfg, cpu, 1000, rank, 4)
        total += int(lens.sum())
        assert job_batch == 40 and q.shape[0] == lens.shape[0]
    assert total == job_tokens


def test_uniform_config_is_split_over_the_ranks():
    """Strong scaling of config 2: the global batch of 32 requests x 4096 tokens is cut into
    equal contiguous slices, each rank holding only its own requests' pages."""
    cpu = torch.device("cpu")
    cfg = dict(bench.CONFIGS["cfg2"], seqlen=256)  # config 2's batch, short requests
    for world in (1, 2, 4, 8):
        total, rows = 0, 0
        for rank in range(world):
            q, kv, lens, bt, job_tokens, job_batch = bench.make_sharded_workload(cfg, cpu, 1000, rank, world)
            assert q.shape == (32 // world, 128, 576) and kv.shape[0] == (32 // world) * 4
            assert sorted(bt.flatten().tolist()) == list(range(kv.shape[0])), "a rank-local pool, every page once"
            total += int(lens.sum())
            rows += q.shape[0]
        assert job_batch == 32 and rows == 32 and total == job_tokens == 32 * 256
    # config 3's four requests over eight ranks: four ranks hold none
    q, kv, lens, bt, _, _ = bench.make_sharded_workload(dict(bench.CONFIGS["cfg3"], seqlen=128), cpu, 1000, 7, 8)
    assert q.shape[0] == 0 and lens.numel() == 0


def test_reference_arm_prints_one_json_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "2", "--warmup", "3"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [line for line in r.stdout.splitlines() if line.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == "TFLOPS"
    assert d["value"] > 0 and d["steps"] == 2 and d["warmup"] == 3
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0

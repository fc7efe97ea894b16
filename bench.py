"""Benchmark of the B200 MLA decode path (one JSON line on stdout, rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg2] [--impl ours|reference|cutlass-mla]

A step is one ``mla_decode`` call over one batch of the workload (BASELINE
config 2 by default: B=32 requests x 4096 cached tokens, H=128, bf16, paged
cache with 64-token pages, shuffled block table, scale 1/sqrt(192)), inputs
resident in HBM, L2 flushed (256 MiB write) before every timed step, each step
timed with CUDA events on the launching stream.

Multi-GPU (``torchrun --nproc-per-node N bench.py --gpus N``): requests are
independent, so the config's batch is split over the ranks (equal contiguous
slices, or token-balanced shards of the ragged config) and every rank decodes its
share from its own page pool; there is no collective on the data path (NCCL only
for barriers, the per-rank times and the max-over-ranks timing).  Scaling is
strong: the total work is fixed.  ``--weak`` gives every rank a whole batch of a
uniform config instead.

``--config cfg5`` times one decode step of the full MLA layer instead (BASELINE
config 5: DeepSeek-V3 dims, random-init weights, 16 requests per GPU with 8192
cached tokens, weights replicated on every rank).

``--impl reference`` times the reference algorithm's CPU restatement (the
numpy oracle) on the host cores on a bounded sample of the same workload.
``--impl cutlass-mla`` times a library kernel (vLLM's CUTLASS sm100 MLA decode)
on the same workload, one GPU, for comparison; ``--impl reference-gpu`` times the
reference's own Triton kernel (installed unmodified in baseline/_ref) the same way.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "triton-mla_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "MLA decode µs/call and TFLOPS (H=128, bf16, paged) vs roofline at 1/2/4/8 B200"
D_QK, D_V, PAGE = 576, 512, 64
SCALE = 192 ** -0.5
L2_FLUSH_BYTES = 256 << 20
HOST_LEAD_CYCLES = 200_000  # ~0.1 ms of device-side wait before each timed step (outside the events)
# The end-to-end figure is the median of E2E_ROUNDS runs of the K pipelined steps, E2E_GAP_S
# apart: the host link is shared with the machine's other GPUs, and a single run of a few
# milliseconds can fall inside an episode where uploads take 2-5x longer.
E2E_ROUNDS = 5
E2E_GAP_S = 0.2

CONFIGS = {
    "cfg2": dict(desc="BASELINE config 2: B=32 H=128 S=4096 (all requests) page 64 bf16 paged, shuffled pages",
                 batch=32, seqlen=4096, ragged=False),
    "cfg3": dict(desc="BASELINE config 3: B=4 H=128 S=65536 page 64 bf16 paged, shuffled pages",
                 batch=4, seqlen=65536, ragged=False),
    "cfg4": dict(desc="BASELINE config 4: B=256 H=128 S~U[1,16384] page 64 bf16, pages from one shared pool",
                 batch=256, seqlen=16384, ragged=True),
    "cfg5": dict(desc="BASELINE config 5: MLA layer decode step, DeepSeek-V3 dims (hidden 7168, q_lora 1536, "
                      "kv_lora 512, nope 128, rope 64, v 128, H=128), 16 requests per GPU x 8192 cached tokens, "
                      "page 64, bf16, random-init weights N(0,0.02)",
                 batch=16, seqlen=8192, ragged=False, layer=True),
}


def decode_flops(total_tokens, heads):
    """Algorithmic FLOPs of one call: T*H*2*(576+512) (the reference bench's model, bench.py:81)."""
    return float(total_tokens) * heads * 2 * (D_QK + D_V)


def decode_bytes(total_tokens, batch, heads, elt=2, row_bytes=None):
    """Algorithmic bytes of one call: cache rows + q + out (bench.py:80 of the reference);
    ``row_bytes`` overrides the cache bytes per token (656 for FP8 rows)."""
    rows = total_tokens * (row_bytes if row_bytes else D_QK * elt)
    return float(rows + (batch * heads * D_QK + batch * heads * D_V) * elt)


def bind_to_gpu_cpus(device_index):
    """Run this process on the CPUs the driver reports as local to the GPU (NVML), so that its
    pinned host buffers sit next to the GPU's PCIe link.  Returns the previous CPU set, or None
    when NVML cannot tell.  Only reads the GPU's topology; changes nothing on the GPU."""
    try:
        import pynvml
        import torch
        props = torch.cuda.get_device_properties(device_index)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        try:
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            words = pynvml.nvmlDeviceGetCpuAffinity(handle, (os.cpu_count() + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
        before = os.sched_getaffinity(0)
        cpus = {64 * w + bit for w, mask in enumerate(words) for bit in range(64) if (mask >> bit) & 1} & before
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return before
    except Exception:  # noqa: BLE001 - best effort: no NVML, no topology, no permission
        return None


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def make_workload(cfg, device, seed):
    import torch
    gen_cpu = torch.Generator().manual_seed(seed)
    if cfg["ragged"]:
        lens = torch.randint(1, cfg["seqlen"] + 1, (cfg["batch"],), generator=gen_cpu, dtype=torch.int32)
    else:
        lens = torch.full((cfg["batch"],), cfg["seqlen"], dtype=torch.int32)
    need = (lens + PAGE - 1) // PAGE
    num_pages = int(need.sum())
    g = torch.Generator(device=device).manual_seed(seed)
    kv = torch.randn(num_pages, PAGE, D_QK, generator=g, device=device, dtype=torch.bfloat16)
    q = torch.randn(cfg["batch"], 128, D_QK, generator=g, device=device, dtype=torch.bfloat16)
    perm = torch.randperm(num_pages, generator=gen_cpu)
    bt = torch.zeros(cfg["batch"], int(need.max()), dtype=torch.int32)
    at = 0
    for b, k in enumerate(need.tolist()):
        bt[b, :k] = perm[at:at + k].int()
        at += k
    return q, kv, lens.to(device), bt.to(device)


def make_sharded_workload(cfg, device, seed, rank, world):
    """One global batch of the config (the same lengths on every rank, from ``seed``) split
    over the ranks: equal contiguous slices of a uniform batch, or, for the ragged config,
    token-balanced shards (longest first onto the least-loaded rank).  This rank builds only
    its own requests' q rows, page pool and block table.  Returns the rank's inputs and the
    global token count and batch size."""
    import torch
    from triton_mla.sharding import balance_requests, contiguous_requests
    gen_cpu = torch.Generator().manual_seed(seed)
    if cfg["ragged"]:
        lens_all = torch.randint(1, cfg["seqlen"] + 1, (cfg["batch"],), generator=gen_cpu, dtype=torch.int32)
        reqs = balance_requests(lens_all.tolist(), world)[rank]
    else:
        lens_all = torch.full((cfg["batch"],), cfg["seqlen"], dtype=torch.int32)
        reqs = contiguous_requests(cfg["batch"], world)[rank]
    lens = lens_all[reqs]
    need = (lens + PAGE - 1) // PAGE
    num_pages = max(1, int(need.sum()))
    g = torch.Generator(device=device).manual_seed(seed + 1 + rank)
    kv = torch.randn(num_pages, PAGE, D_QK, generator=g, device=device, dtype=torch.bfloat16)
    q = torch.randn(len(reqs), 128, D_QK, generator=g, device=device, dtype=torch.bfloat16)
    perm = torch.randperm(num_pages, generator=gen_cpu)
    bt = torch.zeros(len(reqs), max(1, int(need.max()) if len(reqs) else 1), dtype=torch.int32)
    at = 0
    for b, k in enumerate(need.tolist()):
        bt[b, :k] = perm[at:at + k].int()
        at += k
    return q, kv, lens.to(device), bt.to(device), int(lens_all.sum()), cfg["batch"]


def layer_counts(batch, context):
    """Algorithmic FLOPs and bytes of one MLA layer decode step (DeepSeek-V3 dims, bf16):
    the projections wq_a, wq_b, wkv_a, wo and the absorption by W_UK / W_UV read every
    weight once (2 FLOPs per weight and request), plus the decode over context + 1 tokens."""
    hid, qr, h, r = 7168, 1536, 128, 512
    linear = hid * qr + qr * h * 192 + hid * (r + 64) + h * 128 * hid
    absorb = 2 * h * 128 * r
    tokens = batch * (context + 1)
    flops = 2.0 * batch * (linear + absorb) + decode_flops(tokens, h)
    nbytes = 2.0 * (linear + absorb) + decode_bytes(tokens, batch, h) + 2.0 * 2 * batch * hid
    return flops, nbytes


def run_layer(args, cfg, device, world, rank, local):
    """--config cfg5: one MLA layer decode step per timed step (weak scaling: every rank holds
    the weights and its own 16 requests)."""
    import torch
    import torch.distributed as dist
    from triton_mla import MLA, MLAConfig, MLADecodeGraph, get_num_splits
    torch.manual_seed(1000 + rank)
    mcfg = MLAConfig()
    layer = MLA(mcfg)
    with torch.no_grad():
        for name, prm in layer.named_parameters():
            if "norm" in name:
                prm.fill_(1.0)
            else:
                prm.normal_(0.0, 0.02)
    layer = layer.to(device=device, dtype=torch.bfloat16)
    B, ctx = cfg["batch"], cfg["seqlen"]
    need = (ctx + 1 + PAGE - 1) // PAGE
    g = torch.Generator(device=device).manual_seed(1000 + rank)
    kv = torch.randn(B * need, PAGE, D_QK, generator=g, device=device, dtype=torch.bfloat16)
    bt = torch.randperm(B * need, generator=torch.Generator().manual_seed(rank)).view(B, need).int().to(device)
    lens = torch.full((B,), ctx, dtype=torch.int32, device=device)
    x = torch.randn(B, mcfg.hidden_size, generator=g, device=device, dtype=torch.bfloat16)
    splits = get_num_splits(B, 128, ctx + 1, torch.cuda.get_device_properties(device).multi_processor_count)
    # The library's launches per step: kv append (+ q_norm), the decode query's RoPE and W_UK
    # product, W_UV, the decode (+ merge), the projections that take the tcgen05 projection
    # kernel ([wq_a; wkv_a], wq_b, wo) and the L2 prefetch beside the decode.
    from triton_mla import layer_ops
    x_rows = torch.empty(B, mcfg.hidden_size, device=device, dtype=torch.bfloat16)
    q_rows = torch.empty(B, mcfg.q_lora_rank, device=device, dtype=torch.bfloat16)
    o_rows = torch.empty(B, mcfg.num_heads * mcfg.v_head_dim, device=device, dtype=torch.bfloat16)
    layer_launches = 4 + (2 if splits > 1 else 1) + sum(
        layer_ops.linear_preferred(a, w)
        for a, w in ((x_rows, layer._w_a()), (q_rows, layer.wq_b.weight), (o_rows, layer.wo.weight)))
    # the L2 prefetch beside the decode: W_UV, and the first part of wo when asked for
    if layer.l2_prefetch_wo_bytes >= 0:
        layer_launches += 1 + (layer.l2_prefetch_wo_bytes > 0)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    flops, nbytes = layer_counts(B, ctx)

    @torch.no_grad()
    def eager_step(xin):
        # the new token is written at position ctx every step, so the work per step is fixed
        out, _ = layer(xin, kv, lens, bt, num_splits=splits)
        return out

    # The timed step is the layer step captured in a CUDA graph (one launch per step).
    graph = MLADecodeGraph(layer, kv, lens, bt, num_splits=splits)

    def step(xin):
        return graph(xin)

    for _ in range(args.warmup):
        step(x)
        eager_step(x)
    torch.cuda.synchronize()
    eager = []
    for _ in range(args.steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        eager_step(x)
        b.record(stream)
        eager.append((a, b))
    torch.cuda.synchronize()
    eager_us = 1e3 * sum(a.elapsed_time(b) for a, b in eager) / len(eager)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        t_soak = time.perf_counter()
        while time.perf_counter() - t_soak < args.clock_soak:
            for _ in range(8):
                flush.zero_()
                step(x)
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for i in range(args.steps):
            flush.zero_()
            starts[i].record(stream)
            step(x)
            ends[i].record(stream)
        torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in zip(starts, ends)) / args.steps
    t = torch.tensor([ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())

    # end to end: x from pinned host memory in, the layer output back to the host
    x_h = x.cpu().pin_memory()
    out_h = torch.empty(B, mcfg.hidden_size, dtype=torch.bfloat16).pin_memory()
    e_ms = []
    for i in range(args.warmup + args.steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        out_h.copy_(step(x_h.to(device, non_blocking=True)), non_blocking=True)
        b.record(stream)
        b.synchronize()
        if i >= args.warmup:
            e_ms.append(a.elapsed_time(b))
    te = torch.tensor([sum(e_ms) / len(e_ms)], device=device)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    hbm, tflops_peak, peak_kind = peaks()
    t_bytes, t_flops = nbytes / (hbm * 1e9), flops / (tflops_peak * 1e12)
    bound = "hbm" if t_bytes >= t_flops else "tensor"
    achieved = (nbytes / (ms * 1e-3) / 1e9) if bound == "hbm" else (flops / (ms * 1e-3) / 1e12)
    peak = hbm if bound == "hbm" else tflops_peak
    cpu = None
    if world == 1 and args.cpu_budget > 0:
        if getattr(args, "all_cpus", None):
            os.sched_setaffinity(0, args.all_cpus)  # the CPU baseline runs on all of the host's cores
        cpu = cpu_layer_rate(layer, kv, bt, ctx, min(args.cpu_budget, 20.0))
    line = {
        "metric": METRIC, "value": world * flops / (ms_max * 1e-3) / 1e12, "unit": "TFLOPS", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max, "us_per_call": ms_max * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic N(0,1) cache and input, random-init weights (no checkpoint, no dataset)",
        "config": {"workload": cfg["desc"], "batch_per_gpu": B, "global_batch": world * B, "context": ctx,
                   "num_splits": splits, "step": "MLADecodeGraph (the layer step captured in one CUDA graph)",
                   "eager_us_per_step": eager_us, "l2": "flushed (256 MiB write) before every timed step",
                   "parallelism": f"dp{world} (weights replicated, each rank its own requests and page pool)"},
        "roofline": {"bound": bound, "achieved": achieved, "peak": peak, "unit": "GB/s" if bound == "hbm" else "TFLOP/s",
                     "frac": achieved / peak, "traffic": None, "traffic_source": "not captured for this config",
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json)" if peak_kind == "measured" else "fallback",
                     "kernel": "whole layer step (tcgen05 decode; the [wq_a; wkv_a], wq_b, W_UK, W_UV and "
                               "wo products on the tcgen05 projection kernel)",
                     "algorithmic_bytes_per_step": nbytes, "algorithmic_flops_per_step": flops},
        "cpu_baseline": cpu,
        "e2e": {"value": world * flops / (float(te.item()) * 1e-3) / 1e12, "unit": "TFLOPS",
                "ms_per_step": float(te.item()), "h2d_bytes_per_step": x_h.numel() * 2,
                "d2h_bytes_per_step": out_h.numel() * 2,
                "note": "per step: x host->device, layer output device->host; weights and cache resident"},
        "gpu_launches": args.steps * layer_launches,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)
    return 0


def cpu_layer_rate(layer, kv, bt, ctx, budget_s):
    """The numpy layer oracle (absorbed form, fp64) on one request of the workload, timed on
    the host cores for about ``budget_s`` seconds."""
    import numpy as np
    from oracle import mla_oracle as orc
    w = {k: v.float().cpu().numpy() for k, v in layer.state_dict().items()}
    w = {k.replace(".weight", ""): v for k, v in w.items()}
    ocfg = dict(hidden_size=7168, num_heads=128, q_lora_rank=1536, kv_lora_rank=512, qk_nope_head_dim=128,
                qk_rope_head_dim=64, v_head_dim=128, rope_theta=10000.0, rms_norm_eps=1e-6)
    need = bt.shape[1]
    pages = bt[0].long().cpu()
    kv1 = kv.index_select(0, pages.to(kv.device)).float().cpu().numpy()
    bt1 = np.arange(need, dtype=np.int32)[None]
    x = np.random.default_rng(0).standard_normal((1, 7168)).astype(np.float32)
    done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s or done == 0:
        orc.mla_layer_forward_absorbed(w, ocfg, x, kv1, np.array([ctx]), bt1)
        done += 1
    el = time.perf_counter() - t0
    flops, _ = layer_counts(1, ctx)
    return {"value": done * flops / el / 1e12, "unit": "TFLOPS", "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"{done} layer steps of 1 request x {ctx} tokens in {el:.1f}s "
                      "(numpy layer oracle, fp64, BLAS threads = all host cores)"}


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples every 50 ms while running."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "window": "soak of the same steps + timed region"}


def cpu_oracle_rate(budget_s=10.0, seqlen=4096, heads=128):
    """The numpy oracle (reference algorithm) on host cores: TFLOPS on whole requests of the workload."""
    import numpy as np
    from oracle import mla_oracle as orc
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, heads, D_QK), dtype=np.float32)
    kv = rng.standard_normal((1, seqlen, D_QK), dtype=np.float32)
    lens = np.array([seqlen])
    orc.mla_decode_ref(q, kv, lens, None, softmax_scale=SCALE, dtype=np.float32)  # warm
    done, t0 = 0, time.perf_counter()
    while True:
        orc.mla_decode_ref(q, kv, lens, None, softmax_scale=SCALE, dtype=np.float32)
        done += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    flops = decode_flops(seqlen * done, heads)
    return flops / el / 1e12, done, el


def run_reference(args):
    """--impl reference: the reference algorithm's CPU restatement, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import numpy as np
    from oracle import mla_oracle as orc
    cfg = CONFIGS[args.config]
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(0)
    seqlen = cfg["seqlen"] if not cfg["ragged"] else 8192
    q = rng.standard_normal((1, 128, D_QK), dtype=np.float32)
    kv = rng.standard_normal((1, seqlen, D_QK), dtype=np.float32)
    lens = np.array([seqlen])
    for _ in range(args.warmup):
        orc.mla_decode_ref(q, kv, lens, None, softmax_scale=SCALE, dtype=np.float32)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        orc.mla_decode_ref(q, kv, lens, None, softmax_scale=SCALE, dtype=np.float32)
        times.append(time.perf_counter() - t0)
    ms = 1e3 * sum(times) / len(times)
    tflops = decode_flops(seqlen, 128) / (ms * 1e-3) / 1e12
    sample = f"1 request x {seqlen} tokens x 128 heads per step (fp32 numpy, BLAS threads={threads})"
    line = {
        "impl": "reference", "metric": METRIC, "value": tflops, "unit": "TFLOPS", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1)",
        "config": {"workload": cfg["desc"], "sample": sample},
        "cpu_baseline": {"value": tflops, "unit": "TFLOPS", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": tflops, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


REFERENCE_GPU_SCRIPT = r"""
import json, sys, time
sys.path.insert(0, {root!r})
import bench
sys.path[:] = [p for p in sys.path if not p.endswith("triton-mla_b200")]
sys.path.insert(0, {ref!r})
import numpy as np
import torch
import triton_mla
from triton_mla import mla_decode
assert triton_mla.__file__.startswith({ref!r}), triton_mla.__file__
from oracle import mla_oracle as orc
cfg = bench.CONFIGS[{config!r}]
device = torch.device("cuda", 0)
torch.cuda.set_device(device)
q, kv, lens, bt = bench.make_workload(cfg, device, seed=1000)
for _ in range({warmup}):
    out = mla_decode(q, kv, lens, bt, softmax_scale=bench.SCALE)
torch.cuda.synchronize()
flush = torch.empty(bench.L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
stream = torch.cuda.current_stream(device)
starts = [torch.cuda.Event(enable_timing=True) for _ in range({steps})]
ends = [torch.cuda.Event(enable_timing=True) for _ in range({steps})]
for i in range({steps}):
    flush.zero_()
    starts[i].record(stream)
    out = mla_decode(q, kv, lens, bt, softmax_scale=bench.SCALE)
    ends[i].record(stream)
torch.cuda.synchronize()
ms = sum(a.elapsed_time(b) for a, b in zip(starts, ends)) / {steps}
n = int(lens[0])
rows = kv[bt[0, : (n + 63) // 64].long()].reshape(-1, 576)[:n].float().cpu().numpy()
ref, _ = orc.mla_decode_ref(q[:1].float().cpu().numpy(), rows[None], np.array([n]), None, softmax_scale=bench.SCALE,
                            dtype=np.float32)
err = float(np.abs(out[:1].float().cpu().numpy() - ref).max())
print(json.dumps({{"ms": ms, "tokens": int(lens.sum()), "batch": int(q.shape[0]), "max_abs_err_request0": err,
                  "triton": __import__("triton").__version__}}))
"""


def run_reference_gpu(args):
    """--impl reference-gpu: the reference's own Triton ``mla_decode`` (installed unmodified into
    baseline/_ref) on the same workload, GPU 0, for comparison.  It runs in a subprocess, since
    the reference's package has the same import name as this repository's.  Measurement only."""
    line = {"impl": "reference-gpu", "metric": METRIC, "n_gpus": args.gpus}
    ref = ROOT / "baseline" / "_ref"
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    if not (ref / "triton_mla" / "kernel.py").exists():
        line["unavailable"] = "the reference is not installed in baseline/_ref"
        print(json.dumps(line), flush=True)
        return 0
    cfg = CONFIGS[args.config]
    if cfg.get("layer"):
        line["unavailable"] = "the reference GPU comparison covers the decode configs (cfg2-cfg4)"
        print(json.dumps(line), flush=True)
        return 0
    script = REFERENCE_GPU_SCRIPT.format(root=str(ROOT), ref=str(ref), config=args.config, warmup=args.warmup,
                                         steps=args.steps)
    r = subprocess.run([sys.executable, "-c", script], capture_output=True, text=True, timeout=1800)
    if r.returncode != 0:
        line["unavailable"] = "the reference Triton kernel did not run: " + (r.stderr.strip().splitlines() or ["?"])[-1]
        print(json.dumps(line), flush=True)
        return 0
    d = json.loads(r.stdout.strip().splitlines()[-1])
    tflops = decode_flops(d["tokens"], 128) / (d["ms"] * 1e-3) / 1e12
    line.update({
        "value": tflops, "unit": "TFLOPS", "steps": args.steps, "warmup": args.warmup, "ms_per_step": d["ms"],
        "us_per_call": d["ms"] * 1e3, "higher_is_better": True, "dtype": "bf16", "data": "synthetic N(0,1)",
        "config": {"workload": cfg["desc"], "batch": d["batch"], "tokens": d["tokens"],
                   "num_splits": "reference default (num_splits=None: get_num_splits, one host sync)",
                   "l2": "flushed (256 MiB write) before every timed step"},
        "reference": f"triton_mla 0.1.1 (unmodified, baseline/_ref), triton {d['triton']}",
        "max_abs_err_request0_vs_oracle": d["max_abs_err_request0"],
    })
    print(json.dumps(line), flush=True)
    return 0


def run_library(args):
    """--impl cutlass-mla: a library MLA decode kernel on the same workload, for comparison.

    It times vLLM's prebuilt CUTLASS sm100 MLA decode (``torch.ops._C.sm100_cutlass_mla_decode``),
    with its own split choice, on the same inputs and with the same L2 flush and event timing as
    this repository's arm.  It also reports the largest difference from ``mla_decode``'s output.
    One GPU only.  This is a measurement, not part of the decode path.
    """
    line = {"impl": "cutlass-mla", "metric": METRIC, "n_gpus": args.gpus}
    if int(os.environ.get("WORLD_SIZE", "1")) > 1 or args.gpus != 1:
        line["unavailable"] = "the library comparison runs on one GPU"
        print(json.dumps(line), flush=True)
        return 0
    cfg = CONFIGS[args.config]
    if cfg.get("layer"):
        line["unavailable"] = "the library comparison covers the decode configs (cfg2-cfg4)"
        print(json.dumps(line), flush=True)
        return 0
    import torch
    try:
        from vllm import _custom_ops as vops
    except Exception as e:  # noqa: BLE001
        line["unavailable"] = f"vllm's CUTLASS MLA op does not import: {type(e).__name__}"
        print(json.dumps(line), flush=True)
        return 0
    from triton_mla import mla_decode
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    q, kv, lens, bt = make_workload(cfg, device, seed=1000)
    B = q.shape[0]
    ours = mla_decode(q, kv, lens, bt, softmax_scale=SCALE)
    # The library's kernel works on 128-token tiles.  It is timed on the same 64-token pages
    # as this repository's arm (an even number of pages per block-table row), and on a copy
    # of the same tokens in 128-token pages (consecutive page pairs of each request), the
    # page size its fast path reads with TMA.
    if bt.shape[1] % 2:
        bt = torch.cat([bt, bt[:, :1]], dim=1).contiguous()
    kv128 = kv[bt.long()].reshape(B, -1, 2 * PAGE, D_QK).reshape(-1, 2 * PAGE, D_QK).contiguous()
    bt128 = torch.arange(kv128.shape[0], device=device, dtype=torch.int32).view(B, -1).contiguous()
    q_nope, q_pe = q[..., :D_V].contiguous(), q[..., D_V:].contiguous()
    out = torch.empty(B, 128, D_V, dtype=torch.bfloat16, device=device)
    lse = torch.empty(B, 128, dtype=torch.float32, device=device)
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    ws = torch.empty(max(vops.sm100_cutlass_mla_get_workspace_size(int(lens.max()), B, sms, -1), 1),
                     dtype=torch.uint8, device=device)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    results = {}
    for name, cache, table in (("page64", kv, bt), ("page128", kv128, bt128)):
        def step():
            vops.sm100_cutlass_mla_decode(out, lse, q_nope, q_pe, cache, lens, table, ws, SCALE, -1)

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        diff = float((out.float() - ours.float()).abs().max())
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        for i in range(args.steps):
            flush.zero_()
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        torch.cuda.synchronize()
        results[name] = (sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps, diff)
    ms, diff = min(results.values())
    total_tokens = int(lens.sum())
    tflops = decode_flops(total_tokens, 128) / (ms * 1e-3) / 1e12
    import vllm
    line.update({
        "value": tflops, "unit": "TFLOPS", "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "us_per_call": ms * 1e3, "higher_is_better": True, "dtype": "bf16", "data": "synthetic N(0,1)",
        "config": {"workload": cfg["desc"], "batch": B, "tokens": total_tokens, "num_kv_splits": "library default (-1)",
                   "l2": "flushed (256 MiB write) before every timed step"},
        "library": f"vllm {vllm.__version__} torch.ops._C.sm100_cutlass_mla_decode",
        "max_abs_diff_vs_mla_decode": diff,
        "us_per_call_by_page_size": {k: v[0] * 1e3 for k, v in results.items()},
        "max_abs_diff_by_page_size": {k: v[1] for k, v in results.items()},
    })
    print(json.dumps(line), flush=True)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="cfg2", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-gpu", "cutlass-mla"])
    ap.add_argument("--kernel", default="auto", choices=["auto", "sm100", "generic"])
    ap.add_argument("--kv-fp8", action="store_true",
                    help="an FP8 cache (656-byte rows, triton_mla.fp8_cache; CUDA-core kernel)")
    ap.add_argument("--q-len", type=int, default=1,
                    help="query tokens per request (multi-token decode, e.g. speculative / MTP); 1 = the reference's")
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of CPU oracle timing (rank 0, N=1)")
    ap.add_argument("--clock-soak", type=float, default=0.6, help="seconds of untimed steps under the clock sampler")
    ap.add_argument("--weak", action="store_true",
                    help="weak scaling for a uniform config: every rank decodes a whole batch of it "
                         "(default: the config's batch split over the ranks)")
    args = ap.parse_args(argv)
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)
    if args.impl == "cutlass-mla":
        return run_library(args)
    if args.impl == "reference-gpu":
        return run_reference_gpu(args)

    import torch
    import torch.distributed as dist
    from triton_mla import _lib, get_num_splits, make_split_plan, mla_decode
    from triton_mla.kernel import _DTYPE_CODES, _KERNELS, _status_word, selected_kernel

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    all_cpus = args.all_cpus = bind_to_gpu_cpus(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)

    cfg = CONFIGS[args.config]
    if cfg.get("layer"):
        return run_layer(args, cfg, device, world, rank, local)
    # Strong scaling by default: one global batch of the config split over the ranks
    # (contiguous slices of a uniform batch, token-balanced shards of the ragged one).  With
    # --weak every rank decodes a whole batch of a uniform config.
    strong = bool(cfg["ragged"]) or not args.weak
    if strong:
        q, kv, lens, bt, job_tokens, job_batch = make_sharded_workload(cfg, device, 1000, rank, world)
    else:
        q, kv, lens, bt = make_workload(cfg, device, seed=1000 + rank)
    B = q.shape[0]
    QL = max(1, args.q_len)
    HR = 128 * QL  # query rows per request
    total_tokens = int(lens.sum())
    # Rows attended: query token i of a request sees its first len - (QL - 1 - i) rows.
    attended = sum(max(0, int(n) - (QL - 1 - i)) for n in lens.tolist() for i in range(QL))
    if QL > 1:
        g = torch.Generator(device=device).manual_seed(2000 + rank)
        q = torch.randn(B, QL, 128, D_QK, generator=g, device=device, dtype=torch.bfloat16)
    q3 = q.view(B, HR, D_QK)
    if args.kv_fp8:
        from triton_mla import fp8_cache
        kv = fp8_cache.quantize_kv(kv)
    if not strong:
        job_tokens, job_batch = world * total_tokens, world * B
    job_flops = decode_flops(job_tokens * attended / max(total_tokens, 1), 128)
    flops = decode_flops(attended, 128)
    nbytes = decode_bytes(total_tokens, B, HR, row_bytes=656 if args.kv_fp8 else None)
    splits = get_num_splits(B, HR, int(lens.max()), torch.cuda.get_device_properties(device).multi_processor_count)
    kname = selected_kernel(q, kv, bt, num_splits=splits, kernel=args.kernel)
    # A ragged batch follows a per-request split plan, made once outside the timed region
    # (it stays valid for any lengths of the batch); uniform batches use one split count.
    plan = make_split_plan(lens, HR) if (cfg["ragged"] and kname == "sm100") else None
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)

    def step():
        return mla_decode(q, kv, lens, bt, softmax_scale=SCALE, num_splits=splits, return_lse=True,
                          kernel=args.kernel, plan=plan)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---- timed region: K steps, L2 flushed before each, events around each step.  The clock
    # sampler (nvidia-smi, 50 ms period) runs from a short soak of the same steps just before
    # the timed region to its end: the timed region alone is only a few milliseconds long.
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        t_soak = time.perf_counter()
        while time.perf_counter() - t_soak < args.clock_soak:
            for _ in range(8):
                flush.zero_()
                step()
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for i in range(args.steps):
            # A short device-side wait first keeps the GPU ahead of the host: the events then
            # bracket device work only, also when several ranks share the host's cores.
            torch.cuda._sleep(HOST_LEAD_CYCLES)
            flush.zero_()
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    ms = sum(step_ms) / len(step_ms)
    t = torch.tensor([ms], device=device)
    rank_us = [ms * 1e3]
    if world > 1:
        every = [torch.zeros(1, device=device) for _ in range(world)]
        dist.all_gather(every, t)
        rank_us = [float(x.item()) * 1e3 for x in every]
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    gpu_launches = args.steps * (1 + (1 if splits > 1 else 0))

    # ---- dominant kernel alone (stage 1 through the C ABI), same stream, same flush discipline.
    lib = _lib.load()
    lse = torch.empty(B, HR, dtype=torch.float32, device=device)
    out = torch.empty(B, HR, D_V, dtype=torch.bfloat16, device=device)
    if plan is None:
        ws = torch.empty(max(lib.tmla_workspace_bytes(B, HR, max(splits, 2), D_V), 1), dtype=torch.uint8,
                         device=device)
        o_bytes = (B * HR * max(splits, 2) * D_V * 4 + 255) & ~255
    else:
        ws = torch.empty(max(lib.tmla_units_workspace_bytes(plan.num_slots, HR, D_V), 1), dtype=torch.uint8,
                         device=device)
        o_bytes = (plan.num_slots * HR * D_V * 4 + 255) & ~255
    p = _lib.TmlaDecodeParams(
        q3.data_ptr(), q3.stride(0), q3.stride(1), kv.data_ptr(), kv.stride(0), kv.stride(1), kv.shape[0], PAGE,
        lens.data_ptr(), bt.data_ptr(), bt.stride(0), bt.shape[1], out.data_ptr(), out.stride(0), out.stride(1),
        lse.data_ptr(), lse.stride(0), ws.data_ptr(), ws.data_ptr() + o_bytes, _status_word(device).data_ptr(),
        B, HR, D_QK, D_V, splits, _DTYPE_CODES[torch.bfloat16], _KERNELS[args.kernel],
        0 if splits > 1 else _lib.FLAG_PARTIAL_ONLY, SCALE, QL,
        _lib.KV_FP8_E4M3 if args.kv_fp8 else _lib.KV_SAME)
    ks, ke = [], []
    for i in range(args.warmup + args.steps):
        torch.cuda._sleep(HOST_LEAD_CYCLES)
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        if plan is None:
            _lib.check(lib.tmla_decode_partial(ctypes.byref(p), ctypes.c_void_p(stream.cuda_stream)), "partial")
        else:  # the plan's split kernel and its merge of the split requests, through the C ABI
            _lib.check(lib.tmla_decode_units(ctypes.byref(p), plan.units.data_ptr(), plan.req_first.data_ptr(),
                                             plan.num_units, plan.num_slots, ctypes.c_void_p(stream.cuda_stream)),
                       "units")
        b.record(stream)
        if i >= args.warmup:
            ks.append(a)
            ke.append(b)
    torch.cuda.synchronize()
    kern_ms = sum(a.elapsed_time(b) for a, b in zip(ks, ke)) / len(ks)

    # ---- end to end through the public API from pinned host memory.  Each step copies its
    # inputs host->device, decodes (after an L2 flush) and copies out and lse device->host.
    # Steps are pipelined over three streams with two device input sets and two host output
    # sets: step i+1's upload and step i-1's download overlap step i's decode.  The time
    # from the first upload to the last download, over K steps, is the per-step time; the
    # unpipelined latency of one step is reported beside it.
    q_h = q.cpu().pin_memory()
    lens_h = lens.cpu().pin_memory()
    bt_h = bt.cpu().pin_memory()
    nbuf = 2
    o_shape = (B, QL, 128, D_V) if QL > 1 else (B, 128, D_V)
    out_h = [torch.empty(o_shape, dtype=torch.bfloat16).pin_memory() for _ in range(nbuf)]
    lse_h = [torch.empty(o_shape[:-1], dtype=torch.float32).pin_memory() for _ in range(nbuf)]
    h2d = q_h.numel() * 2 + lens_h.numel() * 4 + bt_h.numel() * 4
    d2h = out_h[0].numel() * 2 + lse_h[0].numel() * 4
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    q_d = [torch.empty_like(q) for _ in range(nbuf)]
    lens_d = [torch.empty_like(lens) for _ in range(nbuf)]
    bt_d = [torch.empty_like(bt) for _ in range(nbuf)]
    # The output of each buffer set is allocated once and passed as mla_decode's `out=` (the
    # host's work per step is then the copies, the flush and one mla_decode call).
    o_d = [torch.empty(o_shape, dtype=q.dtype, device=device) for _ in range(nbuf)]
    in_ready = [torch.cuda.Event() for _ in range(nbuf)]
    decoded = [torch.cuda.Event() for _ in range(nbuf)]
    downloaded = [torch.cuda.Event() for _ in range(nbuf)]

    def e2e_steps(n):
        for i in range(n):
            k = i % nbuf
            with torch.cuda.stream(s_in):
                if i >= nbuf:
                    s_in.wait_event(decoded[k])  # the decode of step i - nbuf has read buffer set k
                q_d[k].copy_(q_h, non_blocking=True)
                lens_d[k].copy_(lens_h, non_blocking=True)
                bt_d[k].copy_(bt_h, non_blocking=True)
                in_ready[k].record(s_in)
            stream.wait_event(in_ready[k])
            if i >= nbuf:
                stream.wait_event(downloaded[k])  # step i - nbuf's output has left buffer set k
            flush.zero_()
            o, l = mla_decode(q_d[k], kv, lens_d[k], bt_d[k], softmax_scale=SCALE, num_splits=splits,
                              return_lse=True, kernel=args.kernel, plan=plan, out=o_d[k])
            decoded[k].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(decoded[k])
                out_h[k].copy_(o, non_blocking=True)
                lse_h[k].copy_(l, non_blocking=True)
                downloaded[k].record(s_out)
            l.record_stream(s_out)

    e2e_steps(args.warmup)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_rounds = []
    for r in range(E2E_ROUNDS):
        if r:
            time.sleep(E2E_GAP_S)
        a.record(s_in)
        e2e_steps(args.steps)
        s_out.wait_stream(stream)
        s_out.wait_stream(s_in)
        b.record(s_out)
        torch.cuda.synchronize()
        e2e_rounds.append(a.elapsed_time(b) / args.steps)
    e2e_ms = statistics.median(e2e_rounds)
    # one step at a time (no overlap between steps), for the latency of a single call
    lat = []
    for _ in range(min(args.steps, 10)):
        flush.zero_()
        torch.cuda.synchronize()
        a.record(s_in)
        e2e_steps(1)
        s_out.wait_stream(stream)
        b.record(s_out)
        torch.cuda.synchronize()
        lat.append(a.elapsed_time(b))
    te = torch.tensor([e2e_ms, sum(lat) / len(lat)], device=device)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms, e2e_lat_ms = float(te[0].item()), float(te[1].item())

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0

    hbm, tflops_peak, peak_kind = peaks()
    achieved_gbs = nbytes / (kern_ms * 1e-3) / 1e9
    achieved_tf = flops / (kern_ms * 1e-3) / 1e12
    t_bytes = nbytes / (hbm * 1e9)
    t_flops = flops / (tflops_peak * 1e12)
    bound = "hbm" if t_bytes >= t_flops else "tensor"
    roofline = {
        "bound": bound,
        "achieved": achieved_gbs if bound == "hbm" else achieved_tf,
        "peak": hbm if bound == "hbm" else tflops_peak,
        "unit": "GB/s" if bound == "hbm" else "TFLOP/s",
        "frac": (achieved_gbs / hbm) if bound == "hbm" else (achieved_tf / tflops_peak),
        "traffic": None,
        "traffic_source": "not measured by this run (DRAM bytes come from a separate ncu capture)",
        "peak_source": f"{peak_kind} (MEASURED_PEAKS.json)" if peak_kind == "measured" else "fallback",
        "kernel": f"stage 1 ({kname})",
        "kernel_us": kern_ms * 1e3,
        "tensor_frac": achieved_tf / tflops_peak,
        "call_roofline_frac": max(t_bytes, t_flops) / (ms * 1e-3),
        "algorithmic_bytes_per_launch": nbytes,
        "algorithmic_flops_per_launch": flops,
    }
    cpu = None
    if world == 1 and args.cpu_budget > 0:
        if all_cpus:
            os.sched_setaffinity(0, all_cpus)  # the CPU baseline runs on all of the host's cores
        rate, done, el = cpu_oracle_rate(args.cpu_budget)
        cpu = {"value": rate, "unit": "TFLOPS", "cores": os.cpu_count() or 1, "kind": "port",
               "sample": f"{done} requests x 4096 tokens x 128 heads of the workload in {el:.1f}s "
                         "(numpy oracle, fp32, BLAS threads = all host cores)"}
    line = {
        "metric": METRIC,
        "value": job_flops / (ms_max * 1e-3) / 1e12,
        "unit": "TFLOPS",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_max,
        "us_per_call": ms_max * 1e3,
        "higher_is_better": True,
        "scaling": "strong" if strong else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic N(0,1) (no dataset; BASELINE configs are synthetic)",
        "config": {"workload": cfg["desc"] + (f", {QL} query tokens per request (causal)" if QL > 1 else "")
                   + (", FP8 cache rows (656 B per token)" if args.kv_fp8 else ""),
                   "q_len": QL, "kv_cache": "fp8_e4m3_656" if args.kv_fp8 else "bf16", "batch_per_gpu": B, "global_batch": job_batch, "heads": 128,
                   "page_size": PAGE, "tokens_per_job": job_tokens,
                   "tokens_per_gpu": total_tokens, "us_per_rank": rank_us,
                   "num_splits": splits if plan is None else
                   f"per-request plan: {plan.num_units} units, {plan.num_slots} partial slots",
                   "kernel": kname,
                   "l2": "flushed (256 MiB write) before every timed step",
                   "parallelism": (f"dp{world} (request shards of one global batch, own page pools)" if strong
                                   else f"dp{world} (each rank its own batch and page pool)")},
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": {"value": job_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOPS", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "latency_ms_one_step": e2e_lat_ms,
                "rounds_ms_per_step": e2e_rounds, "mean_ms_per_step": sum(e2e_rounds) / len(e2e_rounds),
                "note": "per step: q, seqlens, block_table host->device from pinned memory, L2 flush, mla_decode, "
                        "out and lse device->host; cache resident; steps pipelined over an upload, a compute "
                        "and a download stream (K steps from the first upload to the last download); "
                        f"ms_per_step is the median of {E2E_ROUNDS} such runs {E2E_GAP_S} s apart (rank 0's "
                        "rounds listed; the host link is shared with the machine's other GPUs)"},
        "gpu_launches": gpu_launches,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())

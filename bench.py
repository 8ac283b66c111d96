"""Benchmark of the headline metric: attention double backward (bwd-of-bwd) TFLOP/s.

Workload (per GPU, weak scaling): causal bf16 B4 H16 S2048 D64 -- BASELINE.json's
``configs[1]``. One step = one double-backward pass over one batch: the
query-tiled pass (D = rowsum(dO o O), dQ', ddO, dD, B) and the key-tiled pass
(dK', dV'), i.e. the work of the reference's
``dot_product_attention_bwd_rule_bwd_rule``. Credited FLOPs are
22 GEMM-equivalents x 2 x D per kept (query, key) pair (378.1 GFLOP per step).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload cfg2|cfg3|cfg4|...]

``--workload`` (default cfg2, the headline) also measures the other GPU
configurations with the same kernels: cfg3 = causal B2 H32 S8192 D128 (plus peak
device memory against the sequence length), cfg4 = non-causal B8 H16 Sq4096
Sk2048 D128, gpt = the grad-norm-penalty training step of a 12-layer GPT (tokens/s,
NCCL gradient all-reduce under torchrun), fwdbwd / fwdbwd128 = the first-order forward
and backward on the cfg2 / cfg3 shapes beside torch SDPA (cuDNN), f32 = fp32 inputs on
the cfg2 shape through the fp32-product kernels. Those lines are reported measurements,
not the headline.

Under torchrun every rank runs the workload on its own GPU (batch x heads of a
global batch 4N; no collective on the data path) and rank 0 prints one JSON line
with the aggregate over ranks (time = max over ranks).

``--impl reference`` times the reference algorithm's CPU path instead: the
reference's own CPU path (XLA on CPU) needs JAX, which is absent, so the oracle
port (torch double autograd of naive attention, fp32, all host threads) stands
in, on bounded samples of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "bwd-of-bwd TFLOP/s/GPU, causal bf16 B4 H16 S2048 D64, at 1/2/4/8 B200"
# name: (batch, heads, seq_q, seq_k, head_dim, causal)
WORKLOADS = {
    "cfg2": (4, 16, 2048, 2048, 64, True),
    "cfg3": (2, 32, 8192, 8192, 128, True),
    "cfg4": (8, 16, 4096, 2048, 128, False),
}
B, H, SQ, SK, D, CAUSAL = WORKLOADS["cfg2"]
S = SQ
SCALE = D ** -0.5


def set_workload(name):
    global B, H, SQ, SK, S, D, CAUSAL, SCALE, METRIC
    B, H, SQ, SK, D, CAUSAL = WORKLOADS[name]
    S, SCALE = SQ, D ** -0.5
    if name != "cfg2":
        METRIC = f"bwd-of-bwd TFLOP/s/GPU, {describe()}"


def set_batch(b):
    """A smaller batch of the same workload (the per-(batch, head) work is unchanged):
    the small case of an ncu capture, whose traffic scales to the full launch by B."""
    global B, METRIC
    B = b
    METRIC = f"bwd-of-bwd TFLOP/s/GPU, {describe()}"


def describe():
    seq = f"S{SQ}" if SQ == SK else f"Sq{SQ} Sk{SK}"
    return f"{'causal' if CAUSAL else 'non-causal'} bf16 B{B} H{H} {seq} D{D}"
N_SETS = 3  # rotating input sets, each larger than the 126 MB L2
PEAKS_FILE = os.path.join(ROOT, "MEASURED_PEAKS.json")
# ncu dram read + write of one query-pass launch (profiles/); cfg3 from its B1 capture
# times 2 (the batches are independent, so the traffic scales with B).
QPASS_DRAM_BYTES = {"cfg2": 212.4e6, "cfg3": 2 * (556.8e6 + 121.3e6)}
FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0}


def pairs(b, h, sq, sk, causal):
    """Kept (query, key) pairs; the causal mask is top-left (key <= query)."""
    if not causal:
        return b * h * sq * sk
    if sq <= sk:
        return b * h * sq * (sq + 1) // 2
    return b * h * (sk * (sk + 1) // 2 + (sq - sk) * sk)


def credited_flops(b, h, gemms=22):
    return gemms * 2 * D * pairs(b, h, SQ, SK, CAUSAL)


def load_peaks():
    if os.path.exists(PEAKS_FILE):
        with open(PEAKS_FILE) as f:
            p = json.load(f)
        return p, "measured"
    return FALLBACK_PEAKS, "fallback"


# ----------------------------------------------------------------------------------
# clocks
# ----------------------------------------------------------------------------------

class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", ",".join(str(g) for g in self.gpus)], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        with open(self.file.name) as f:
            rows = [[c.strip() for c in line.split(",")] for line in f if line.strip()]
        os.unlink(self.file.name)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        sm, smax, reasons, power = [], [], set(), []
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
                power.append(float(r[3]))
            except (ValueError, IndexError):
                continue
            for i, n in enumerate(names):
                if len(r) > 5 + i and r[5 + i].lower() == "active":
                    reasons.add(n)
        loaded = [c for c, p in zip(sm, power) if p > 200.0] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power) if power else None}


# ----------------------------------------------------------------------------------
# reference arm and CPU baseline (the oracle port on host cores)
# ----------------------------------------------------------------------------------

CPU_CHUNK_HEADS = 4  # heads per oracle call on the host (B1 H4 S2048 D64: ~0.6 GB of autograd graph)


class CpuWorkload:
    """The headline workload on the host: the oracle port (torch double autograd of
    naive attention, fp32, all host threads) over the whole B x H batch, a chunk of
    ``CPU_CHUNK_HEADS`` heads per call. Both the reference arm and our arm's
    ``cpu_baseline`` time this same procedure, so their rates agree."""

    def __init__(self, threads=None):
        from oracle import attention_oracle as ora

        self.ora = ora
        self.threads = threads or os.cpu_count()
        torch.set_num_threads(self.threads)
        x = ora.make_inputs(B, H, SQ, SK, D, seed=0, dtype=torch.float32)
        names = ("q", "k", "v", "do", "ddq", "ddk", "ddv")
        self.chunks = []
        for b in range(B):
            for h0 in range(0, H, CPU_CHUNK_HEADS):
                self.chunks.append([x[n][b:b + 1, :, h0:h0 + CPU_CHUNK_HEADS].contiguous() for n in names])

    def run_chunk(self, i):
        self.ora.autograd_all(*self.chunks[i % len(self.chunks)], scale=SCALE, causal=CAUSAL)

    def chunk_flops(self):
        return credited_flops(1, CPU_CHUNK_HEADS)

    def host(self):
        try:
            import cpuinfo

            name = cpuinfo.get_cpu_info().get("brand_raw", "")
        except Exception:  # noqa: BLE001 - the model name is informational
            name = ""
        return {"threads": self.threads, "logical_cpus": os.cpu_count(), "model": name}


def cpu_baseline_sample(warmup=1, steps=5):
    """Our arm's CPU baseline: ``steps`` chunks of the workload (after ``warmup``
    chunks), median chunk time, as a rate over the chunk's credited FLOPs."""
    w = CpuWorkload()
    for i in range(warmup):
        w.run_chunk(i)
    times = []
    for i in range(steps):
        t0 = time.perf_counter()
        w.run_chunk(warmup + i)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": w.chunk_flops() / t / 1e12, "unit": "TFLOP/s", "cores": w.threads, "kind": "port",
            "host": w.host(),
            "sample": f"{steps} chunks of {CPU_CHUNK_HEADS} heads (B1 H{CPU_CHUNK_HEADS} S{S} D{D} causal fp32, torch "
                      f"double autograd of naive attention; {B * H // CPU_CHUNK_HEADS} chunks make the full "
                      f"workload) after {warmup} warm-up chunk(s), median chunk time"}


def run_reference(args):
    """The reference algorithm's CPU path on the full workload: every step runs all
    B x H heads (chunk by chunk); rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    w = CpuWorkload()
    n_chunks = len(w.chunks)
    for i in range(args.warmup):
        w.run_chunk(i)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        for c in range(n_chunks):
            w.run_chunk(c)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    value = credited_flops(B, H) / t / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"bwdbwd {describe()} per GPU", "name": args.workload,
                   "reference_sample": f"the full B{B} H{H} batch every step, {n_chunks} chunks of "
                                       f"{CPU_CHUNK_HEADS} heads",
                   "reference_path": "oracle port: torch CPU double autograd (the reference's XLA CPU path needs "
                                     "JAX, absent)",
                   "warmup_unit": "chunks", "step_time": "median over steps"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": w.threads, "kind": "port", "host": w.host(),
                         "sample": f"the full workload per step ({n_chunks} chunks of {CPU_CHUNK_HEADS} heads)"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------------
# our arm
# ----------------------------------------------------------------------------------

# Workloads whose global batch is fixed and sharded over the ranks (strong scaling):
# configuration 4 is "sharded over batch x heads across 1/2/4/8 GPUs".
STRONG = {"cfg4"}


def make_set(seed, device, shard=None, rank=0):
    """One input set on the device. With ``shard`` (a BatchHeadsSharding) the set is
    this rank's slice of the global batch drawn from ``seed``; otherwise the whole
    B x H batch is this rank's own."""
    from flash_hog_b200 import MaskType
    from flash_hog_b200 import _attention_impl as impl
    from oracle.attention_oracle import make_inputs

    x = make_inputs(B, H, SQ, SK, D, seed=seed)
    if shard is not None:
        x = {k: (shard.shard(v, rank) if k in ("q", "do", "ddq") else shard.shard_kv(v, rank)).contiguous()
             for k, v in x.items()}
    g = {k: v.to(device) for k, v in x.items()}
    mask = MaskType.CAUSAL if CAUSAL else MaskType.NO_MASK
    o, lse = impl.cuda_dot_product_attention(g["q"], g["k"], g["v"], mask, SCALE, return_residual=True)
    g["o"], g["lse"] = o, lse
    return g


def memory_vs_seq(dev, seqs=(1024, 2048, 4096, 8192)):
    """Device memory of one double backward (inputs + outputs + scratch) against the
    sequence length, at the workload's batch, heads and head_dim: linear in S since
    no (Sq, Sk) array is ever allocated."""
    from flash_hog_b200 import MaskType, flash_bwdbwd

    rows = []
    for s in seqs:
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        base = torch.cuda.memory_allocated(dev)
        torch.cuda.reset_peak_memory_stats(dev)
        g = torch.Generator(device="cpu").manual_seed(s)
        shape = (B, s, H, D)
        x = [torch.randn(shape, generator=g).to(dev, torch.bfloat16) for _ in range(8)]
        lse = torch.randn((B, H, s), generator=g).to(dev) + 8.0
        flash_bwdbwd(*x, lse, mask_type=MaskType.CAUSAL if CAUSAL else MaskType.NO_MASK, scale=SCALE)
        torch.cuda.synchronize()
        rows.append({"seq_len": s, "peak_bytes": torch.cuda.max_memory_allocated(dev) - base,
                     "input_bytes": sum(t.numel() * t.element_size() for t in x) + lse.numel() * 4})
        del x, lse
    return rows


def run_gpt(args):
    """The grad-norm-penalty GPT training step (12 layers, d768, 12 heads of 64, MLP
    3072, vocab 32000, sequence 1024, 4 sequences per GPU; tokens uniform in
    [0, 32000)), data-parallel over the ranks with an NCCL gradient all-reduce.
    Metric: tokens per second of the whole job.

    ``value``: attention, LayerNorm and GELU on this package's kernels (first- and
    second-order), the step's compute replayed as one CUDA graph (PenaltyStepGraph),
    then the NCCL all-reduce and the SGD update. ``baseline_torch_autograd``: the same
    model with torch's LayerNorm and GELU and eager launches (attention still on the
    kernels), timed the same way on the same GPUs."""
    import datetime
    from flash_hog_b200 import _capi
    from flash_hog_b200.gpt import GPT, GPTConfig, PenaltyStepGraph, train_step

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        pin_host_cores(local, local_world)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    distributed = dist is not None
    cfg, batch, lam = GPTConfig(), 4, 1e-2
    g = torch.Generator().manual_seed(1000 + rank)
    host = [torch.randint(0, cfg.vocab, (batch, cfg.seq_len + 1), generator=g).pin_memory() for _ in range(2)]
    resident = [t.to(dev) for t in host]

    def make(fused):
        torch.manual_seed(0)  # the same initial weights on every rank
        model = GPT(cfg, fused=fused).to(dev)
        return model, torch.optim.SGD(model.parameters(), lr=1e-4)

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local])

    def timed(step_fn, steps):
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n0 = _capi.launch_count()
        e0.record()
        for i in range(steps):
            step_fn(i)
        e1.record()
        torch.cuda.synchronize()
        barrier()
        ms = e0.elapsed_time(e1) / steps
        if dist is not None:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms, _capi.launch_count() - n0

    # Baseline: torch LayerNorm/GELU, eager launches.
    base_model, base_opt = make(False)
    base_step = lambda i: train_step(base_model, resident[i % 2], lam, optimizer=base_opt, distributed=distributed)
    for i in range(args.warmup):
        base_step(i)
    base_ms, _ = timed(base_step, max(3, min(args.steps, 10)))
    del base_model, base_opt
    torch.cuda.empty_cache()

    # Ours: fused kernels, the step's compute replayed as a CUDA graph.
    model, opt = make(True)
    graph = PenaltyStepGraph(model, batch, lam, warmup=args.warmup)
    device_step = lambda i: graph.step(resident[i % 2], optimizer=opt, distributed=distributed)
    with ClockSampler(list(range(world)) if rank == 0 else []) as clocks:
        ms, _ = timed(device_step, args.steps)
    launches = graph.kernels_per_step * args.steps  # replays do not pass through the C ABI's counter
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()

    def e2e_step(i):
        tokens = host[i % 2].to(dev, non_blocking=True)
        loss, _ = graph.step(tokens, optimizer=opt, distributed=distributed)
        loss_host.copy_(loss, non_blocking=True)

    e2e_ms, _ = timed(e2e_step, max(3, min(args.steps, 10)))
    if _capi.device_status() != 0:
        raise RuntimeError("device-side error in the GPT step")
    peak = torch.cuda.max_memory_allocated(dev)
    del graph
    if dist is not None:
        dist.destroy_process_group()
    if rank != 0:
        return 0
    tokens_step = world * batch * cfg.seq_len
    print(json.dumps({
        "metric": "grad-norm-penalty GPT training step, tokens/s (12L d768 h12 D64 causal, seq 1024, 4 seq/GPU)",
        "value": tokens_step / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (tokens uniform in [0, 32000), random init)",
        "value_per_gpu": tokens_step / world / (ms * 1e-3),
        "config": {"workload": "gpt grad-norm penalty L + 0.01 ||dL/dtheta||^2, SGD update", "name": "gpt",
                   "layers": cfg.n_layer, "d_model": cfg.d_model, "heads": cfg.n_head, "seq_len": cfg.seq_len,
                   "global_batch": world * batch, "parallelism": f"dp{world} (NCCL all-reduce of gradients)",
                   "step": "fused LayerNorm/GELU kernels, compute replayed as one CUDA graph, then all-reduce + SGD",
                   "peak_device_bytes": peak},
        "baseline_torch_autograd": {"tokens_per_s": tokens_step / (base_ms * 1e-3), "ms_per_step": base_ms,
                                    "step": "torch LayerNorm/GELU autograd, eager launches (attention on the "
                                            "kernels)"},
        "roofline": None, "cpu_baseline": None,
        "e2e": {"value": tokens_step / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": host[0].numel() * host[0].element_size(), "d2h_bytes_per_step": 4},
        "clocks": clocks.summary(), "gpu_launches": launches,
    }), flush=True)
    return 0


def run_fwdbwd(args):
    """Diagnostic line, not the headline: the first-order forward and backward on the
    cfg2 (``fwdbwd``) or cfg3 (``fwdbwd128``) shapes, beside torch's SDPA (cuDNN on
    B200) on the same inputs -- the kernels the reference calls for these two rules
    (flash_hog/jax/_attention_impl.py:224-261). Credited work: forward 2 and backward
    5 GEMM-equivalents per kept pair; one step = forward + backward. 1 GPU."""
    import torch.nn.functional as F
    from flash_hog_b200 import _capi

    set_workload("cfg2" if args.workload == "fwdbwd" else "cfg3")
    dev = torch.device("cuda", 0)
    sets = [make_set(i, dev) for i in range(N_SETS)]
    outs = [(torch.empty_like(x["q"]), torch.empty((B, H, SQ), dtype=torch.float32, device=dev),
             torch.empty_like(x["q"]), torch.empty_like(x["k"]), torch.empty_like(x["k"]),
             torch.empty((B, H, SQ), dtype=torch.float32, device=dev)) for x in sets]

    def ours(i, ev):
        x, (o, lse, dq, dk, dv, delta) = sets[i % N_SETS], outs[i % N_SETS]
        ev[0].record()
        _capi.attn_fwd(x["q"], x["k"], x["v"], o, lse, SCALE, CAUSAL)
        ev[1].record()
        _capi.attn_bwd(x["q"], x["k"], x["v"], o, x["do"], lse, dq, dk, dv, delta, SCALE, CAUSAL)
        ev[2].record()

    bhtd = [{n: x[n].transpose(1, 2) for n in ("q", "k", "v", "do")} for x in sets]

    def sdpa(i, ev):
        x = bhtd[i % N_SETS]
        q, k, v = (x[n].detach().requires_grad_(True) for n in ("q", "k", "v"))
        ev[0].record()
        out = F.scaled_dot_product_attention(q, k, v, is_causal=CAUSAL, scale=SCALE)
        ev[1].record()
        torch.autograd.grad(out, (q, k, v), x["do"])
        ev[2].record()

    def timed(fn, steps):
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
        for i in range(args.warmup):
            fn(i, evs[0])
        torch.cuda.synchronize()
        n0 = _capi.launch_count()
        for i in range(steps):
            fn(i, evs[i])
        torch.cuda.synchronize()
        f = statistics.median(e[0].elapsed_time(e[1]) for e in evs)
        b = statistics.median(e[1].elapsed_time(e[2]) for e in evs)
        return f, b, _capi.launch_count() - n0

    with ClockSampler([0]) as clocks:
        f, b, launches = timed(ours, args.steps)
    fs, bs, _ = timed(sdpa, args.steps)
    if _capi.device_status() != 0:
        raise RuntimeError("device-side error in the forward/backward")
    p = pairs(B, H, SQ, SK, CAUSAL)
    tf = lambda gemms, ms: gemms * 2 * D * p / (ms * 1e-3) / 1e12
    print(json.dumps({
        "metric": f"attention forward + backward TFLOP/s ({describe()})", "value": tf(7, f + b),
        "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": f + b,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"fwd + bwd {describe()}", "name": args.workload, "l2": "3 rotating input sets",
                   "credited_gemm_eq": {"fwd": 2, "bwd": 5}},
        "fwd": {"ms": f, "tflops": tf(2, f)}, "bwd": {"ms": b, "tflops": tf(5, b)},
        "torch_sdpa": {"fwd_ms": fs, "fwd_tflops": tf(2, fs), "bwd_ms": bs, "bwd_tflops": tf(5, bs)},
        "roofline": None, "cpu_baseline": None, "e2e": None, "clocks": clocks.summary(), "gpu_launches": launches,
    }), flush=True)
    return 0


FP32_FMA_TFLOPS_NOMINAL = 148 * 128 * 2 * 1.965e9 / 1e12  # SMs x fp32 lanes x 2 x max SM clock


def run_f32(args):
    """Diagnostic line, not the headline: fp32 inputs on the cfg2 shape (causal
    B4 H16 S2048 D64) through the fp32-product kernels -- forward, backward and
    double backward per step, each timed with CUDA events -- beside torch's SDPA
    on the same fp32 inputs for the forward and backward. Roofline: the CUDA cores'
    fp32 FMA rate (nominal; no measured figure exists for it). 1 GPU."""
    import torch.nn.functional as F
    from flash_hog_b200 import _capi
    from oracle.attention_oracle import make_inputs

    set_workload("cfg2")
    dev = torch.device("cuda", 0)
    sets = []
    for i in range(N_SETS):
        x = {k: v.to(dev) for k, v in make_inputs(B, H, SQ, SK, D, seed=i, dtype=torch.float32).items()}
        x["o"], x["lse"] = torch.empty_like(x["q"]), torch.empty((B, H, SQ), dtype=torch.float32, device=dev)
        x["out"] = [torch.empty_like(x[n]) for n in ("q", "k", "v", "q", "k", "v", "q")]
        x["stats"] = torch.empty((3, B, H, SQ), dtype=torch.float32, device=dev)
        sets.append(x)

    def ours(i, ev):
        x = sets[i % N_SETS]
        dq, dk, dv, dq2, dk2, dv2, ddo = x["out"]
        st = x["stats"]
        ev[0].record()
        _capi.attn_fwd_f32(x["q"], x["k"], x["v"], x["o"], x["lse"], SCALE, CAUSAL)
        ev[1].record()
        _capi.attn_bwd_f32(x["q"], x["k"], x["v"], x["o"], x["do"], x["lse"], dq, dk, dv, st[0], SCALE, CAUSAL)
        ev[2].record()
        _capi.attn_bwdbwd_f32(x["q"], x["k"], x["v"], x["o"], x["do"], x["ddq"], x["ddk"], x["ddv"], x["lse"], dq2,
                              ddo, dk2, dv2, st[0], st[1], st[2], SCALE, CAUSAL)
        ev[3].record()

    bhtd = [{n: x[n].transpose(1, 2) for n in ("q", "k", "v", "do")} for x in sets]

    def sdpa(i, ev):
        x = bhtd[i % N_SETS]
        q, k, v = (x[n].detach().requires_grad_(True) for n in ("q", "k", "v"))
        ev[0].record()
        out = F.scaled_dot_product_attention(q, k, v, is_causal=CAUSAL, scale=SCALE)
        ev[1].record()
        torch.autograd.grad(out, (q, k, v), x["do"])
        ev[2].record()
        ev[3].record()

    def timed(fn, steps):
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(steps)]
        for i in range(args.warmup):
            fn(i, evs[0])
        torch.cuda.synchronize()
        n0 = _capi.launch_count()
        for i in range(steps):
            fn(i, evs[i])
        torch.cuda.synchronize()
        return [statistics.median(e[j].elapsed_time(e[j + 1]) for e in evs) for j in range(3)], \
            _capi.launch_count() - n0

    with ClockSampler([0]) as clocks:
        (f, b, bb), launches = timed(ours, args.steps)
    (fs, bs, _), _ = timed(sdpa, args.steps)
    p = pairs(B, H, SQ, SK, CAUSAL)
    tf = lambda gemms, ms: gemms * 2 * D * p / (ms * 1e-3) / 1e12
    print(json.dumps({
        "metric": f"attention double backward TFLOP/s, fp32 inputs ({describe().replace('bf16', 'fp32')})",
        "value": tf(22, bb), "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": f + b + bb, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": f"fwd + bwd + bwdbwd {describe().replace('bf16', 'fp32')}", "name": "f32",
                   "l2": "3 rotating input sets of ~270 MB each", "credited_gemm_eq": {"fwd": 2, "bwd": 5, "bwdbwd": 22}},
        "fwd": {"ms": f, "tflops": tf(2, f)}, "bwd": {"ms": b, "tflops": tf(5, b)},
        "bwdbwd": {"ms": bb, "tflops": tf(22, bb)},
        "torch_sdpa_fp32": {"fwd_ms": fs, "fwd_tflops": tf(2, fs), "bwd_ms": bs, "bwd_tflops": tf(5, bs)},
        "roofline": {"bound": "fp32 FMA (CUDA cores)", "achieved": tf(22, bb), "peak": FP32_FMA_TFLOPS_NOMINAL,
                     "unit": "TFLOP/s", "frac": tf(22, bb) / FP32_FMA_TFLOPS_NOMINAL,
                     "peak_source": "nominal: 148 SMs x 128 lanes x 2 x 1.965 GHz", "traffic": None},
        "cpu_baseline": None, "e2e": None, "clocks": clocks.summary(), "gpu_launches": launches,
    }), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--skip-e2e", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["gpt", "fwdbwd", "fwdbwd128", "f32"], default="cfg2")
    ap.add_argument("--batch", type=int, default=None,
                    help="double-backward workloads: a smaller batch (a small case for ncu captures)")
    args = ap.parse_args()
    if args.workload in ("fwdbwd", "fwdbwd128"):
        args.warmup = max(args.warmup, 3)
        return run_fwdbwd(args)
    if args.workload == "f32":
        args.warmup = max(args.warmup, 3)
        return run_f32(args)
    if args.workload == "gpt":
        if args.warmup < 3:
            args.warmup = 3
        return run_gpt(args)
    set_workload(args.workload)
    if args.batch:
        set_batch(args.batch)
    if args.workload != "cfg2" or args.batch:
        args.skip_cpu = True  # the CPU baseline samples the headline workload only
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)

    return run_ours(args)


def pin_host_cores(local, local_world):
    """Restricts this rank's host threads to its share of its GPU's CPU affinity set
    (NVML), so ranks do not contend for cores and pinned buffers are first touched on
    the GPU's NUMA node. Returns the cores used (None if NVML is unavailable)."""
    try:
        import pynvml

        pynvml.nvmlInit()
        hdl = pynvml.nvmlDeviceGetHandleByIndex(torch.cuda.current_device())
        words = pynvml.nvmlDeviceGetCpuAffinity(hdl, (os.cpu_count() + 63) // 64)
        pynvml.nvmlShutdown()
    except Exception:  # noqa: BLE001 - affinity is an optimisation, not a requirement
        return None
    cpus = [64 * w + b for w, word in enumerate(words) for b in range(64) if (word >> b) & 1]
    cpus = [c for c in cpus if c in os.sched_getaffinity(0)]
    if len(cpus) < local_world:
        return None
    share = len(cpus) // local_world
    mine = cpus[local * share:(local + 1) * share]
    os.sched_setaffinity(0, mine)
    torch.set_num_threads(max(1, len(mine)))
    return mine


def e2e_sharded(args, dev, rank, world, barrier, gather, sharded_flash_bwdbwd, MaskType):
    """End to end through ``sharded_flash_bwdbwd`` for a strong-scaling workload: every
    rank holds the same global batch in pinned host memory; each step, each rank copies
    its slice to its GPU, runs the kernels and copies its results back to pinned host
    buffers (one step after another on one stream)."""
    from oracle.attention_oracle import make_inputs

    from flash_hog_b200 import _attention_impl as impl

    x = make_inputs(B, H, SQ, SK, D, seed=0)
    mask = MaskType.CAUSAL if CAUSAL else MaskType.NO_MASK
    o, lse = impl.cuda_dot_product_attention(x["q"].to(dev), x["k"].to(dev), x["v"].to(dev), mask, SCALE,
                                             return_residual=True)  # the global forward, once
    host = [t.cpu().pin_memory() for t in (x["q"], x["k"], x["v"], o, x["do"], x["ddq"], x["ddk"], x["ddv"], lse)]
    del o, lse
    local, sh = sharded_flash_bwdbwd(*host, mask_type=mask, scale=SCALE, rank=rank, world=world, device=dev)
    res_host = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in local]
    sb, hs = sh.slices(rank)
    h2d = sum(t[sb].numel() * t.element_size() for t in host) // (1 if sh.head_parts == 1 else sh.head_parts)
    d2h = sum(t.numel() * t.element_size() for t in res_host)

    def step():
        r, _ = sharded_flash_bwdbwd(*host, mask_type=mask, scale=SCALE, rank=rank, world=world, device=dev)
        for dst, src in zip(res_host, r):
            dst.copy_(src, non_blocking=True)

    for _ in range(2):
        step()
    n = max(3, min(args.steps, 10))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(n):
        step()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    ms = max(r[0] for r in gather([e0.elapsed_time(e1) / n]))
    flops = credited_flops(B, H)
    return {"value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "value_per_gpu": flops / world / (ms * 1e-3) / 1e12,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": ms,
            "api": "flash_hog_b200.sharding.sharded_flash_bwdbwd (global batch in pinned host memory)",
            "pipeline": "one stream: slice upload, kernels, result download per step"}


def run_ours(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cores = pin_host_cores(local, local_world) if world > 1 else None
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    from flash_hog_b200 import _capi
    from flash_hog_b200 import flash_bwdbwd, MaskType
    from flash_hog_b200.sharding import BatchHeadsSharding, sharded_flash_bwdbwd

    strong = args.workload in STRONG
    shard = BatchHeadsSharding(B, H, world) if strong else None
    # Weak scaling: rank r holds its own B x H batch (rows [B r, B r + B) of a global
    # batch B N): distinct seeds. Strong scaling: every rank draws the same global batch
    # and keeps its batch x heads slice.
    sets = [make_set(i if strong else 1000 * rank + i, dev, shard, rank) for i in range(N_SETS)]
    b_loc, h_loc = sets[0]["q"].shape[0], sets[0]["q"].shape[2]
    flops_rank = credited_flops(b_loc, h_loc)  # this rank's credited FLOPs per step
    flops_job = credited_flops(B, H) if strong else world * credited_flops(B, H)
    stats = torch.empty((N_SETS, 3, b_loc, h_loc, SQ), dtype=torch.float32, device=dev)
    outs = [(torch.empty_like(s["q"]), torch.empty_like(s["q"]), torch.empty_like(s["k"]), torch.empty_like(s["k"]))
            for s in sets]

    def launch(i, ev=None):
        s, (dq2, ddo, dk2, dv2), st = sets[i], outs[i], stats[i]
        if ev is not None:
            ev[0].record()
        _capi.attn_bwdbwd_o(s["q"], s["k"], s["v"], s["o"], s["do"], s["ddq"], s["ddk"], s["ddv"], s["lse"],
                            dq2, ddo, dk2, dv2, st[0], st[1], st[2], SCALE, CAUSAL, _capi.PASS_QUERY)
        if ev is not None:
            ev[1].record()
        _capi.attn_bwdbwd_o(s["q"], s["k"], s["v"], s["o"], s["do"], s["ddq"], s["ddk"], s["ddv"], s["lse"],
                            dq2, ddo, dk2, dv2, st[0], st[1], st[2], SCALE, CAUSAL, _capi.PASS_KEY)
        if ev is not None:
            ev[2].record()

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local])

    def gather(vals):
        """Every rank's floats (rank order) on every rank."""
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        if dist is None:
            return [t.tolist()]
        out = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(out, t)
        return [o.tolist() for o in out]

    for i in range(args.warmup):
        launch(i % N_SETS)
    torch.cuda.synchronize()
    if _capi.device_status() != 0:
        raise RuntimeError("device-side error during warm-up")

    # Per-pass times, eagerly launched with events between the passes (not the timed region).
    n_eager = max(args.steps, 20)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(n_eager)]
    for i in range(n_eager):
        launch(i % N_SETS, evs[i])
    torch.cuda.synchronize()
    t_q = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    t_k = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    eager_ms = evs[0][0].elapsed_time(evs[-1][2]) / n_eager

    # The timed region: the K steps captured once as a CUDA graph and replayed, so the
    # host's launch timing (Python, ctypes, several ranks sharing host cores) cannot
    # leave a GPU idle between steps. The graph holds exactly the 2K kernel launches.
    graph, launches = None, 0
    try:
        cap = torch.cuda.Stream(dev)
        cap.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        n0 = _capi.launch_count()
        with torch.cuda.graph(graph, stream=cap, capture_error_mode="relaxed"):
            for i in range(args.steps):
                launch(i % N_SETS)
        launches = _capi.launch_count() - n0
        graph.replay()  # one untimed replay: the graph's first launch uploads it
        torch.cuda.synchronize()
    except Exception as e:  # noqa: BLE001 - fall back to eager launches, recorded in the line
        graph = None
        print(f"bench: CUDA graph capture failed ({e}); timing eager launches", file=sys.stderr)

    def timed_region():
        nonlocal launches
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        start.record()
        if graph is not None:
            graph.replay()
        else:
            n0 = _capi.launch_count()
            for i in range(args.steps):
                launch(i % N_SETS)
            launches = _capi.launch_count() - n0
        stop.record()
        torch.cuda.synchronize()
        barrier()
        return start.elapsed_time(stop) / args.steps

    with ClockSampler(list(range(world)) if rank == 0 else []) as clocks:
        ms_rank = timed_region()
    if _capi.device_status() != 0:
        raise RuntimeError("device-side error during the timed region")
    # Stability check outside the timed region: the same region again until >= 200 steps.
    reps = max(1, -(-200 // args.steps))
    long_ms = statistics.mean(timed_region() for _ in range(reps))
    peak_bytes = torch.cuda.max_memory_allocated(dev)
    per_rank = gather([ms_rank, long_ms, eager_ms, t_q, t_k])
    ms = max(r[0] for r in per_rank)

    # end to end through the public API, host buffers, copies inside the timed region.
    # Steps are pipelined the way a serving loop would run them: step i's inputs go
    # up on a copy stream while step i-1 computes and step i-2's results come down
    # on another (device inputs double-buffered); every step still copies all its
    # inputs host -> device and all its results device -> host inside the region.
    e2e = None
    if not args.skip_e2e and strong:
        e2e = e2e_sharded(args, dev, rank, world, barrier, gather, sharded_flash_bwdbwd, MaskType)
    elif not args.skip_e2e:
        host = {k: v.cpu().pin_memory() for k, v in sets[0].items()}
        names = ("q", "k", "v", "o", "do", "ddq", "ddk", "ddv", "lse")
        h2d = sum(host[n].numel() * host[n].element_size() for n in names)
        # flash_bwdbwd returns (dQ2, dK2, dV2, ddO)
        res_host = [[torch.empty(host[n].shape, dtype=torch.bfloat16).pin_memory() for n in ("q", "k", "k", "q")]
                    for _ in range(2)]
        d2h = sum(t.numel() * t.element_size() for t in res_host[0])
        compute = torch.cuda.current_stream(dev)
        copy_in, copy_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        dev_in = [{n: torch.empty_like(sets[0][n]) for n in names} for _ in range(2)]
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_done = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]
        for e in ev_done + ev_out:
            e.record(compute)

        def e2e_step(i):
            slot = i % 2
            with torch.cuda.stream(copy_in):
                copy_in.wait_event(ev_done[slot])  # the slot's previous step has read its inputs
                for n in names:
                    dev_in[slot][n].copy_(host[n], non_blocking=True)
                ev_in[slot].record(copy_in)
            compute.wait_event(ev_in[slot])
            d = dev_in[slot]
            r = flash_bwdbwd(d["q"], d["k"], d["v"], d["o"], d["do"], d["ddq"], d["ddk"], d["ddv"], d["lse"],
                             mask_type=MaskType.CAUSAL if CAUSAL else MaskType.NO_MASK, scale=SCALE)
            ev_done[slot].record(compute)
            with torch.cuda.stream(copy_out):
                copy_out.wait_event(ev_done[slot])
                copy_out.wait_event(ev_out[slot])  # the slot's host result buffers are free
                for dst, src in zip(res_host[slot], r):
                    src.record_stream(copy_out)
                    dst.copy_(src, non_blocking=True)
                ev_out[slot].record(copy_out)

        for i in range(3):
            e2e_step(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_e2e = max(3, args.steps)  # the same K steps as the kernel-only timing
        barrier()
        torch.cuda.synchronize()
        e0.record(compute)
        copy_in.wait_stream(compute)  # the first upload starts inside the timed region
        for i in range(n_e2e):
            e2e_step(i)
        compute.wait_event(ev_out[(n_e2e - 1) % 2])  # the last results are on the host
        e1.record(compute)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = e0.elapsed_time(e1) / n_e2e

        # The host links alone, all ranks at once: one step's inputs up, then its results
        # down (outside the timed region; attributes the e2e bound to a link).
        def link_gbs(copy_fn, nbytes, reps=5):
            a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            barrier()
            torch.cuda.synchronize()
            a.record()
            for _ in range(reps):
                copy_fn()
            b_.record()
            torch.cuda.synchronize()
            return reps * nbytes / (a.elapsed_time(b_) * 1e-3) / 1e9

        h2d_gbs = link_gbs(lambda: [dev_in[0][n].copy_(host[n], non_blocking=True) for n in names], h2d)
        d2h_gbs = link_gbs(lambda: [dst.copy_(src, non_blocking=True) for dst, src in zip(res_host[0], outs[0])],
                           d2h)
        pinned = all(t.is_pinned() for t in list(host.values()) + [x for r in res_host for x in r])
        e2e_rank = gather([e2e_ms, h2d_gbs, d2h_gbs, 1.0 if pinned else 0.0])
        e2e_ms = max(r[0] for r in e2e_rank)
        e2e = {"value": flops_job / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
               "value_per_gpu": flops_job / world / (e2e_ms * 1e-3) / 1e12,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
               "host_buffers_pinned": all(r[3] > 0.5 for r in e2e_rank),
               "per_rank": [{"rank": i, "ms_per_step": r[0], "h2d_gbs_alone": r[1], "d2h_gbs_alone": r[2]}
                            for i, r in enumerate(e2e_rank)],
               "host_links_gbs_aggregate": {"h2d": sum(r[1] for r in e2e_rank),
                                            "d2h": sum(r[2] for r in e2e_rank)},
               "api": "flash_hog_b200.flash_bwdbwd",
               "pipeline": "copy-in, compute and copy-out streams; device inputs double-buffered"}

    mem_rows = memory_vs_seq(dev) if args.workload == "cfg3" and rank == 0 else None
    graphed = graph is not None
    del graph
    if dist is not None:
        dist.destroy_process_group()
    if rank != 0:
        return 0

    peaks, peak_kind = load_peaks()
    flops_q = credited_flops(b_loc, h_loc, gemms=14)
    achieved = flops_q / (t_q * 1e-3) / 1e12
    roofline = {"bound": "tensor", "kernel": "bwdbwd_q_kernel (query-tiled pass, 14 of 22 GEMM-eq)",
                "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": achieved / peaks["bf16_tflops"], "peak_source": f"{peak_kind} bf16 dense (burst)",
                # dram__bytes_read.sum + dram__bytes_write.sum of one query-pass launch of this
                # workload, from the ncu capture summarised in profiles/bwdbwd_b4h16s2048d64_causal.md
                "traffic": QPASS_DRAM_BYTES.get(args.workload) if not args.batch else None,
                "traffic_unit": "bytes per launch (ncu)",
                "per_launch_ms": {"query_pass": t_q, "key_pass": t_k},
                "key_pass": {"achieved": credited_flops(b_loc, h_loc, gemms=8) / (t_k * 1e-3) / 1e12,
                             "frac": credited_flops(b_loc, h_loc, gemms=8) / (t_k * 1e-3) / 1e12
                             / peaks["bf16_tflops"]},
                "step": {"achieved": flops_rank / (ms * 1e-3) / 1e12,
                         "frac_of_sustained": flops_rank / (ms * 1e-3) / 1e12
                         / peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])}}
    cpu = None
    if not args.skip_cpu and world == 1:  # the CPU baseline is reported at N=1 only
        cpu = cpu_baseline_sample()
    value = flops_job / (ms * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong" if strong else "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "value_per_gpu": value / world,
        "config": {"workload": (f"bwdbwd {describe()} sharded over the ranks" if strong
                                else f"bwdbwd {describe()} per GPU"), "name": args.workload,
                   "value": "aggregate over all n_gpus ranks (value_per_gpu = value / n_gpus)",
                   "global_batch": B if strong else B * world, "heads": H, "seq_len": SQ, "seq_len_k": SK,
                   "head_dim": D, "causal": CAUSAL, "per_rank_slice": {"batch": b_loc, "heads": h_loc},
                   "parallelism": f"dp{world} (batch x heads sharded, no collective)",
                   "l2": f"{N_SETS} rotating input sets of ~136 MB each (> 126 MB L2)",
                   "timed_region": ("the K steps as one CUDA graph (2K kernel launches), replayed once"
                                    if graphed else "K steps launched eagerly"),
                   "credited_gflop_per_step_per_gpu": flops_rank / 1e9,
                   "peak_device_bytes": peak_bytes},
        "per_rank": [{"rank": i, "ms_per_step": r[0], "ms_per_step_200": r[1], "ms_per_step_eager": r[2],
                      "query_pass_ms": r[3], "key_pass_ms": r[4]} for i, r in enumerate(per_rank)],
        "host_cores_per_rank": len(cores) if cores else None,
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks.summary(),
        **({"memory_vs_seq": mem_rows} if mem_rows else {}),
        "gpu_launches": launches,  # counted by the library (fh_launch_count) for the timed region's launches
    }
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())

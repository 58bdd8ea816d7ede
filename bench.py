"""Benchmark of the B200 QLoRA path: train-step tokens/s (headline), fused CE, memory-bound ops.

Default line (``python bench.py --gpus N --steps K --warmup W``): the
Qwen2.5-1.5B-architecture QLoRA train step, data parallel over the N ranks
(one process per GPU, torchrun). Per GPU: batch 4 x 2048 tokens of uniform
random ids (weak scaling: the per-GPU batch is the same at every N), 28
decoder layers with NF4 (blocksize 64) base weights, LoRA r16 / alpha 32 on
q/k/v/o/gate/up/down, the fused RMSNorm / RoPE / SwiGLU / head-CE ops, AdamW
2e-4, and with N > 1 one NCCL all-reduce of the flat 73.9 MB LoRA gradient
per step. The whole step (forward, backward, all-reduce, AdamW) is one CUDA
graph replay. The MLP keeps [g | u] for its backward (the reference recomputes it
to save memory; the results are bit-identical, ``--recompute`` restores it).

* ``value``: tokens/s of all ranks, device-resident ids, CUDA events around
  exactly K replays (barrier + synchronize on both sides, max over ranks).
* ``e2e``: the same step with the ids and labels copied from pinned host
  memory and the loss read back every step, inside the timed region.
* ``roofline``: the step's dominant kernel, the gate/up GEMM with the SwiGLU
  epilogue (2 launches per layer), timed live by CUDA events on its stream at
  the step's shape; ``step_mfu``: algorithmic FLOPs per token (formula in
  ``oracle.qlora_step.train_flop_per_token``) x tokens/s per GPU over the
  measured sustained bf16 peak.
* ``allreduce``: the gradient all-reduce alone (N > 1), CUDA events.
* nested results of the same run: ``ce`` (fused head CE fwd+bwd TFLOP/s on
  2048 tokens per rank, with its e2e, roofline, stages and a sustained run),
  ``mem_ops`` (RMSNorm / SwiGLU / RoPE fwd+bwd HBM GB/s at the benchmark
  shapes), ``ce_vp`` (vocab-parallel CE on 65536 tokens, strong scaling over
  the N ranks, with its collective / compute split) and, at N = 1,
  ``qlora_s512`` (the 1-GPU configuration: batch 4 x 512).
* ``cpu_baseline`` (rank 0, N = 1): the reference's eager formulation of the
  step on the host cores (``oracle.qlora_step``) on a bounded sample,
  normalised by algorithmic FLOPs per token to the benchmark configuration.

``--impl reference`` times only that CPU step and prints its own line.
``--workload ce|rmsnorm|swiglu|rope|qlora|ce_vp`` prints one section alone.
"""

from __future__ import annotations

import argparse
import gc
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402

# fused head CE workload
N_TOK, DIM, VOCAB, CHUNK = 2048, 1536, 151936, 32
FLOP_PER_GEMM = 2.0 * N_TOK * DIM * VOCAB
FLOP_PER_STEP = 3 * FLOP_PER_GEMM
CE_METRIC = "fused-CE TFLOP/s (fwd+bwd, logits+dX+dW GEMMs)"
CE_WORKLOAD = "chunked lm_head cross-entropy fwd+bwd, hidden [2048,1536] bf16, W [151936,1536] bf16"

# QLoRA step workload
METRIC = "QLoRA train tokens/s"
QLORA_BATCH, QLORA_SEQ, QLORA_LAYERS = 4, 2048, 28
INTER = 8960
# bounded CPU sample of the step: all 28 layers, one sequence of 256 tokens
CPU_LAYERS, CPU_BATCH, CPU_SEQ = 28, 1, 256


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 6650.0, "fallback"


def _sustained_peak():
    """(bf16 TFLOP/s of a seconds-long cuBLAS loop under the power cap, source)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops_sustained"]), "measured"
    except Exception:
        return 1400.0, "fallback"


def _committed_traffic(key):
    """Mean DRAM bytes per launch of a kernel from the committed ncu summary, if any."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f).get(f"{key}_bytes_per_launch")
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi SM clock / throttle samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(
                    ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                     "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                parts = [p.strip() for p in out.stdout.strip().split(",")]
                if len(parts) >= 9:
                    self.samples.append(parts)
            except Exception:
                pass
            self._stop.wait(0.1)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for s in self.samples:
            for name, val in zip(names, s[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.samples)}


class Ranks:
    """One process per GPU (torchrun env), NCCL process group with a bounded timeout."""

    def __init__(self, timeout_s: int = 300):
        import torch.distributed as dist

        self.dist = dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            from datetime import timedelta
            dist.init_process_group("nccl", timeout=timedelta(seconds=timeout_s), device_id=self.dev)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max(self, v: float) -> float:
        if self.world == 1:
            return v
        t = torch.tensor([v], device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t)

    def close(self):
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


def _free():
    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def ctypes_void_p_array(values):
    import ctypes

    return (ctypes.c_void_p * len(values))(*values)


def count_own_kernels(step, n_steps=1):
    """Launches per step of this library's kernels (namespace soup::), from a CUPTI trace."""
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(n_steps):
            step()
        torch.cuda.synchronize()
    import re

    mine = re.compile(r"\b(soup|tc)::")  # the library's namespaces (soup::, soup::tc::)
    own = other = 0
    for e in prof.events():
        if e.device_type == torch.autograd.DeviceType.CUDA:
            if mine.search(e.name):
                own += 1
            elif "Memcpy" not in e.name and "Memset" not in e.name:
                other += 1
    return own // n_steps, other // n_steps


def kernel_table(step, n_steps, top=40):
    """Per-kernel device time of `n_steps` calls of `step` (CUPTI through
    torch.profiler; kernels run back to back as in the timed region), printed to
    stderr as: ms per step, share, launches per step, kernel name."""
    import collections

    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(n_steps):
            step()
        torch.cuda.synchronize()
    agg = collections.defaultdict(lambda: [0, 0.0])
    for e in prof.events():
        if e.device_type == torch.autograd.DeviceType.CUDA:
            agg[e.name][0] += 1
            agg[e.name][1] += e.device_time_total
    total = sum(v[1] for v in agg.values())
    print(f"kernel time per step {total / n_steps / 1000:.3f} ms", file=sys.stderr)
    for name, (n, t) in sorted(agg.items(), key=lambda kv: -kv[1][1])[:top]:
        print(f"{t / n_steps / 1000:8.3f} ms {100 * t / total:5.1f}% {n // n_steps:5d}x  {name[:140]}",
              file=sys.stderr)


# ============================================================ CPU baseline ===
def cpu_step_sample(steps: int, warmup: int, seconds: float = 0.0):
    """Time the reference's eager step on the host (oracle.qlora_step) and
    normalise by algorithmic FLOPs per token to the benchmark configuration.

    Returns (tokens/s at the benchmark configuration, seconds per sample step,
    steps timed, threads)."""
    from oracle import qlora_step as ref

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    model = ref.build_model(CPU_LAYERS, seed=0)
    runner = ref.EagerQLoRAStep(model)
    g = torch.Generator().manual_seed(1234)
    ids = torch.randint(0, VOCAB, (CPU_BATCH, CPU_SEQ), generator=g)
    labels = ref.causal_labels(ids)
    for _ in range(warmup):
        runner.step(ids, labels)
    n, t0 = 0, time.perf_counter()
    while True:
        runner.step(ids, labels)
        n += 1
        el = time.perf_counter() - t0
        if n >= steps and el >= seconds:
            break
    per = el / n
    sample_flop = CPU_BATCH * CPU_SEQ * ref.train_flop_per_token(CPU_SEQ, CPU_LAYERS)
    full_fpt = ref.train_flop_per_token(QLORA_SEQ, QLORA_LAYERS)
    tok_s = sample_flop / per / full_fpt
    del runner, model
    gc.collect()
    return tok_s, per, n, threads


def _cpu_sample_text(per, n):
    from oracle import qlora_step as ref

    return (f"{n} steps of the eager PyTorch QLoRA step on the host (transformers Qwen2, "
            f"{CPU_LAYERS} layers, bf16 dense frozen base, LoRA r16 on 7 projections, chunked "
            f"fp32 head CE, AdamW) on batch {CPU_BATCH} x {CPU_SEQ} tokens, {per:.3f} s/step = "
            f"{CPU_BATCH * CPU_SEQ * ref.train_flop_per_token(CPU_SEQ, CPU_LAYERS) / per / 1e12:.3f} "
            f"TFLOP/s; tokens/s normalised by FLOPs per token to batch {QLORA_BATCH} x "
            f"{QLORA_SEQ} ({ref.train_flop_per_token(QLORA_SEQ) / 1e9:.3f} GFLOP/token); "
            "same_config false")


def run_reference(args):
    """--impl reference: the reference's eager step on the host cores (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    tok_s, per, n, threads = cpu_step_sample(args.steps, args.warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tok_s, 3), "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(per * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (uniform random token ids)",
        "config": {"workload": "Qwen2.5-1.5B-architecture QLoRA step, eager PyTorch on the host",
                   "sample": f"batch {CPU_BATCH} x {CPU_SEQ} tokens per step, {CPU_LAYERS} layers",
                   "normalised_to": f"batch {QLORA_BATCH} x {QLORA_SEQ} per step",
                   "same_config": False, "l2": "n/a (CPU)"},
        "cpu_baseline": {"value": round(tok_s, 3), "unit": "tokens/s", "cores": threads,
                         "kind": "port", "sample": _cpu_sample_text(per, n)},
        "e2e": {"value": round(tok_s, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ============================================================= QLoRA step ===
def measure_qlora(args, R: Ranks, batch: int, seq: int, with_extras: bool = True):
    """Train-step tokens/s of the QLoRA step on this rank group (see module doc)."""
    from auspex_soup_demo_b200 import _lib, apply, qlora
    from oracle import qlora_step as ref

    apply()
    # The reference recomputes gate/up in the MLP backward to fit a 16 GB T4
    # (solution/kernels/swiglu.py:205-214). Its results are bit-identical to keeping
    # [g | u] (tests/test_gpu_qlora.py), which at B4 x S2048 costs 294 MB per layer
    # (8.2 GB for 28 layers) of the B200's 180 GB and saves one gate/up GEMM per layer.
    from auspex_soup_demo_b200.kernels import swiglu as _swiglu
    _swiglu.RECOMPUTE = bool(args.recompute)
    qlora.RANK_KERNELS = bool(getattr(args, "rank_kernels", False))
    qlora.DUAL_RANK = not bool(getattr(args, "no_dual_rank", False))
    dev = R.dev
    model = qlora.build_qwen2_qlora(qlora.qwen2_1p5b_config(num_layers=args.layers,
                                                            attention=args.attention),
                                    device=dev, seed=0)
    trainer = qlora.QLoRATrainer(model, lr=2e-4, ddp=R.world > 1)
    g = torch.Generator().manual_seed(1234 + R.rank)
    ids_cpu = torch.randint(0, VOCAB, (batch, seq), generator=g)
    labels_cpu = qlora.causal_labels(ids_cpu)
    ids, labels = ids_cpu.to(dev), labels_cpu.to(dev)
    den = float((labels_cpu != -100).sum())
    # every rank's batch has the same number of labelled tokens (no padding), so
    # averaging the per-rank gradients gives the gradient of the global mean loss
    use_graph = not args.no_graph
    if use_graph:
        trainer.capture(ids, labels, den, warmup=max(args.warmup, 3))

    def one_step():
        return trainer.replay() if use_graph else trainer.step(ids, labels, den)

    for _ in range(max(args.warmup, 3)):
        one_step()
    torch.cuda.synchronize()
    assert _lib.device_error(dev) == 0
    stream = torch.cuda.current_stream(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(R.local) as clocks:
        R.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            loss, _ = one_step()
        e1.record(stream)
        torch.cuda.synchronize()
        R.barrier()
    ms = R.max(e0.elapsed_time(e1) / args.steps)
    tok_s = R.world * batch * seq / (ms * 1e-3)

    # e2e: ids and labels from pinned host memory each step, loss read back
    ids_pin = ids_cpu.pin_memory()
    lab_pin = labels_cpu.pin_memory()
    out_pin = torch.empty(1, dtype=torch.float32).pin_memory()
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    R.barrier()
    torch.cuda.synchronize()
    e2.record(stream)
    for _ in range(args.steps):
        ids.copy_(ids_pin, non_blocking=True)
        labels.copy_(lab_pin, non_blocking=True)
        loss, _ = one_step()
        out_pin.copy_(loss.view(1), non_blocking=True)
    e3.record(stream)
    torch.cuda.synchronize()
    R.barrier()
    e2e_ms = R.max(e2.elapsed_time(e3) / args.steps)
    assert _lib.device_error(dev) == 0
    res = {"tokens_per_s": tok_s, "ms": ms, "e2e_ms": e2e_ms, "loss": float(out_pin[0]),
           "clocks": clocks.summary(), "graph": use_graph,
           "lora_params": sum(p.numel() for p in qlora.lora_parameters(model))}

    if with_extras:
        # kernels of this library per step (every rank replays: the graph holds the all-reduce)
        own, other = count_own_kernels(one_step)
        res["own_kernels_per_step"] = own
        res["other_kernels_per_step"] = other
        # the gradient all-reduce alone
        if R.world > 1:
            ar = []
            for _ in range(6):
                a0 = torch.cuda.Event(enable_timing=True)
                a1 = torch.cuda.Event(enable_timing=True)
                R.barrier()
                a0.record(stream)
                trainer._allreduce_grads()
                a1.record(stream)
                torch.cuda.synchronize()
                ar.append(a0.elapsed_time(a1))
            ar_ms = R.max(statistics.median(ar[1:]))
            nbytes = trainer.flat_grad.numel() * 4
            res["allreduce"] = {"ms": round(ar_ms, 4), "bytes": nbytes,
                                "busbw_gbs": round(2 * (R.world - 1) / R.world * nbytes / (ar_ms * 1e-3) / 1e9, 1),
                                "share_of_step": round(ar_ms / ms, 4),
                                "op": "NCCL all_reduce(AVG) of the flat fp32 LoRA gradient, eager, "
                                      "CUDA events, median of 5, max over ranks"}
        # dominant kernel: the gate/up GEMM with the SwiGLU epilogue, at the step's shape
        grp = model.model.layers[0].mlp.gate_proj.lora_group
        if grp is not None and grp.interleaved:
            res["dominant"] = time_gate_up_gemm(grp, batch * seq, dev, recompute=bool(args.recompute))
        if args.profile and R.rank == 0:
            kernel_table(one_step, 2)
        sus_peak, sus_src = _sustained_peak()
        fpt = ref.train_flop_per_token(seq, args.layers)
        res["step_mfu"] = {"flop_per_token": fpt,
                           "achieved_tflops_per_gpu": round(fpt * tok_s / R.world / 1e12, 1),
                           "frac": round(fpt * tok_s / R.world / 1e12 / sus_peak, 4),
                           "peak": sus_peak,
                           "peak_source": f"{sus_src} bf16_tflops_sustained (the step runs for "
                                          "seconds under the power cap)",
                           "formula": "oracle.qlora_step.train_flop_per_token: 4 x base and head "
                                      "params (fwd + dX), 3 x causal attention fwd, 6 r (in+out) "
                                      "per LoRA projection; recompute, NF4 and AdamW not counted"}
    trainer.release_graph()
    del trainer, model
    _free()
    return res


def time_mlp_backward(m: int, dev, reps: int = 20, hidden: int = 1536, inter: int = 8960,
                      r: int = 16):
    """The MLP backward's first step at m tokens (Qwen2.5-1.5B shapes): down_proj's
    input-gradient GEMM dh = dout W + dxa As with the SwiGLU backward in its
    epilogue ([dg | du] written over [g | u], soup_gemm_bf16_lora_dswiglu) against
    the same GEMM storing dh (soup_gemm_bf16_lora) followed by the elementwise
    SwiGLU backward. CUDA events, reps back-to-back launches each."""
    from auspex_soup_demo_b200 import qlora
    from auspex_soup_demo_b200.kernels.swiglu import swiglu_backward

    g = torch.Generator(device=dev).manual_seed(6)
    d = torch.randn(m, hidden, device=dev, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(hidden, inter, device=dev, generator=g)).to(torch.bfloat16)
    dxa = torch.randn(m, r, device=dev, generator=g).to(torch.bfloat16)
    As = (0.02 * torch.randn(r, inter, device=dev, generator=g)).to(torch.bfloat16)
    y = torch.randn(m, 2 * inter, device=dev, generator=g).to(torch.bfloat16)
    dh = torch.empty(m, inter, device=dev, dtype=torch.bfloat16)
    dy = torch.empty_like(y)
    y2, d2 = y.view(-1, 256), dy.view(-1, 256)
    stream = torch.cuda.current_stream(dev)

    def timed(fn):
        for _ in range(3):
            fn()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    t_gemm = timed(lambda: qlora.lora_gemm(d, w, True, dxa, As, dh))
    t_ew = timed(lambda: swiglu_backward(dh.view(-1, 128), y2[:, :128], y2[:, 128:],
                                         dg=d2[:, :128], du=d2[:, 128:]))
    yy = y.clone()
    t_fused = timed(lambda: qlora.dswiglu_gemm(d, w, dxa, As, yy))
    flop = 2.0 * m * inter * (hidden + r)
    peak, _, src = _peaks()
    sus_peak, sus_src = _sustained_peak()
    return {"kernel": "soup::tc::gemm_pair_kernel<EpiDSwiGLU> (down dX + rank-16 k-block, SwiGLU "
                      "backward in the epilogue, [dg | du] over [g | u])",
            "shape": f"M {m} x N {inter} x K {hidden} + rank {r}",
            "ms_fused": round(t_fused, 4), "ms_unfused_gemm": round(t_gemm, 4),
            "ms_unfused_swiglu_bwd": round(t_ew, 4),
            "saving_ms": round(t_gemm + t_ew - t_fused, 4),
            "achieved": round(flop / (t_fused * 1e-3) / 1e12, 1), "peak": peak,
            "frac": round(flop / (t_fused * 1e-3) / 1e12 / peak, 4),
            "frac_of_sustained": round(flop / (t_fused * 1e-3) / 1e12 / sus_peak, 4),
            "peak_source": f"{src} bf16_tflops (burst); sustained {sus_src}",
            "epilogue_bytes": 4 * m * inter * 2}


def time_rank_products(m: int, dev, reps: int = 20):
    """The four rank-r products of each Qwen2.5-1.5B LoRA linear at m tokens (xa =
    x (sA)^T, dxa = dy B, gA += s dxa^T x, gB += dy^T xa) on soup_lora_rank_gemm
    against cuBLAS. Each product is captured reps times in a CUDA graph, replayed
    5 times (microseconds per product, CUDA events)."""
    from auspex_soup_demo_b200 import qlora

    stream = torch.cuda.current_stream(dev)
    g = torch.Generator(device=dev).manual_seed(8)

    def timed(fn):
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        stream.wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(reps):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(5):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        del graph
        return round(e0.elapsed_time(e1) / (5 * reps) * 1e3, 2)

    def rnd(*shape):
        return torch.randn(*shape, device=dev, generator=g).to(torch.bfloat16)

    out = {}
    for name, k_in, n_out, r in (("qkv", 1536, 2048, 48), ("o", 1536, 1536, 16),
                                 ("gate_up", 1536, 17920, 32), ("down", 8960, 1536, 16)):
        x, dy, a, bt = rnd(m, k_in), rnd(m, n_out), 0.05 * rnd(r, k_in), 0.05 * rnd(r, n_out)
        b = bt.t().contiguous()
        xa, dxa = rnd(m, r), rnd(m, r)
        xat, dxat = xa.t().contiguous(), dxa.t().contiguous()
        c = torch.empty(m, r, device=dev, dtype=torch.bfloat16)
        ct = torch.empty(r, m, device=dev, dtype=torch.bfloat16)
        ga = torch.zeros(r, k_in, device=dev)
        gb = torch.zeros(n_out, r, device=dev)
        out[name] = {
            "xa_us": [timed(lambda: qlora.rank_gemm(x, a, c=c, ct=ct)), timed(lambda: x @ a.t())],
            "dxa_us": [timed(lambda: qlora.rank_gemm(dy, bt, c=c, ct=ct)), timed(lambda: dy @ b)],
            "gA_us": [timed(lambda: qlora.rank_gemm(x, dxat, a_mn_major=True, g=ga, g_trans=True, alpha=2.0)),
                      timed(lambda: torch.addmm(ga, dxa.t(), x, alpha=2.0, out_dtype=torch.float32, out=ga))],
            "gB_us": [timed(lambda: qlora.rank_gemm(dy, xat, a_mn_major=True, g=gb)),
                      timed(lambda: torch.addmm(gb, dy.t(), xa, out_dtype=torch.float32, out=gb))],
        }
    # both products of the gate/up gradient in one pass (soup_lora_rank_dual) against cuBLAS's two
    dy, bt = rnd(m, 17920), 0.05 * rnd(32, 17920)
    xa = rnd(m, 32)
    b = bt.t().contiguous()
    xt = xa.t().contiguous()
    dual = {"dxa_and_dyT_xa_us": [timed(lambda: qlora.rank_dual(dy, bt, xt)),
                                  timed(lambda: (dy @ b, torch.mm(dy.t(), xa, out_dtype=torch.float32)))],
            "shape": f"dy [{m}, 17920], rank 32"}
    return {"shape": f"{m} tokens; [kernel, cuBLAS] microseconds per product", "products": out,
            "dual": dual}


def time_projection_gemms(m: int, dev, reps: int = 40, rounds: int = 3):
    """CUDA-event time (us) of the QLoRA projections' one-GEMM LoRA linears
    (soup_gemm_bf16_lora: y = a op(b) + a2 op(b2)) at m tokens, with the
    stream-K tail on (default threshold), forced on every tail
    (soup_gemm_set_stream_k_min_saved(0)) and off, and of cuBLAS's GEMM plus its
    accumulating rank-r GEMM. Each is a CUDA graph of `reps` launches replayed
    5 times; the variants alternate `rounds` times (medians), since the GPU's
    power-capped clock drifts over a run."""
    import statistics

    import torch.nn.functional as F

    from auspex_soup_demo_b200 import _lib, qlora

    stream = torch.cuda.current_stream(dev)
    g = torch.Generator(device=dev).manual_seed(9)

    def timed(fn):
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        stream.wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(reps):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(5):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        del graph
        return e0.elapsed_time(e1) / (5 * reps) * 1e3

    def rnd(*shape):
        return (0.5 * torch.randn(*shape, device=dev, generator=g)).to(torch.bfloat16)

    lib = _lib.lib()
    out = {}
    # (name, K, N, rank, B stored [K, N] (the input-gradient GEMMs) or [N, K])
    for name, k, n, r, mn in (("qkv_fwd", 1536, 2048, 48, False), ("qkv_dx", 2048, 1536, 48, True),
                              ("o_fwd", 1536, 1536, 16, False), ("o_dx", 1536, 1536, 16, True),
                              ("down_fwd", 8960, 1536, 16, False), ("gate_up_dx", 17920, 1536, 32, True)):
        a, a2 = rnd(m, k), rnd(m, r)
        b, b2 = (rnd(k, n), rnd(r, n)) if mn else (rnd(n, k), rnd(n, r))
        c = torch.empty(m, n, device=dev, dtype=torch.bfloat16)

        def ours():
            qlora.lora_gemm(a, b, mn, a2, b2, c)

        def cublas():
            y = a @ b if mn else F.linear(a, b)
            y.addmm_(a2, b2 if mn else b2.t())

        t = {"tail_default": [], "tail_forced": [], "tail_off": [], "cublas": []}
        try:
            for _ in range(rounds):
                for mode in t:
                    _lib.set_stream_k(mode != "tail_off")
                    lib.soup_gemm_set_stream_k_min_saved(0 if mode == "tail_forced" else -1)
                    t[mode].append(timed(cublas if mode == "cublas" else ours))
        finally:
            _lib.set_stream_k(True)
            lib.soup_gemm_set_stream_k_min_saved(-1)
        flop = 2 * m * n * (k + r)
        med = {mode: statistics.median(v) for mode, v in t.items()}
        out[name] = {**{f"{mode}_us": round(v, 2) for mode, v in med.items()},
                     "tflops_tail_default": round(flop / med["tail_default"] / 1e6, 1),
                     "tflops_cublas": round(flop / med["cublas"] / 1e6, 1),
                     "tiles": -(-m // 256) * -(-n // 256)}
    return {"shape": f"{m} tokens; microseconds per launch (medians of {rounds} alternating rounds)",
            "gemms": out}


def time_gate_up_gemm(group, m: int, dev, reps: int = 20, recompute: bool = False):
    """CUDA-event duration of the gate/up GEMM + SwiGLU epilogue launch at m tokens,
    the QLoRA step's largest kernel, in the modes the step runs: the forward that
    also keeps [g | u] for the backward, or (recompute) the forward that writes h
    only and the recompute-backward that turns dh into [dg | du]."""
    from auspex_soup_demo_b200 import qlora

    k = group.in_features
    g = torch.Generator(device=dev).manual_seed(5)
    x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
    w = group.base_weight(torch.bfloat16)
    As16, Bblk = group.factors(torch.bfloat16)
    xa = x @ As16.t()
    inter = group.outs[0]
    h = torch.empty(m, inter, device=dev, dtype=torch.bfloat16)
    dh = torch.randn(m, inter, device=dev, generator=g).to(torch.bfloat16)
    dy = torch.empty(m, group.n_total, device=dev, dtype=torch.bfloat16)
    stream = torch.cuda.current_stream(dev)
    out = {}
    modes = ((0, "fwd"), (1, "bwd")) if recompute else ((2, "fwd"),)
    for mode, name in modes:
        def launch():
            if mode == 0:
                qlora.swiglu_gemm(x, w, xa, Bblk, None, 0, h)
            elif mode == 2:  # forward keeping [g | u] for the backward
                qlora.swiglu_gemm(x, w, xa, Bblk, None, 0, h, dy)
            else:
                qlora.swiglu_gemm(x, w, xa, Bblk, None, 1, dh, dy)
        for _ in range(3):
            launch()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(reps):
            launch()
        e1.record(stream)
        torch.cuda.synchronize()
        out[name] = e0.elapsed_time(e1) / reps
    n = group.n_total
    r = Bblk.shape[1]
    flop = 2.0 * m * n * (k + r)
    peak, _, src = _peaks()
    sus_peak, sus_src = _sustained_peak()
    mean_ms = sum(out.values()) / len(out)
    achieved = flop / (mean_ms * 1e-3) / 1e12
    modes_text = ("forward (h only) and recompute-backward modes" if recompute
                  else "forward writing h and [g | u]")
    return {"kernel": "soup::tc::gemm_pair_kernel<EpiSwiGLU> (gate/up + rank-32 LoRA k-block, "
                      f"SwiGLU epilogue; {modes_text})",
            "shape": f"M {m} x N {n} (gate/up interleaved) x K {k} + rank {r}",
            "flop_per_launch": flop, "ms_fwd": round(out["fwd"], 4),
            "ms_bwd": round(out["bwd"], 4) if "bwd" in out else None,
            "achieved": round(achieved, 1), "peak": peak, "frac": round(achieved / peak, 4),
            "peak_source": f"{src} bf16_tflops (burst: the launch is timed alone, {reps} back to back)",
            "frac_of_sustained": round(achieved / sus_peak, 4), "sustained_peak": sus_peak,
            "sustained_peak_source": f"{sus_src} bf16_tflops_sustained",
            "traffic": _committed_traffic(f"gemm_pair_kernel_swiglu_m{m}"
                                          + ("" if recompute else "_keep"))}


# ============================================================== fused CE ====
def make_inputs(seed: int, device):
    g = torch.Generator().manual_seed(seed)
    hidden = torch.randn(N_TOK, DIM, generator=g).to(torch.bfloat16)
    labels = torch.randint(0, VOCAB, (N_TOK,), generator=g)
    labels[torch.rand(N_TOK, generator=g) < 0.1] = -100
    gw = torch.Generator(device=device).manual_seed(1000 + seed)
    weight = (0.02 * torch.randn(VOCAB, DIM, device=device, generator=gw)).to(torch.bfloat16)
    return hidden, labels, weight


def cpu_eager_chunk(hidden_chunk, weight_cpu, labels_chunk, den):
    """One chunk of the reference's eager formulation: h@W^T, fp32 CE, autograd for dh and dW."""
    h = hidden_chunk.clone().requires_grad_(True)
    w = weight_cpu.detach().requires_grad_(True)
    logits = (h @ w.t()).float()
    loss = torch.nn.functional.cross_entropy(logits, labels_chunk, ignore_index=-100,
                                             reduction="sum") / den
    with torch.no_grad():
        logp = torch.log_softmax(logits, -1)
        _ = -(logp.exp() * logp).sum(-1)
        _ = (logits.argmax(-1) == labels_chunk).sum()
    loss.backward()
    return float(loss.detach())


def ce_cpu_baseline(seconds: float = 8.0, rows: int = 4 * CHUNK):
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(7)
    weight = (0.02 * torch.randn(VOCAB, DIM, generator=g)).to(torch.bfloat16)
    hidden = torch.randn(rows, DIM, generator=g).to(torch.bfloat16)
    labels = torch.randint(0, VOCAB, (rows,), generator=g)
    den = float(rows)
    cpu_eager_chunk(hidden, weight, labels, den)  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        cpu_eager_chunk(hidden, weight, labels, den)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds or n >= 50:
            break
    per = el / n
    flop = 3 * 2.0 * rows * DIM * VOCAB
    return {"value": flop / per / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{n} x one {rows}-token chunk (B=4 x chunk {CHUNK}) of the same workload, "
                      f"PyTorch eager bf16 GEMMs + fp32 CE + autograd dh/dW, {per * 1e3:.1f} ms/chunk"}


def measure_ce(args, R: Ranks):
    """Fused head CE fwd+bwd on 2048 tokens per rank (weak scaling, no collective)."""
    from auspex_soup_demo_b200 import _lib
    from auspex_soup_demo_b200.kernels import make_triton_chunked_loss_function
    from auspex_soup_demo_b200.kernels.chunked_ce import fused_linear_cross_entropy

    dev = R.dev
    world = R.world
    hidden_cpu, labels_cpu, weight = make_inputs(R.rank, dev)
    hidden = hidden_cpu.to(dev)
    labels = labels_cpu.to(dev)
    den = float((labels_cpu != -100).sum())
    stream = torch.cuda.current_stream(dev)

    # stage events recorded by the library inside each fused call
    start_ev = torch.cuda.Event(enable_timing=True)
    stage_ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
    for e in [start_ev, *stage_ev]:
        e.record(stream)  # materialise the handles
    torch.cuda.synchronize()

    def step():
        return fused_linear_cross_entropy(hidden, weight, labels, den, -100, True, compute_dw=True,
                                          dw_dtype=torch.bfloat16)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    assert _lib.device_error(dev) == 0

    # per-stage timing (one extra pass per step, outside the timed loop)
    handles = ctypes_void_p_array([e.cuda_event for e in stage_ev])
    _lib.lib().soup_set_stage_events(handles, 6)
    stage_ms = [[] for _ in range(6)]
    for _ in range(max(3, min(args.steps, 10))):
        start_ev.record(stream)
        step()
        torch.cuda.synchronize()
        prev = start_ev
        for i, e in enumerate(stage_ev):
            stage_ms[i].append(prev.elapsed_time(e))
            prev = e
    _lib.lib().soup_set_stage_events(None, 0)
    st = [statistics.median(v) for v in stage_ms]

    # timed region: device-resident inputs
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(R.local) as clocks:
        R.barrier()
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
        R.barrier()
    ms_all = R.max(ev0.elapsed_time(ev1) / args.steps)
    value = world * FLOP_PER_STEP / (ms_all * 1e-3) / 1e12

    # e2e through the reference-facing autograd Function, host buffers
    head = torch.nn.Linear(DIM, VOCAB, bias=False, dtype=torch.bfloat16, device=dev)
    with torch.no_grad():
        head.weight.copy_(weight)
    Fn = make_triton_chunked_loss_function()
    h_pin = hidden_cpu.view(1, N_TOK, DIM).pin_memory()
    l_pin = labels_cpu.view(1, N_TOK).pin_memory()
    res_pin = torch.empty(2, dtype=torch.float32).pin_memory()

    # Inputs are double-buffered: a copy stream brings step i+1's hidden states and
    # labels from pinned host memory while step i computes (every step's copy is
    # still inside the timed region: the first one waits for the start event).
    copy_stream = torch.cuda.Stream(dev)
    h_buf = [torch.empty(1, N_TOK, DIM, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    l_buf = [torch.empty(1, N_TOK, dtype=torch.int64, device=dev) for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    for e in consumed:
        e.record(stream)

    def prefetch(i):
        j = i % 2
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(consumed[j])  # step i-2 is done with this buffer
            h_buf[j].copy_(h_pin, non_blocking=True)
            l_buf[j].copy_(l_pin, non_blocking=True)
            copied[j].record(copy_stream)

    def e2e_step(i):
        j = i % 2
        stream.wait_event(copied[j])
        h = h_buf[j].detach().requires_grad_(True)
        head.weight.grad = None
        loss, ent, tok, corr = Fn.apply(h, head, l_buf[j], CHUNK, den, -100, True)
        loss.backward()
        res = torch.stack([loss.detach().float(), corr.float()])
        res_pin.copy_(res, non_blocking=True)
        consumed[j].record(stream)
        return res

    def e2e_run(n, start_event=None):
        if start_event is not None:
            copy_stream.wait_event(start_event)
        prefetch(0)
        for i in range(n):
            if i + 1 < n:
                prefetch(i + 1)
            e2e_step(i)

    e2e_run(3)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    R.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    e2e_run(args.steps, e0)
    e1.record(stream)
    torch.cuda.synchronize()
    R.barrier()
    e2e_ms = R.max(e0.elapsed_time(e1) / args.steps)
    e2e_val = world * FLOP_PER_STEP / (e2e_ms * 1e-3) / 1e12
    assert _lib.device_error(dev) == 0

    # sustained: the device-resident step back to back for ~1 s; the K-step region
    # runs mostly at boost clocks before the power controller reacts, this one
    # settles under the 1 kW cap (sw_power_cap in its clock record)
    sustained = None
    if args.sustained_steps > 0:
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        with ClockSampler(R.local) as sclocks:
            R.barrier()
            torch.cuda.synchronize()
            s0.record(stream)
            for _ in range(args.sustained_steps):
                step()
            s1.record(stream)
            torch.cuda.synchronize()
            R.barrier()
        sus_ms = R.max(s0.elapsed_time(s1) / args.sustained_steps)
        sus_val = world * FLOP_PER_STEP / (sus_ms * 1e-3) / 1e12
        sus_peak, sus_src = _sustained_peak()
        sustained = {"steps": args.sustained_steps, "value": round(sus_val, 2),
                     "unit": "TFLOP/s", "ms_per_step": round(sus_ms, 4),
                     "clocks": sclocks.summary(),
                     "step_frac_of_sustained_peak": round(sus_val / world / sus_peak, 4),
                     "sustained_peak": sus_peak,
                     "peak_source": f"{sus_src} bf16_tflops_sustained (cuBLAS, seconds-long loop)"}
        assert _lib.device_error(dev) == 0

    peak_tf, _, peak_src = _peaks()
    pairs = os.environ.get("SOUP_GEMM_PAIRS", "1") != "0"
    gemm_ms = [st[0], st[3], st[5]]
    achieved = FLOP_PER_GEMM / (statistics.mean(gemm_ms) * 1e-3) / 1e12
    # stage 0 includes the row-shift kernel, stage 1 the gated fallback GEMM launch
    stage_names = ["logits_gemm", "row_stats", "sums", "dx_gemm", "dx_reduce", "dw_gemm"]
    traffic = _committed_traffic("gemm_pair_kernel" if pairs else "gemm_kernel")
    out = {
        "metric": CE_METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
        "ms_per_step": round(ms_all, 4), "scaling": "weak",
        "config": {"workload": CE_WORKLOAD, "tokens_per_gpu": N_TOK, "chunk": CHUNK,
                   "ignore_frac": 0.1, "parallelism": f"dp{world} (tokens sharded, no collective)",
                   "l2": "inputs larger than L2 (W 467 MB, logits buffer 622 MB)"},
        "e2e": {"value": round(e2e_val, 2), "unit": "TFLOP/s",
                "h2d_bytes_per_step": N_TOK * DIM * 2 + N_TOK * 8, "d2h_bytes_per_step": 8,
                "ms_per_step": round(e2e_ms, 4),
                "api": "make_triton_chunked_loss_function().apply + backward (head weight trainable)",
                "input_copies": "pinned host -> device on a copy stream, double-buffered: step i+1's "
                                "copy overlaps step i's compute"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak_tf,
                     "unit": "TFLOP/s", "frac": round(achieved / peak_tf, 4), "traffic": traffic,
                     "kernel": ("soup::tc::gemm_pair_kernel" if pairs else "soup::tc::gemm_kernel")
                     + " (logits / dX / dW launches, 2*N*V*D each)",
                     "peak_source": f"{peak_src} bf16_tflops (burst)"},
        "stages_ms": {k: round(v, 4) for k, v in zip(stage_names, st)},
        # per step: row shifts, logits GEMM, row stats, gated fallback GEMM (returns at
        # entry unless a row overflowed), sums, dX GEMM, dX reduce, dW GEMM
        "gpu_launches_per_step": 8,
        "clocks": clocks.summary(),
        "sustained": sustained,
    }
    del head, weight, hidden, h_buf
    _free()
    return out


# ----------------------------------------------- memory-bound op workloads ---
def measure_mem_op(wl: str, batch: int, seq: int, steps: int, warmup: int, dev):
    """HBM GB/s of one memory-bound fused op (fwd + bwd) at its benchmark shape.

    Inputs rotate over enough buffer sets to exceed twice the L2 (126 MB);
    `graph_steps` steps are captured once in a CUDA graph and replayed, so
    host launch overhead stays out of the device time. Algorithmic bytes:
    rmsnorm 5*N*D*4 (x, y; dy, x, dx) fp32 [N, 1536]; swiglu 8*N*I*2
    (g, u, out; dy, g, u, dg, du) bf16 [N, 8960]; rope 2 passes x (read +
    write of Q and K + cos/sin reads) bf16 Q [B,12,S,128], K [B,2,S,128].
    N = batch * seq; 4 x 512 are the benchmark shapes.
    """
    from auspex_soup_demo_b200.kernels.rmsnorm import rmsnorm_backward, rmsnorm_forward
    from auspex_soup_demo_b200.kernels.rope import rope_apply, rope_tables
    from auspex_soup_demo_b200.kernels.swiglu import swiglu_backward, swiglu_forward

    g = torch.Generator(device=dev).manual_seed(0)
    l2 = 126 * 2 ** 20
    if wl == "rmsnorm":
        N, D = batch * seq, 1536
        per_set = 4 * N * D * 4
        nsets = max(2, -(-2 * l2 // per_set))
        w = (1 + 0.1 * torch.randn(D, device=dev, generator=g))
        sets = [dict(x=torch.randn(N, D, device=dev, generator=g),
                     dy=torch.randn(N, D, device=dev, generator=g),
                     y=torch.empty(N, D, device=dev), dx=torch.empty(N, D, device=dev),
                     rstd=torch.empty(N, device=dev)) for _ in range(nsets)]
        algo = 5 * N * D * 4 + 3 * D * 4 + 2 * N * 4

        def one(s):
            rmsnorm_forward(s["x"], w, 1e-6, out=s["y"], rstd=s["rstd"])
            rmsnorm_backward(s["dy"], s["x"], w, s["rstd"], True, dx=s["dx"])
        shape = f"x [{N},1536] fp32, dw included"
        dtype = "f32"
    elif wl == "swiglu":
        N, I = batch * seq, INTER
        per_set = 7 * N * I * 2
        nsets = max(2, -(-2 * l2 // per_set))
        sets = [dict(g=torch.randn(N, I, device=dev, generator=g).to(torch.bfloat16),
                     u=torch.randn(N, I, device=dev, generator=g).to(torch.bfloat16),
                     dy=torch.randn(N, I, device=dev, generator=g).to(torch.bfloat16),
                     o=torch.empty(N, I, device=dev, dtype=torch.bfloat16),
                     dg=torch.empty(N, I, device=dev, dtype=torch.bfloat16),
                     du=torch.empty(N, I, device=dev, dtype=torch.bfloat16)) for _ in range(nsets)]
        algo = 8 * N * I * 2

        def one(s):
            swiglu_forward(s["g"], s["u"], out=s["o"])
            swiglu_backward(s["dy"], s["g"], s["u"], dg=s["dg"], du=s["du"])
        shape = f"gate/up [{N},8960] bf16"
        dtype = "bf16"
    elif wl == "rope":
        B, S, Hq, Hk, D = batch, seq, 12, 2, 128
        qk_bytes = (Hq + Hk) * B * S * D * 2
        per_set = 4 * qk_bytes
        nsets = max(2, -(-2 * l2 // per_set))
        cos, sin = rope_tables(S, D, 1e6, torch.bfloat16, dev)
        cos = cos[None, None]
        sin = sin[None, None]
        sets = [dict(q=torch.randn(B, Hq, S, D, device=dev, generator=g).to(torch.bfloat16),
                     k=torch.randn(B, Hk, S, D, device=dev, generator=g).to(torch.bfloat16),
                     qo=torch.empty(B, Hq, S, D, device=dev, dtype=torch.bfloat16),
                     ko=torch.empty(B, Hk, S, D, device=dev, dtype=torch.bfloat16))
                for _ in range(nsets)]
        algo = 2 * (2 * qk_bytes + 2 * S * (D // 2) * 2)

        def one(s):
            rope_apply(s["q"], s["k"], cos, sin, False, q_out=s["qo"], k_out=s["ko"])
            rope_apply(s["qo"], s["ko"], cos, sin, True, q_out=s["q"], k_out=s["k"])
        shape = f"Q [{B},12,{S},128] + K [{B},2,{S},128] bf16, theta 1e6, fwd + inverse"
        dtype = "bf16"
    else:
        raise SystemExit(f"unknown workload {wl}")
    launches_per_step = {"rmsnorm": 3, "swiglu": 2, "rope": 2}[wl]

    graph_steps = max(nsets, 16)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for i in range(3):  # warm-up (also sizes the dw scratch before capture)
            one(sets[i % nsets])
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(graph_steps):
            one(sets[i % nsets])
    for _ in range(max(warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    reps = max(1, steps)
    with ClockSampler(dev.index) as clocks:
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (reps * graph_steps)
    gbs = algo / (ms * 1e-3) / 1e9
    _, peak_hbm, src = _peaks()
    res = {"metric": f"{wl} fwd+bwd HBM GB/s", "value": round(gbs, 1), "unit": "GB/s",
           "steps": reps * graph_steps, "ms_per_step": round(ms, 5), "dtype": dtype,
           "config": {"workload": f"{wl}: {shape}", "buffer_sets": nsets,
                      "l2": f"rotating {nsets} input sets, {nsets * per_set / 2**20:.0f} MiB > 2x L2",
                      "timing": f"CUDA graph of {graph_steps} steps, replayed {reps}x"},
           "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak_hbm, "unit": "GB/s",
                        "frac": round(gbs / peak_hbm, 4),
                        "traffic": _committed_traffic(f"{wl}_b{batch}_s{seq}"),
                        "algorithmic_bytes_per_step": algo, "peak_source": f"{src} hbm_gbs"},
           "launches_per_step": launches_per_step, "clocks": clocks.summary()}
    del graph, sets
    _free()
    return res


# ============================================================= attention ====
def measure_attention(args, R: Ranks, batch: int = QLORA_BATCH, seq: int = QLORA_SEQ):
    """The step's attention alone (B x S tokens, 12 query / 2 KV heads of 128, causal):
    this library's tcgen05 kernels against torch SDPA (cuDNN) on the same inputs,
    forward and forward + backward, CUDA events. FLOPs: forward 4 B H S^2 D / 2
    (causal), backward 2.5x that (5 products, the causal half)."""
    import math

    from auspex_soup_demo_b200.kernels.attention import attention_forward, flash_attention

    dev = R.dev
    H, Hk, D = 12, 2, 128
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(batch, seq, H, D, device=dev, generator=g).to(torch.bfloat16).transpose(1, 2)
    k = torch.randn(batch, seq, Hk, D, device=dev, generator=g).to(torch.bfloat16).transpose(1, 2)
    v = torch.randn(batch, seq, Hk, D, device=dev, generator=g).to(torch.bfloat16).transpose(1, 2)
    do = torch.randn(batch, seq, H, D, device=dev, generator=g).to(torch.bfloat16)
    sc = 1.0 / math.sqrt(D)
    qg, kg, vg = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    sdpa = torch.nn.functional.scaled_dot_product_attention

    def timed(fn, n):
        for _ in range(3):
            fn()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    def soup_fb():
        flash_attention(qg, kg, vg, sc, True).backward(do)

    def sdpa_fb():
        sdpa(qg, kg, vg, is_causal=True, scale=sc, enable_gqa=True).transpose(1, 2).backward(do)

    n = max(args.steps, 5)
    t = {"soup_fwd": timed(lambda: attention_forward(q, k, v, sc, True), n),
         "sdpa_fwd": timed(lambda: sdpa(q, k, v, is_causal=True, scale=sc, enable_gqa=True), n),
         "soup_fwd_bwd": timed(soup_fb, n), "sdpa_fwd_bwd": timed(sdpa_fb, n)}
    fwd_flop = 4.0 * batch * H * seq * seq * D / 2
    peak, _, src = _peaks()
    out = {"config": f"batch {batch} x seq {seq}, 12 query / 2 KV heads of 128, causal, bf16",
           "unit": "us / TFLOP/s", "peak": peak, "peak_source": f"{src} bf16_tflops (burst)",
           "in_step": "sdpa (cuDNN): faster at this shape; the tcgen05 kernels run with "
                      "--attention soup"}
    for key, ms in t.items():
        flop = fwd_flop * (3.5 if key.endswith("fwd_bwd") else 1.0)
        out[key] = {"us": round(ms * 1e3, 1), "tflops": round(flop / (ms * 1e-3) / 1e12, 1),
                    "frac": round(flop / (ms * 1e-3) / 1e12 / peak, 4)}
    del q, k, v, do, qg, kg, vg
    _free()
    return out


# ===================================================== vocab-parallel CE ====
def measure_ce_vp(args, R: Ranks):
    """Vocab-parallel fused CE: T tokens, W [151936, 1536] bf16 sharded over the ranks.

    Strong scaling: the whole problem (6*T*D*V FLOP per step) is fixed; each rank
    computes its vocabulary shard for all tokens. Collectives per step: one
    all-gather of the per-token softmax records and one reduce-scatter of the
    bf16 partial dhidden (each rank keeps its token block).
    """
    from auspex_soup_demo_b200 import _lib
    from auspex_soup_demo_b200.kernels.vocab_parallel import (shard_range,
                                                              vocab_parallel_cross_entropy)

    dev = R.dev
    T = args.tokens
    g = torch.Generator(device=dev).manual_seed(7)  # same hidden/targets on every rank
    hidden = torch.randn(T, DIM, device=dev, generator=g).to(torch.bfloat16)
    targets = torch.randint(0, VOCAB, (T,), device=dev, generator=g)
    targets[torch.rand(T, device=dev, generator=g) < 0.1] = -100
    den = float((targets != -100).sum())
    off, size = shard_range(VOCAB, R.rank, R.world)
    gw = torch.Generator(device=dev).manual_seed(1000 + R.rank)
    w_shard = (0.02 * torch.randn(size, DIM, device=dev, generator=gw)).to(torch.bfloat16)
    ws = torch.empty(_lib.lib().soup_ce_vp_workspace_bytes(T, size, DIM), dtype=torch.uint8,
                     device=dev)
    stream = torch.cuda.current_stream(dev)
    timers = {}

    def step(timed=False):
        return vocab_parallel_cross_entropy(hidden, w_shard, off, VOCAB, targets, den,
                                            workspace=ws, timers=timers if timed else None)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(R.local) as clocks:
        R.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            out = step()
        e1.record(stream)
        torch.cuda.synchronize()
        R.barrier()
    ms = R.max(e0.elapsed_time(e1) / args.steps)
    # stage split (extra steps with events between the stages)
    split = {}
    for _ in range(3):
        timers.clear()
        R.barrier()
        step(timed=True)
        torch.cuda.synchronize()
        for k, (a, b) in timers.items():
            split.setdefault(k, []).append(a.elapsed_time(b))
    split = {k: round(R.max(statistics.median(v)), 4) for k, v in sorted(split.items())}
    flop = 6.0 * T * DIM * VOCAB
    assert _lib.device_error(dev) == 0
    res = {"metric": "vocab-parallel fused-CE TFLOP/s (fwd+bwd)",
           "value": round(flop / (ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s", "n_gpus": R.world,
           "ms_per_step": round(ms, 3), "scaling": "strong",
           "config": {"workload": f"vocab-parallel CE, {T} tokens, W [151936,1536] bf16 "
                                  f"sharded {R.world} ways ({size} rows on rank 0)",
                      "collectives": "all_gather of per-token records + reduce_scatter of the bf16 "
                                     "partial dhidden (token blocks)",
                      "l2": "inputs larger than L2"},
           "stages_ms": split, "loss": float(out[3][0]) / den, "clocks": clocks.summary()}
    del ws, w_shard, hidden
    _free()
    return res


# ================================================================== runs ====
def run_step(args):
    """The default line: QLoRA step tokens/s with the other measurements nested."""
    R = Ranks()
    seq = args.seq or QLORA_SEQ
    q = measure_qlora(args, R, args.batch, seq, with_extras=True)
    extras = {}
    if not args.no_extras:
        if R.world == 1:
            s512 = measure_qlora(args, R, 4, 512, with_extras=False)
            extras["qlora_s512"] = {"metric": METRIC, "value": round(s512["tokens_per_s"], 1),
                                    "unit": "tokens/s", "ms_per_step": round(s512["ms"], 3),
                                    "e2e_tokens_per_s": round(4 * 512 / (s512["e2e_ms"] * 1e-3), 1),
                                    "config": "batch 4 x 512 on 1 GPU (CUDA graph)",
                                    "clocks": s512["clocks"]}
        extras["ce"] = measure_ce(args, R)
        extras["mem_ops"] = {wl: measure_mem_op(wl, 4, 512, args.steps, args.warmup, R.dev)
                             for wl in ("rmsnorm", "swiglu", "rope")}
        extras["ce_vp"] = measure_ce_vp(args, R)
        extras["attention"] = measure_attention(args, R)
    B = args.batch
    own = q.get("own_kernels_per_step", 0)
    line = {
        "metric": METRIC, "value": round(q["tokens_per_s"], 1), "unit": "tokens/s",
        "n_gpus": R.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(q["ms"], 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (uniform random token ids)",
        "config": {"workload": "Qwen2.5-1.5B-architecture QLoRA train step",
                   "model": "Qwen2.5-1.5B architecture, random init", "layers": args.layers,
                   "batch_per_gpu": B, "seq_len": seq, "global_batch": B * R.world,
                   "lora": "r16 a32 q/k/v/o/gate/up/down", "lora_params": q["lora_params"],
                   "base": "NF4 blocksize 64, dequantised per use", "optimizer": "AdamW 2e-4",
                   "mlp_recompute": bool(args.recompute), "attention": args.attention,
                   "rank_products": "soup_lora_rank_gemm" if args.rank_kernels else
                                    ("cuBLAS; gate/up dxa + dy^T xa on soup_lora_rank_dual at >= 4096 tokens"
                                     if not args.no_dual_rank else "cuBLAS"),
                   "parallelism": f"dp{R.world}" + (" (one NCCL all-reduce of the flat fp32 LoRA "
                                                    "gradient per step)" if R.world > 1 else ""),
                   "l2": "weights and activations far larger than L2"},
        "e2e": {"value": round(R.world * B * seq / (q["e2e_ms"] * 1e-3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": 2 * B * seq * 8, "d2h_bytes_per_step": 4,
                "ms_per_step": round(q["e2e_ms"], 3),
                "api": "QLoRATrainer (CUDA graph replay) with ids + labels copied from pinned host "
                       "memory and the loss read back every step"},
        "gpu_launches": own * args.steps,
        "gpu_launches_note": f"{own} launches of this library's kernels per step "
                             f"({q.get('other_kernels_per_step', 0)} other kernels: cuBLAS, cuDNN "
                             "attention, PyTorch elementwise, NCCL), counted from a CUPTI trace of "
                             "one step",
        "clocks": q["clocks"],
        "final_loss": q["loss"], "cuda_graph": q["graph"],
    }
    dom = q.get("dominant")
    if dom:
        line["roofline"] = {"bound": "tensor", "achieved": dom["achieved"], "peak": dom["peak"],
                            "unit": "TFLOP/s", "frac": dom["frac"], "traffic": dom["traffic"],
                            "kernel": dom["kernel"], "shape": dom["shape"],
                            "ms_per_launch": {k: v for k, v in (("fwd", dom["ms_fwd"]),
                                                                ("bwd", dom["ms_bwd"])) if v},
                            "flop_per_launch": dom["flop_per_launch"],
                            "peak_source": dom["peak_source"],
                            "frac_of_sustained": dom["frac_of_sustained"],
                            "sustained_peak": dom["sustained_peak"],
                            "note": "the step runs power-capped (sw_power_cap, see clocks); the "
                                    "sustained peak is cuBLAS's bf16 GEMM under the same cap"}
    line["step_mfu"] = q.get("step_mfu")
    if "allreduce" in q:
        line["allreduce"] = q["allreduce"]
    line.update(extras)
    if R.rank == 0 and R.world == 1 and not args.no_cpu:
        tok_s, per, n, threads = cpu_step_sample(2, 1, seconds=12.0)
        line["cpu_baseline"] = {"value": round(tok_s, 3), "unit": "tokens/s", "cores": threads,
                                "kind": "port", "sample": _cpu_sample_text(per, n)}
        if "ce" in line:
            line["ce"]["cpu_baseline"] = ce_cpu_baseline()
    if R.rank == 0:
        print(json.dumps(line), flush=True)
    R.close()


def run_section(args):
    """One section alone (--workload ...), printed as its own line."""
    R = Ranks()
    base = {"n_gpus": R.world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "vs_baseline": None, "data": "synthetic"}
    if args.workload == "ce":
        res = measure_ce(args, R)
        if R.rank == 0 and R.world == 1 and not args.no_cpu:
            res["cpu_baseline"] = ce_cpu_baseline()
        res["dtype"] = "bf16"
    elif args.workload == "qlora":
        q = measure_qlora(args, R, args.batch, args.seq or QLORA_SEQ, with_extras=True)
        res = {"metric": METRIC, "value": round(q["tokens_per_s"], 1), "unit": "tokens/s",
               "ms_per_step": round(q["ms"], 3), "dtype": "bf16", "scaling": "weak",
               "config": {"workload": "Qwen2.5-1.5B-architecture QLoRA train step",
                          "layers": args.layers, "batch_per_gpu": args.batch,
                          "seq_len": args.seq or QLORA_SEQ},
               **{k: v for k, v in q.items() if k not in ("tokens_per_s", "ms")}}
    elif args.workload == "ce_vp":
        res = measure_ce_vp(args, R)
        res["dtype"] = "bf16"
    elif args.workload == "attention":
        att = measure_attention(args, R, args.batch, args.seq or QLORA_SEQ)
        res = {"metric": "causal GQA attention forward + backward TFLOP/s",
               "value": att["soup_fwd_bwd"]["tflops"], "unit": "TFLOP/s", "dtype": "bf16", **att}
    elif args.workload == "mlp_bwd":
        mb = time_mlp_backward(args.batch * (args.seq or QLORA_SEQ), R.dev, reps=max(args.steps, 1))
        res = {"metric": "down dX GEMM + SwiGLU backward epilogue TFLOP/s", "value": mb["achieved"],
               "unit": "TFLOP/s", "dtype": "bf16", **mb}
    elif args.workload == "rank":
        rk = time_rank_products(args.batch * (args.seq or QLORA_SEQ), R.dev, reps=max(args.steps, 1))
        kern = sum(v[0] for p in rk["products"].values() for v in p.values())
        cub = sum(v[1] for p in rk["products"].values() for v in p.values())
        res = {"metric": "LoRA rank products per layer, kernel / cuBLAS time", "value": round(kern / cub, 3),
               "unit": "ratio", "higher_is_better": False, "dtype": "bf16", **rk}
    elif args.workload == "gemm":
        pg = time_projection_gemms(args.batch * (args.seq or QLORA_SEQ), R.dev, reps=max(args.steps, 1))
        ours = sum(v["tail_default_us"] for v in pg["gemms"].values())
        cub = sum(v["cublas_us"] for v in pg["gemms"].values())
        res = {"metric": "QLoRA projection GEMMs per layer, tcgen05 (stream-K tail) / cuBLAS time",
               "value": round(ours / cub, 3), "unit": "ratio", "higher_is_better": False, "dtype": "bf16",
               **pg}
    elif args.workload == "gateup":
        from auspex_soup_demo_b200 import qlora

        model = qlora.build_qwen2_qlora(qlora.qwen2_1p5b_config(num_layers=1), device=R.dev, seed=0)
        grp = model.model.layers[0].mlp.gate_proj.lora_group
        dom = time_gate_up_gemm(grp, args.batch * (args.seq or QLORA_SEQ), R.dev,
                                reps=max(args.steps, 1), recompute=bool(args.recompute))
        res = {"metric": "gate/up GEMM + SwiGLU epilogue TFLOP/s", "value": dom["achieved"],
               "unit": "TFLOP/s", "dtype": "bf16", **dom}
    else:
        res = measure_mem_op(args.workload, args.batch, args.seq or 512, args.steps, args.warmup,
                             R.dev)
    if R.rank == 0:
        print(json.dumps({**base, **res}), flush=True)
    R.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline legs")
    ap.add_argument("--no-extras", action="store_true",
                    help="default line: skip the nested ce / mem_ops / ce_vp / qlora_s512 results")
    ap.add_argument("--workload", default="step",
                    choices=["step", "qlora", "ce", "rmsnorm", "swiglu", "rope", "ce_vp", "gateup",
                             "attention", "mlp_bwd", "rank", "gemm"],
                    help="step (default): the QLoRA train step with the other results nested; "
                         "qlora: the step alone; ce: the fused head CE; rmsnorm/swiglu/rope: one "
                         "memory-bound op's HBM GB/s; ce_vp: the vocab-parallel CE over all ranks; "
                         "gateup: the step's gate/up GEMM with the SwiGLU epilogue alone; attention: "
                         "this library's attention against torch SDPA at the step's shape; mlp_bwd: "
                         "down_proj's dX GEMM with the SwiGLU backward in its epilogue against the "
                         "unfused pair; rank: the LoRA rank products on soup_lora_rank_gemm against "
                         "cuBLAS; gemm: the projections' LoRA GEMMs with the stream-K tail on, "
                         "forced and off, against cuBLAS")
    ap.add_argument("--sustained-steps", type=int, default=500,
                    help="ce: extra back-to-back steps timed under the power cap (0: skip)")
    ap.add_argument("--tokens", type=int, default=65536, help="ce_vp: tokens per step")
    ap.add_argument("--batch", type=int, default=QLORA_BATCH,
                    help="step/qlora: sequences per GPU; rmsnorm/swiglu/rope: batch of the op's shape")
    ap.add_argument("--seq", type=int, default=None,
                    help="step/qlora: tokens per sequence (2048); rmsnorm/swiglu/rope: sequence "
                         "length of the op's shape (512)")
    ap.add_argument("--layers", type=int, default=QLORA_LAYERS, help="step/qlora: decoder layers")
    ap.add_argument("--no-graph", action="store_true", help="step/qlora: launch eagerly, no CUDA graph")
    ap.add_argument("--attention", default="sdpa", choices=["sdpa", "soup"],
                    help="step/qlora: transformers' SDPA (cuDNN; default) or this library's tcgen05 "
                         "flash attention")
    ap.add_argument("--recompute", action="store_true",
                    help="step/qlora: recompute gate/up in the MLP backward, as the reference does "
                         "(default: keep [g | u] from the forward; same results, more memory)")
    ap.add_argument("--no-dual-rank", action="store_true",
                    help="step/qlora: the gate/up group's dxa and B-gradient products on cuBLAS instead "
                         "of one soup_lora_rank_dual pass")
    ap.add_argument("--rank-kernels", action="store_true",
                    help="step/qlora: LoRA rank products on soup_lora_rank_gemm (default: cuBLAS, "
                         "faster in the step)")
    ap.add_argument("--profile", action="store_true",
                    help="step/qlora: after the timed region, print a per-kernel device-time table "
                         "of two steps (torch.profiler, CUDA activity) to stderr")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "step":
        run_step(args)
    else:
        run_section(args)


if __name__ == "__main__":
    main()

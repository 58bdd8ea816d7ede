"""Benchmark of the fused lm_head cross-entropy (forward + backward) on B200.

Workload (default): hidden [2048, 1536] bf16 ~N(0,1), lm_head W [151936, 1536]
bf16 ~N(0, 0.02), labels uniform in [0, 151936) with 10 % set to -100, chunk 32;
outputs mean loss, entropy, top-1 hits, dhidden and dW. One step = one pass of
the fused path over the 2048 tokens. Algorithmic work: 3 GEMMs x 2*N*V*D =
2.868 TFLOP per step (logits, dX, dW). Metric: TFLOP/s, higher is better.

* ``value``: device-resident inputs, the tensor-level fused call, CUDA events
  around exactly K steps (barrier + synchronize on both sides, max over ranks).
* ``e2e``: the reference-facing autograd Function
  (``make_triton_chunked_loss_function``) with the hidden states and labels
  copied host->device (pinned) each step and loss + hit count read back.
* ``roofline``: the tcgen05 GEMM kernel (three launches per step, 2*N*V*D
  FLOP each) timed by CUDA events the library records between its stages.
* ``cpu_baseline``: the same computation in PyTorch eager on the host cores
  (the oracle restatement), on one 128-token chunk, all threads.

``--impl reference`` times only that CPU path (the reference's PyTorch eager
formulation of the op) and prints its own line. With N > 1 GPUs (torchrun),
every rank runs the same per-GPU workload on its own tokens (weak scaling,
no collective on the data path).
"""

from __future__ import annotations

import argparse
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

N_TOK, DIM, VOCAB, CHUNK = 2048, 1536, 151936, 32
FLOP_PER_GEMM = 2.0 * N_TOK * DIM * VOCAB
FLOP_PER_STEP = 3 * FLOP_PER_GEMM
METRIC = "fused-CE TFLOP/s (fwd+bwd, logits+dX+dW GEMMs)"
WORKLOAD = "chunked lm_head cross-entropy fwd+bwd, hidden [2048,1536] bf16, W [151936,1536] bf16"


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


# ----------------------------------------------------------------- inputs ---
def make_inputs(seed: int, device):
    g = torch.Generator().manual_seed(seed)
    hidden = torch.randn(N_TOK, DIM, generator=g).to(torch.bfloat16)
    labels = torch.randint(0, VOCAB, (N_TOK,), generator=g)
    labels[torch.rand(N_TOK, generator=g) < 0.1] = -100
    gw = torch.Generator(device=device).manual_seed(1000 + seed)
    weight = (0.02 * torch.randn(VOCAB, DIM, device=device, generator=gw)).to(torch.bfloat16)
    return hidden, labels, weight


# ----------------------------------------------------------- CPU baseline ---
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
    return float(loss)


def cpu_baseline(seconds: float = 8.0, rows: int = 4 * CHUNK):
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


# ------------------------------------------------------------------- runs ---
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    rows = 4 * CHUNK
    g = torch.Generator().manual_seed(7)
    weight = (0.02 * torch.randn(VOCAB, DIM, generator=g)).to(torch.bfloat16)
    hidden = torch.randn(rows, DIM, generator=g).to(torch.bfloat16)
    labels = torch.randint(0, VOCAB, (rows,), generator=g)
    labels[torch.rand(rows, generator=g) < 0.1] = -100
    den = float((labels != -100).sum())
    for _ in range(args.warmup):
        cpu_eager_chunk(hidden, weight, labels, den)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_eager_chunk(hidden, weight, labels, den)
    el = time.perf_counter() - t0
    per = el / args.steps
    flop = 3 * 2.0 * rows * DIM * VOCAB
    val = flop / per / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": round(val, 4), "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(per * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample": f"{rows}-token chunk per step",
                   "l2": "n/a (CPU)"},
        "cpu_baseline": {"value": round(val, 4), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": f"one {rows}-token chunk per step, PyTorch eager on the host"},
        "e2e": {"value": round(val, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_b200(args):
    import torch.distributed as dist

    from auspex_soup_demo_b200 import _lib
    from auspex_soup_demo_b200.kernels import make_triton_chunked_loss_function
    from auspex_soup_demo_b200.kernels.chunked_ce import fused_linear_cross_entropy

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    hidden_cpu, labels_cpu, weight = make_inputs(rank, dev)
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

    # ---- per-stage timing (one extra pass per step, outside the timed loop) ----
    handles = (ctypes_void_p_array([e.cuda_event for e in stage_ev]))
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

    # ---- timed region: device-resident inputs ----
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(args.steps):
            out = step()
        ev1.record(stream)
        torch.cuda.synchronize()
        barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    ms_all = ms
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_all = float(t)
    value = world * FLOP_PER_STEP / (ms_all * 1e-3) / 1e12

    # ---- e2e through the reference-facing autograd Function, host buffers ----
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
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    e2e_run(args.steps, e0)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t)
    e2e_val = world * FLOP_PER_STEP / (e2e_ms * 1e-3) / 1e12
    assert _lib.device_error(dev) == 0

    # ---- sustained: the device-resident step back to back for ~1 s. The K-step
    # region above lasts K x ~2.2 ms, mostly at boost clocks before the power
    # controller reacts; this run settles under the 1 kW cap and its clock record
    # shows it (sw_power_cap). Every rank runs it (same collectives).
    sustained = None
    if args.sustained_steps > 0:
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as sclocks:
            barrier()
            torch.cuda.synchronize()
            s0.record(stream)
            for _ in range(args.sustained_steps):
                step()
            s1.record(stream)
            torch.cuda.synchronize()
            barrier()
        sus_ms = s0.elapsed_time(s1) / args.sustained_steps
        if world > 1:
            t = torch.tensor([sus_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            sus_ms = float(t)
        sus_val = world * FLOP_PER_STEP / (sus_ms * 1e-3) / 1e12
        sus_peak, sus_src = _sustained_peak()
        sustained = {"steps": args.sustained_steps, "value": round(sus_val, 2),
                     "unit": "TFLOP/s", "ms_per_step": round(sus_ms, 4),
                     "clocks": sclocks.summary(),
                     "step_frac_of_sustained_peak": round(sus_val / world / sus_peak, 4),
                     "sustained_peak": sus_peak,
                     "peak_source": f"{sus_src} bf16_tflops_sustained (cuBLAS, seconds-long loop)"}
        assert _lib.device_error(dev) == 0

    peak_tf, peak_hbm, peak_src = _peaks()
    pairs = os.environ.get("SOUP_GEMM_PAIRS", "1") != "0"
    gemm_ms = [st[0], st[3], st[5]]
    achieved = FLOP_PER_GEMM / (statistics.mean(gemm_ms) * 1e-3) / 1e12
    # stage 0 includes the row-shift kernel, stage 1 the gated fallback GEMM launch
    stage_names = ["logits_gemm", "row_stats", "sums", "dx_gemm", "dx_reduce", "dw_gemm"]
    traffic = _committed_traffic("gemm_pair_kernel" if pairs else "gemm_kernel")

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_all, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": WORKLOAD, "tokens_per_gpu": N_TOK, "chunk": CHUNK,
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
        "gpu_launches": 8 * args.steps,
        "clocks": clocks.summary(),
        "sustained": sustained,
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ----------------------------------------------- memory-bound op workloads ---
def run_memory_op(args):
    """HBM GB/s of one memory-bound fused op (fwd + bwd) at its benchmark shape.

    Inputs rotate over enough buffer sets to exceed twice the L2 (126 MB);
    `graph_steps` steps are captured once in a CUDA graph and replayed, so
    host launch overhead stays out of the device time. Algorithmic bytes:
    rmsnorm 5*N*D*4 (x, y; dy, x, dx) fp32 [N, 1536]; swiglu 8*N*I*2
    (g, u, out; dy, g, u, dg, du) bf16 [N, 8960]; rope 2 passes x (read +
    write of Q and K + cos/sin reads) bf16 Q [B,12,S,128], K [B,2,S,128].
    B = --batch, S = --seq, N = B*S; the defaults (4 x 512) are the benchmark
    shapes, larger batches show the same kernels with the per-launch fixed cost
    amortised.
    """
    from auspex_soup_demo_b200.kernels.rmsnorm import rmsnorm_backward, rmsnorm_forward
    from auspex_soup_demo_b200.kernels.rope import rope_apply
    from auspex_soup_demo_b200.kernels.swiglu import swiglu_backward, swiglu_forward

    import oracle

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    wl = args.workload
    l2 = 126 * 2 ** 20
    if wl == "rmsnorm":
        N, D = args.batch * args.seq, 1536
        per_set = 4 * N * D * 4
        nsets = max(2, -(-2 * l2 // per_set))
        w = (1 + 0.1 * torch.randn(D, device=dev, generator=g))
        sets = [dict(x=torch.randn(N, D, device=dev, generator=g),
                     dy=torch.randn(N, D, device=dev, generator=g),
                     y=torch.empty(N, D, device=dev), dx=torch.empty(N, D, device=dev),
                     rstd=torch.empty(N, device=dev)) for _ in range(nsets)]
        algo = 5 * N * D * 4 + 3 * D * 4 + 2 * N * 4
        launches = 3

        def one(s):
            rmsnorm_forward(s["x"], w, 1e-6, out=s["y"], rstd=s["rstd"])
            rmsnorm_backward(s["dy"], s["x"], w, s["rstd"], True, dx=s["dx"])
        shape = f"x [{N},1536] fp32, dw included"
    elif wl == "swiglu":
        N, I = args.batch * args.seq, 8960
        per_set = 7 * N * I * 2
        nsets = max(2, -(-2 * l2 // per_set))
        sets = [dict(g=torch.randn(N, I, device=dev, generator=g).to(torch.bfloat16),
                     u=torch.randn(N, I, device=dev, generator=g).to(torch.bfloat16),
                     dy=torch.randn(N, I, device=dev, generator=g).to(torch.bfloat16),
                     o=torch.empty(N, I, device=dev, dtype=torch.bfloat16),
                     dg=torch.empty(N, I, device=dev, dtype=torch.bfloat16),
                     du=torch.empty(N, I, device=dev, dtype=torch.bfloat16)) for _ in range(nsets)]
        algo = 8 * N * I * 2
        launches = 2

        def one(s):
            swiglu_forward(s["g"], s["u"], out=s["o"])
            swiglu_backward(s["dy"], s["g"], s["u"], dg=s["dg"], du=s["du"])
        shape = f"gate/up [{N},8960] bf16"
    elif wl == "rope":
        B, S, Hq, Hk, D = args.batch, args.seq, 12, 2, 128
        qk_bytes = (Hq + Hk) * B * S * D * 2
        per_set = 4 * qk_bytes
        nsets = max(2, -(-2 * l2 // per_set))
        cos, sin = oracle.rope_cos_sin(S, D, 1e6, torch.bfloat16)
        cos = cos[None, None].to(dev)
        sin = sin[None, None].to(dev)
        sets = [dict(q=torch.randn(B, Hq, S, D, device=dev, generator=g).to(torch.bfloat16),
                     k=torch.randn(B, Hk, S, D, device=dev, generator=g).to(torch.bfloat16),
                     qo=torch.empty(B, Hq, S, D, device=dev, dtype=torch.bfloat16),
                     ko=torch.empty(B, Hk, S, D, device=dev, dtype=torch.bfloat16))
                for _ in range(nsets)]
        algo = 2 * (2 * qk_bytes + 2 * S * (D // 2) * 2)
        launches = 2

        def one(s):
            rope_apply(s["q"], s["k"], cos, sin, False, q_out=s["qo"], k_out=s["ko"])
            rope_apply(s["qo"], s["ko"], cos, sin, True, q_out=s["q"], k_out=s["k"])
        shape = f"Q [{B},12,{S},128] + K [{B},2,{S},128] bf16, theta 1e6, fwd + inverse"
    else:
        raise SystemExit(f"unknown workload {wl}")

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
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    reps = max(1, args.steps)
    with ClockSampler(dev.index) as clocks:
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (reps * graph_steps)
    gbs = algo / (ms * 1e-3) / 1e9
    _, peak_hbm, src = _peaks()
    line = {"metric": f"{wl} fwd+bwd HBM GB/s", "value": round(gbs, 1), "unit": "GB/s",
            "n_gpus": 1, "steps": reps * graph_steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 5), "higher_is_better": True, "dtype": "bf16" if wl != "rmsnorm" else "f32",
            "data": "synthetic",
            "config": {"workload": f"{wl}: {shape}", "buffer_sets": nsets,
                       "l2": f"rotating {nsets} input sets, {nsets * per_set / 2**20:.0f} MiB > 2x L2",
                       "timing": f"CUDA graph of {graph_steps} steps, replayed {reps}x"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak_hbm, "unit": "GB/s",
                         "frac": round(gbs / peak_hbm, 4), "traffic": None,
                         "algorithmic_bytes_per_step": algo, "peak_source": f"{src} hbm_gbs"},
            "gpu_launches": launches * reps * graph_steps, "clocks": clocks.summary()}
    print(json.dumps(line), flush=True)


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


def run_qlora(args):
    """Qwen2.5-1.5B-architecture QLoRA train step: tokens/s (whole job).

    Random-init model (28 layers, NF4 blocksize 64, LoRA r16/a32 on
    q/k/v/o/gate/up/down), uniform random token ids, AdamW 2e-4, the fused
    patches installed. One step = forward + backward + optimiser step on
    `batch` x `seq` tokens per GPU. N > 1: DDP over NCCL, LoRA grads only.
    """
    import torch.distributed as dist

    from auspex_soup_demo_b200 import _lib, apply, qlora

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    apply()
    if args.no_recompute:
        from auspex_soup_demo_b200.kernels import swiglu as _swiglu
        _swiglu.RECOMPUTE = False
    B, S = args.batch, args.seq
    model = qlora.build_qwen2_qlora(qlora.qwen2_1p5b_config(num_layers=args.layers), device=dev,
                                    seed=0)
    trainer = qlora.QLoRATrainer(model, lr=2e-4, ddp=world > 1)
    g = torch.Generator().manual_seed(1234 + rank)
    ids_cpu = torch.randint(0, 151936, (B, S), generator=g)
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
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream(dev)
    with ClockSampler(local) as clocks:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            loss, _ = one_step()
        e1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t)
    tok_s = world * B * S / (ms * 1e-3)
    # e2e: token ids from pinned host memory each step, loss read back
    ids_pin = ids_cpu.pin_memory()
    lab_pin = labels_cpu.pin_memory()
    out_pin = torch.empty(1, dtype=torch.float32).pin_memory()
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e2.record(stream)
    for _ in range(args.steps):
        ids.copy_(ids_pin, non_blocking=True)
        labels.copy_(lab_pin, non_blocking=True)
        loss, _ = one_step()
        out_pin.copy_(loss.view(1), non_blocking=True)
    e3.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e2.elapsed_time(e3) / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t)
    assert _lib.device_error(dev) == 0
    if args.profile and rank == 0:
        kernel_table(one_step, 2)
    n_lora = sum(p.numel() for p in qlora.lora_parameters(model))
    line = {"metric": "QLoRA train tokens/s", "value": round(tok_s, 1), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (uniform random token ids)",
            "config": {"workload": "Qwen2.5-1.5B-architecture QLoRA step",
                       "layers": args.layers, "batch_per_gpu": B, "seq_len": S,
                       "lora": "r16 a32 q/k/v/o/gate/up/down", "lora_params": n_lora,
                       "base": "NF4 blocksize 64, dequantised per use", "optimizer": "AdamW 2e-4",
                       "mlp_recompute": not args.no_recompute,
                       "parallelism": f"dp{world}" + (" (one NCCL allreduce of the flat LoRA grads)"
                                                      if world > 1 else ""),
                       "l2": "weights and activations far larger than L2"},
            "e2e": {"value": round(world * B * S / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": 2 * B * S * 8, "d2h_bytes_per_step": 4,
                    "ms_per_step": round(e2e_ms, 3)},
            "final_loss": float(loss), "cuda_graph": use_graph, "clocks": clocks.summary()}
    if rank == 0:
        print(json.dumps(line), flush=True)
    trainer.release_graph()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_ce_vp(args):
    """Vocab-parallel fused CE: 65536 tokens, W [151936, 1536] bf16 sharded over N GPUs.

    Strong scaling: the whole problem (6*T*D*V = 91.77 TFLOP per step) is fixed;
    each rank computes its vocabulary shard for all tokens. Collectives per
    step: all-gather of per-token softmax records, all-reduce of dhidden (fp32).
    """
    import torch.distributed as dist

    from auspex_soup_demo_b200 import _lib
    from auspex_soup_demo_b200.kernels.vocab_parallel import shard_range, vocab_parallel_cross_entropy

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    T = args.tokens
    g = torch.Generator(device=dev).manual_seed(7)  # same hidden/targets on every rank
    hidden = torch.randn(T, DIM, device=dev, generator=g).to(torch.bfloat16)
    targets = torch.randint(0, VOCAB, (T,), device=dev, generator=g)
    targets[torch.rand(T, device=dev, generator=g) < 0.1] = -100
    den = float((targets != -100).sum())
    off, size = shard_range(VOCAB, rank, world)
    gw = torch.Generator(device=dev).manual_seed(1000 + rank)
    w_shard = (0.02 * torch.randn(size, DIM, device=dev, generator=gw)).to(torch.bfloat16)
    ws = torch.empty(_lib.lib().soup_ce_vp_workspace_bytes(T, size, DIM), dtype=torch.uint8,
                     device=dev)

    def step():
        return vocab_parallel_cross_entropy(hidden, w_shard, off, VOCAB, targets, den,
                                            workspace=ws)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream(dev)
    with ClockSampler(local) as clocks:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            out = step()
        e1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t)
    flop = 6.0 * T * DIM * VOCAB
    assert _lib.device_error(dev) == 0
    line = {"metric": "vocab-parallel fused-CE TFLOP/s (fwd+bwd)", "value": round(flop / (ms * 1e-3) / 1e12, 2),
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"vocab-parallel CE, {T} tokens, W [151936,1536] bf16 "
                                   f"sharded {world} ways ({size} rows on rank 0)",
                       "collectives": "all_gather of per-token records + all_reduce(sum) of fp32 dhidden",
                       "l2": "inputs larger than L2"},
            "loss": float(out[3][0]) / den, "clocks": clocks.summary()}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _committed_traffic(kernel):
    """Mean DRAM bytes per GEMM launch of `kernel` from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(f"{kernel}_bytes_per_launch")
    except Exception:
        return None


def ctypes_void_p_array(values):
    import ctypes

    return (ctypes.c_void_p * len(values))(*values)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--sustained-steps", type=int, default=500,
                    help="ce: extra back-to-back steps timed under the power cap (0: skip)")
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--workload", default="ce",
                    choices=["ce", "rmsnorm", "swiglu", "rope", "qlora", "ce_vp"],
                    help="ce (default): the fused head CE; rmsnorm/swiglu/rope: one memory-bound "
                         "op's HBM GB/s; qlora: the Qwen2.5-1.5B QLoRA train step's tokens/s; "
                         "ce_vp: the vocab-parallel CE over all ranks")
    ap.add_argument("--tokens", type=int, default=65536, help="ce_vp: tokens per step")
    ap.add_argument("--batch", type=int, default=4,
                    help="qlora: sequences per GPU; rmsnorm/swiglu/rope: batch of the op's shape")
    ap.add_argument("--seq", type=int, default=512,
                    help="qlora: tokens per sequence; rmsnorm/swiglu/rope: sequence length of the op's shape")
    ap.add_argument("--layers", type=int, default=28, help="qlora: decoder layers")
    ap.add_argument("--no-graph", action="store_true", help="qlora: launch eagerly, no CUDA graph")
    ap.add_argument("--no-recompute", action="store_true",
                    help="qlora: keep MLP activations instead of recomputing gate/up in backward")
    ap.add_argument("--profile", action="store_true",
                    help="qlora: after the timed region, print a per-kernel device-time table of "
                         "two steps (torch.profiler, CUDA activity) to stderr")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "qlora":
        run_qlora(args)
    elif args.workload == "ce_vp":
        run_ce_vp(args)
    elif args.workload != "ce":
        run_memory_op(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()

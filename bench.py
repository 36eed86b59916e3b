"""Benchmark of the B200-native SPLADE head: fused forward + backward.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload config2|config3|config4|config5]
    (N > 1: python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N)

Default workload (benchmark configuration 2, the one the metric is quoted
on): B=128, S=256, D=768, V=30522, bf16 with fp32 accumulation, hidden
~ N(0,1), W ~ N(0,0.02), bias ~ N(0,0.02), right-padded mask with lengths
U[32,256], upstream grad g ~ N(0,1); seeded synthetic data standing in for
SPLADE batches. ``--workload`` selects the other benchmark configurations
(WORKLOADS below: config 3 V=250002, config 4 fp16 B=512 S=512, config 5
D=4096 V=128256 without bias), with the same distributions.
With N GPUs the decoder is vocabulary-sharded over the ranks (the same total
workload: strong scaling) and the partial d_hidden is all-reduced (fp32, NCCL,
in chunks of batch rows overlapping the backward; high-priority NCCL streams).

One step = head forward (mask reduction + fused GEMM/max/argmax/log1p kernel)
+ backward (sort by argmax, dH, dW, db; single GPU: the dH and dW halves on two
streams) [+ all-reduce of dH].

Prints ONE JSON line on rank 0. ``value`` is the benchmark's metric, nominal
fwd+bwd TFLOP/s = 4*B*S*D*V / step time, with inputs resident in HBM and the
L2 flushed (256 MiB write) before every timed step; time is the max over ranks
of CUDA-event time. ``e2e`` is the same metric through the public module
(SpartonHead autograd) with host->device copies of the step's inputs from
pinned memory and a device->host read of reps inside the timed region.
``roofline`` covers the dominant kernel (the forward): algorithmic FLOPs
2*D*V*T (T = valid tokens) over its CUDA-event duration, against the measured
bf16 peak. ``cpu_baseline`` times the reference torch head (oracle/torch_head.py,
a restatement of the reference's --head torch path) on the host cores on a
bounded sample of the same workload.

Further legs (``--legs``), reported as objects in the same line: ``losses``
(InfoNCE and the fused regularisers on reps-shaped input), ``sparse`` (CSR and
top-k of reps), ``transform`` (the MLM transform's kernels, its dense GEMMs and
SpartonProjection forward + backward). Each leg call is timed with CUDA events
after an L2 flush and a short spin kernel (``preroll``), so that its span holds
the call's GPU work rather than Python's queueing ahead of it.

``--impl reference`` times that CPU reference alone (rank 0; other ranks exit)
and prints its line with ``"impl": "reference"``.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

METRIC = "fused head fwd+bwd TFLOP/s (4·B·S·D·V) & tokens/s at 1/2/4/8 B200; % of bf16 peak"
# The benchmark configurations "config 2" .. "config 5". Config 2 is the one the
# metric is quoted on and the default; the others are selected with --workload.
WORKLOADS = {
    "config2": dict(name="config 2 (BERT-base SPLADE head)", B=128, S=256, D=768, V=30522,
                    dtype=torch.bfloat16, lengths=(32, 256), bias=True, w_std=0.02,
                    full_frac=0.0, cpu_rows=8),
    "config3": dict(name="config 3 (XLM-R-base large-vocab head)", B=32, S=256, D=768, V=250002,
                    dtype=torch.bfloat16, lengths=(32, 256), bias=True, w_std=0.02,
                    full_frac=0.0, cpu_rows=2),
    "config4": dict(name="config 4 (long-sequence head)", B=512, S=512, D=768, V=30522,
                    dtype=torch.float16, lengths=(64, 512), bias=True, w_std=0.02,
                    full_frac=0.1, cpu_rows=4),
    "config5": dict(name="config 5 (decoder-LLM-size head)", B=64, S=1024, D=4096, V=128256,
                    dtype=torch.bfloat16, lengths=(256, 1024), bias=False, w_std=0.01,
                    full_frac=0.0, cpu_rows=1),
}
CFG = WORKLOADS["config2"]
DTYPE_NAME = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}
FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0}
L2_FLUSH_BYTES = 256 << 20


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def nominal_flops(c) -> float:
    return 4.0 * c["B"] * c["S"] * c["D"] * c["V"]


def preroll() -> None:
    """A ~0.1 ms spin kernel queued between the L2 flush and a leg's start event:
    the GPU stays busy while Python queues the call under test, so the timed
    span holds that call's GPU work, not the host's launch latency before it."""
    torch.cuda._sleep(200_000)


def make_inputs(c, seed=0):
    """CPU tensors of the workload (seeded; identical on every rank)."""
    gen = torch.Generator().manual_seed(seed)
    B, S, D, V = c["B"], c["S"], c["D"], c["V"]
    H = torch.randn(B, S, D, generator=gen).to(c["dtype"])
    W = (torch.randn(V, D, generator=gen) * c["w_std"]).to(c["dtype"])
    b = (torch.randn(V, generator=gen) * 0.02).to(c["dtype"]) if c["bias"] else None
    lo, hi = c["lengths"]
    L = torch.randint(lo, hi + 1, (B,), generator=gen)
    if c.get("full_frac", 0.0) > 0:  # config 4: a fraction of the rows at full length
        full = torch.rand(B, generator=gen) < c["full_frac"]
        L = torch.where(full, torch.full_like(L, S), L)
    mask = (torch.arange(S)[None, :] < L[:, None]).to(torch.int64)
    g = torch.randn(B, V, generator=gen).to(c["dtype"])
    return H, W, b, mask, g, L


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


def workload_desc(c) -> str:
    lo, hi = c["lengths"]
    full = f", {int(c['full_frac'] * 100)}% of rows full length" if c.get("full_frac") else ""
    return (f"{c['name']}: B={c['B']} S={c['S']} D={c['D']} V={c['V']} {DTYPE_NAME[c['dtype']]}, "
            f"lengths U[{lo},{hi}]{full}, {'bias' if c['bias'] else 'no bias'}")


def profile_traffic(workload: str):
    """DRAM bytes per forward launch from the committed ncu summary of this
    workload, if any."""
    path = os.path.join(REPO, "profiles", f"fwd_tc_{workload}_traffic.txt")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


class ClockSampler:
    """Samples SM clock and clock-event reasons of this process's GPU via NVML
    every 20 ms while active (read-only)."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x2: "applications_clocks_setting", 0x10: "sync_boost"}

    def __init__(self, device: torch.device):
        self.samples, self.reasons, self.max_mhz, self.err = [], set(), None, None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self._h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid).encode())
            self._nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # pragma: no cover - depends on the box
            self.err = repr(e)
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception as e:  # pragma: no cover
                self.err = repr(e)
                return
            time.sleep(0.02)

    def __enter__(self):
        if self._nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": 0, "error": self.err}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


def cpu_rows_for(c, rows=None) -> int:
    """Batch rows one CPU step runs: the whole batch when the torch head's
    [B,S,V] fp32 intermediates (about six of them alive at the peak of
    forward + backward) fit in half the host's free memory (configs 1-3);
    otherwise (configs 4, 5) a slice
    of rows, and the result is extrapolated (rows are independent)."""
    if rows:
        return min(rows, c["B"])
    try:
        import psutil

        free = psutil.virtual_memory().available
    except Exception:  # pragma: no cover - psutil is in the image
        free = 32 << 30
    per_row = 6 * c["S"] * c["V"] * 4
    fit = max(1, int(free * 0.5 // per_row))
    return c["B"] if fit >= c["B"] else min(fit, c["cpu_rows"])


def cpu_baseline(c, rows: int, steps: int, warmup: int) -> dict:
    """The reference torch head (oracle/torch_head.py: training/model.py:56-62
    under autograd) timed on the host cores, fp32, on `rows` batch rows of the
    workload (its own seeded lengths); the whole batch when rows == B."""
    from oracle.torch_head import time_fwd_bwd

    L = make_inputs(c)[5][:rows]
    r = time_fwd_bwd(rows, c["S"], c["D"], c["V"], L.tolist(), use_bias=c["bias"],
                     steps=steps, warmup=warmup, w_std=c["w_std"])
    full = rows == c["B"]
    sec_full = r["seconds_per_step"] * c["B"] / rows
    flops = nominal_flops(c)
    what = (f"the whole batch (B={c['B']} S={c['S']} D={c['D']} V={c['V']})" if full else
            f"B={rows} of {c['B']} rows (S={c['S']} D={c['D']} V={c['V']}), time extrapolated "
            f"x{c['B'] / rows:g} (rows are independent)")
    return {"value": flops / sec_full / 1e12, "unit": "TFLOP/s", "cores": r["threads"],
            "kind": "port", "cpu_model": cpu_model(),
            "sample": f"{what}, fp32, torch head (training/model.py:56-62) fwd + bwd on the host "
                      f"cores, {steps} steps after {warmup} warm-up",
            "seconds_per_step": sec_full, "extrapolated": not full}


def run_reference_arm(args, rank: int) -> int:
    if rank != 0:
        return 0
    c = WORKLOADS[args.workload]
    rows = cpu_rows_for(c, args.cpu_rows)
    res = cpu_baseline(c, rows, steps=args.steps, warmup=args.warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": res["value"], "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": res["seconds_per_step"] * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": workload_desc(c),
                   "B": c["B"], "S": c["S"], "D": c["D"], "V": c["V"],
                   "rows_per_step": rows, "extrapolated": res["extrapolated"],
                   "device": "host CPU", "cpu_model": res["cpu_model"]},
        "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample",
                                             "cpu_model")},
        "e2e": {"value": res["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def e2e_bytes(H, mask, gs, B, Vs, dtype):
    """Host<->device bytes per e2e step: the step's inputs in, reps out."""
    h2d = (H.numel() * H.element_size() + mask.numel() * mask.element_size()
           + gs.numel() * gs.element_size())
    d2h = B * Vs * torch.empty((), dtype=dtype).element_size()
    return h2d, d2h


def run_e2e(args, c, dev, group, W, b, H, mask, gs, Vs, flush, stream, barrier, max_over_ranks):
    """ms per step of the public path: SpartonHead forward + autograd backward on
    inputs that start in pinned host memory, with reps read back to the host.

    Inputs are double-buffered the way a training input pipeline does it: the
    host->device copy of step i+1's hidden states, mask and output gradient runs
    on its own stream while step i computes, and step i's reps go back on a
    third stream (each copy direction has its own copy engine). A device buffer
    is refilled only after the step that read it has finished. Every step's
    copies, its L2 flush and its compute lie inside the timed region, which runs
    from before the first copy to after the last read-back; time per step is
    that span / steps. The parameters' gradients are set to None before each
    backward, as a training loop's zero_grad does (and the reference arm's
    torch head every step), so each backward writes them instead of adding."""
    from sparton_b200.head import SpartonHead

    from torch import nn

    B, D, V = c["B"], c["D"], c["V"]
    # As the reference's ProjectionSparton does (training/model.py:72-84): a
    # head tied to the decoder nn.Linear; sharded, it trains this rank's rows of
    # the decoder with a shard-sized gradient.
    decoder = nn.Linear(D, V, bias=c["bias"]).to(dev, c["dtype"])
    with torch.no_grad():
        decoder.weight.copy_(W)
        if b is not None:
            decoder.bias.copy_(b)
    head = SpartonHead(V, D, use_bias=c["bias"], process_group=group).to(dev, c["dtype"])
    head.tie_weights(decoder)
    params = list(head.parameters()) + list(decoder.parameters())
    H_pin, m_pin, g_pin = H.pin_memory(), mask.pin_memory(), gs.pin_memory()
    H_dev = [torch.empty_like(H, device=dev) for _ in range(2)]
    m_dev = [torch.empty_like(mask, device=dev) for _ in range(2)]
    g_dev = [torch.empty_like(gs, device=dev) for _ in range(2)]
    reps_host = [torch.empty(B, Vs, dtype=c["dtype"]).pin_memory() for _ in range(2)]
    h2d = torch.cuda.Stream(dev)
    d2h = torch.cuda.Stream(dev)
    copied = [torch.cuda.Event() for _ in range(2)]
    freed = [None, None]  # event: the step that last read buffer k has finished

    def upload(i):
        k = i % 2
        with torch.cuda.stream(h2d):
            if freed[k] is not None:
                h2d.wait_event(freed[k])
            H_dev[k].copy_(H_pin, non_blocking=True)
            m_dev[k].copy_(m_pin, non_blocking=True)
            g_dev[k].copy_(g_pin, non_blocking=True)
            copied[k].record(h2d)

    def run(n, timed):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        start.record(stream)
        h2d.wait_stream(stream)
        upload(0)
        for i in range(n):
            k = i % 2
            if i + 1 < n:
                upload(i + 1)
            flush.zero_()
            stream.wait_event(copied[k])
            hid = H_dev[k].detach().requires_grad_(True)
            for prm in params:  # a training loop's zero_grad(set_to_none=True), as the
                prm.grad = None  # reference arm's torch head does every step
            out = head(hid, m_dev[k])
            out.backward(g_dev[k])
            done = torch.cuda.Event()
            done.record(stream)
            freed[k] = done
            with torch.cuda.stream(d2h):
                d2h.wait_event(done)
                reps_host[k].copy_(out.detach(), non_blocking=True)
            out.record_stream(d2h)  # not reused before the read-back has finished
        stream.wait_stream(d2h)
        end.record(stream)
        barrier()
        return start.elapsed_time(end) / n if timed else None

    run(args.warmup, False)
    return max_over_ranks(run(args.steps, True))


def run_losses(args, c, dev, group, world, Vs, flush, stream, barrier, max_over_ranks):
    """The training losses that consume the head (sparton_b200.losses), timed at
    the workload's reps shape [B, V_s] (queries and documents both B rows), L2
    flushed before every iteration, CUDA events, max over ranks:
    * reg_kernels: the fused regulariser kernels alone (csrc/reg.cu, C ABI);
    * reg: l1 + flops regularisers, forward + backward through the autograd API;
    * reg_torch: the same through upstream's torch formulation (train.py:80-87),
      for comparison (single GPU only: it has no sharded form);
    * info_nce: InfoNCE loss forward + backward, partial scores all-reduced
      when sharded.
    Algorithmic bytes of the fused regulariser pass: reps read twice (forward,
    backward) and the gradient written once = 3 * B * V_s * 2 bytes."""
    from sparton_b200 import _lib, losses

    B = c["B"]
    gen = torch.Generator().manual_seed(7)
    q = (torch.rand(B, Vs, generator=gen) * 2).to(c["dtype"]).to(dev)
    d = (torch.rand(B, Vs, generator=gen) * 2).to(c["dtype"]).to(dev)
    V = c["V"]

    def reg():
        x = q.detach().requires_grad_(True)
        l1, fl = losses.regularizers(x, process_group=group, vocab_size=V)
        (l1 + fl).backward()

    def reg_torch():
        x = q.detach().requires_grad_(True)
        l1 = torch.mean(torch.sum(torch.abs(x), dim=-1))
        fl = torch.mean(torch.sum(x, dim=0) ** 2)
        (l1 + fl).backward()

    def nce():
        a, b_ = q.detach().requires_grad_(True), d.detach().requires_grad_(True)
        losses.info_nce_loss(a, b_, 1.0, process_group=group).backward()

    def timed(fn, n=20):
        for _ in range(3):
            fn()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(n)]
        barrier()
        for e0, e1 in evs:
            flush.zero_()
            preroll()
            e0.record(stream)
            fn()
            e1.record(stream)
        barrier()
        return max_over_ranks(sum(a.elapsed_time(e) for a, e in evs) / n)

    # The two regulariser kernels alone, through the C ABI (no autograd around them).
    lib = _lib.load()
    colsum = torch.empty(Vs, dtype=torch.float32, device=dev)
    pair = torch.empty(2, dtype=torch.float32, device=dev)
    gpair = torch.ones(2, dtype=torch.float32, device=dev)
    grad = torch.empty_like(q)
    ws = torch.zeros(lib.sparton_reg_workspace_size(B, Vs), dtype=torch.uint8, device=dev)
    sh, dt = stream.cuda_stream, _lib.DTYPE[c["dtype"]]

    def reg_kernels():
        _lib.check(lib.sparton_reg_fwd(q.data_ptr(), dt, B, Vs, 1.0 / B, 1.0 / V, colsum.data_ptr(),
                                       pair.data_ptr(), ws.data_ptr(), ws.numel(), sh), "reg_fwd")
        _lib.check(lib.sparton_reg_bwd(q.data_ptr(), colsum.data_ptr(), gpair.data_ptr(),
                                       gpair.data_ptr() + 4, 1.0 / B, 2.0 / V, dt, B, Vs,
                                       grad.data_ptr(), sh), "reg_bwd")

    out = {"shape": [B, Vs], "dtype": str(c["dtype"]).split(".")[-1]}
    out["reg_kernels_ms"] = round(timed(reg_kernels), 4)
    out["reg_fwd_bwd_ms"] = round(timed(reg), 4)
    out["reg_algorithmic_bytes"] = 3 * B * Vs * 2
    out["reg_kernels_gbs"] = round(out["reg_algorithmic_bytes"] / (out["reg_kernels_ms"] * 1e-3)
                                   / 1e9, 1)
    if world == 1:
        out["reg_torch_fwd_bwd_ms"] = round(timed(reg_torch), 4)
    out["info_nce_fwd_bwd_ms"] = round(timed(nce), 4)
    return out


def run_sparse(args, c, dev, group, world, Vs, flush, stream, barrier, max_over_ranks):
    """Sparse forms of the head's output for indexing (sparton_b200.sparse), on
    SPLADE-like reps of the workload's shape [B, V_s] (about half the entries
    zero), L2 flushed before every iteration, CUDA events, max over ranks:
    * csr_kernels: sparton_reps_csr with capacity B*V_s (one look-back kernel);
    * csr_api: sparse.reps_to_csr, which reads nnz back to size its output;
    * topk: sparton_reps_topk, k = 256.
    Algorithmic bytes: reps read once plus the output written (CSR: 6 bytes
    per kept 16-bit entry and the row pointers; top-k: 6 bytes per entry)."""
    from sparton_b200 import _lib, sparse

    B = c["B"]
    gen = torch.Generator().manual_seed(11)
    x = torch.log1p(torch.relu(torch.randn(B, Vs, generator=gen) * 2.0))
    x[torch.rand(B, Vs, generator=gen) < 0.5] = 0.0
    reps = x.to(c["dtype"]).to(dev)
    lib = _lib.load()
    sh, dt = stream.cuda_stream, _lib.DTYPE[c["dtype"]]
    es = reps.element_size()
    crow = torch.empty(B + 1, dtype=torch.int64, device=dev)
    cols = torch.empty(B * Vs, dtype=torch.int32, device=dev)
    vals = torch.empty(B * Vs, dtype=c["dtype"], device=dev)
    ws = torch.zeros(max(lib.sparton_sparse_workspace_size(B, Vs), 1), dtype=torch.uint8,
                     device=dev)
    k = min(256, Vs)
    tv = torch.empty(B, k, dtype=c["dtype"], device=dev)
    ti = torch.empty(B, k, dtype=torch.int32, device=dev)

    def csr_kernels():
        _lib.check(lib.sparton_reps_csr(reps.data_ptr(), dt, B, Vs, 0.0, crow.data_ptr(),
                                        cols.data_ptr(), vals.data_ptr(), B * Vs, ws.data_ptr(),
                                        ws.numel(), sh), "reps_csr")

    def topk():
        _lib.check(lib.sparton_reps_topk(reps.data_ptr(), dt, B, Vs, k, tv.data_ptr(),
                                         ti.data_ptr(), sh), "reps_topk")

    def timed(fn, n=20):
        for _ in range(3):
            fn()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(n)]
        barrier()
        for e0, e1 in evs:
            flush.zero_()
            preroll()
            e0.record(stream)
            fn()
            e1.record(stream)
        barrier()
        return max_over_ranks(sum(a.elapsed_time(e) for a, e in evs) / n)

    out = {"shape": [B, Vs], "dtype": str(c["dtype"]).split(".")[-1], "k": k}
    out["csr_kernels_ms"] = round(timed(csr_kernels), 4)
    nnz = int(crow[B].item())
    out["nnz"] = nnz
    out["csr_algorithmic_bytes"] = B * Vs * es + nnz * (4 + es) + (B + 1) * 8
    out["csr_gbs"] = round(out["csr_algorithmic_bytes"] / (out["csr_kernels_ms"] * 1e-3) / 1e9, 1)
    out["csr_api_ms"] = round(timed(lambda: sparse.reps_to_csr(reps)), 4)
    out["topk_ms"] = round(timed(topk), 4)
    out["topk_algorithmic_bytes"] = B * Vs * es + B * k * (4 + es)
    out["topk_gbs"] = round(out["topk_algorithmic_bytes"] / (out["topk_ms"] * 1e-3) / 1e9, 1)
    return out


def run_transform(args, c, dev, group, world, Vs, flush, stream, barrier, max_over_ranks):
    """The MLM transform in front of the head (sparton_b200.transform) at the
    workload's shape, L2 flushed before every iteration, CUDA events, max over
    ranks (single GPU: the projection's head is unsharded):
    * kernels_fwd / kernels_bwd: sparton_transform_fwd / _bwd alone (gelu +
      LayerNorm, and its backward with the d_gamma / d_beta / d_bias sums);
    * gemm_*: the dense layer's three products on the library's tcgen05 GEMM
      (y = x Wd^T + bd, dx = dy Wd, dWd = dy^T x; [B*S, D] x [D, D]) against
      torch's matmuls (cuBLAS), each alone;
    * projection: SpartonProjection forward + backward (the dense products on
      the tcgen05 GEMM, the transform kernels, the head), against
    * projection_torch_transform: the same with the transform as torch modules
      (nn.Linear, gelu, nn.LayerNorm: the reference's ProjectionSparton path).
    Algorithmic bytes of the transform kernels: forward reads y and writes h
    (2·B·S·D·2); backward reads dh and y and writes dy, the column sums
    coming from the same pass (3·B·S·D·2)."""
    from torch import nn

    from sparton_b200 import transform as tr

    B, S, D, V = c["B"], c["S"], c["D"], c["V"]
    dt = c["dtype"]
    gen = torch.Generator().manual_seed(13)
    x = torch.randn(B, S, D, generator=gen).to(dt).to(dev)
    y = (torch.randn(B, S, D, generator=gen) * 1.5).to(dt).to(dev)
    gamma = torch.ones(D, dtype=dt, device=dev)
    beta = torch.zeros(D, dtype=dt, device=dev)
    dh = torch.randn(B, S, D, generator=gen).to(dt).to(dev)
    _, mean, rstd = tr.transform_fwd_impl(y, gamma, beta, 1e-12)

    dense = nn.Linear(D, D).to(dev, dt)
    ln = nn.LayerNorm(D, eps=1e-12).to(dev, dt)
    decoder = nn.Linear(D, V, bias=c["bias"]).to(dev, dt)

    class Transform(nn.Module):  # the reference's RobertaTransform layout
        def __init__(self):
            super().__init__()
            self.dense, self.layer_norm = dense, ln

        def forward(self, t):
            return self.layer_norm(torch.nn.functional.gelu(self.dense(t)))

    ref_t = Transform()
    proj = tr.SpartonProjection(ref_t, decoder)
    mask = make_inputs(c)[3].to(dev)
    g = torch.randn(B, V, generator=gen).to(dt).to(dev)

    def projection():
        xi = x.detach().requires_grad_(True)
        proj(xi, mask).backward(g)

    def projection_torch_transform():
        xi = x.detach().requires_grad_(True)
        proj.sparton_head(ref_t(xi), mask).backward(g)

    def timed(fn, n=10):
        for _ in range(3):
            fn()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(n)]
        barrier()
        for e0, e1 in evs:
            flush.zero_()
            preroll()
            e0.record(stream)
            fn()
            e1.record(stream)
        barrier()
        return max_over_ranks(sum(a.elapsed_time(e) for a, e in evs) / n)

    es = torch.empty((), dtype=dt).element_size()
    out = {"shape": [B, S, D], "dtype": str(dt).split(".")[-1]}
    out["kernels_fwd_ms"] = round(timed(lambda: tr.transform_fwd_impl(y, gamma, beta, 1e-12)), 4)
    out["kernels_bwd_ms"] = round(timed(lambda: tr.transform_bwd_impl(dh, y, gamma, mean, rstd)), 4)
    out["kernels_fwd_gbs"] = round(2 * B * S * D * es / (out["kernels_fwd_ms"] * 1e-3) / 1e9, 1)
    out["kernels_bwd_gbs"] = round(3 * B * S * D * es / (out["kernels_bwd_ms"] * 1e-3) / 1e9, 1)
    # the dense layer's products alone: ours, then torch (cuBLAS)
    from sparton_b200.gemm import gemm
    x2, dy2 = x.view(-1, D), dh.view(-1, D)
    wd, bd = dense.weight.detach(), dense.bias.detach()
    flops = 2.0 * B * S * D * D
    for name, ours, ref in (
            ("y", lambda: gemm(x2, wd, bias=bd), lambda: torch.nn.functional.linear(x2, wd, bd)),
            ("dx", lambda: gemm(dy2, wd, b_t=True), lambda: dy2 @ wd),
            ("dw", lambda: gemm(dy2, x2, a_t=True, b_t=True), lambda: dy2.t() @ x2)):
        t_ours, t_ref = timed(ours), timed(ref)
        out[f"gemm_{name}_ms"] = round(t_ours, 4)
        out[f"gemm_{name}_torch_ms"] = round(t_ref, 4)
        out[f"gemm_{name}_tflops"] = round(flops / (t_ours * 1e-3) / 1e12, 1)
    if world == 1:
        out["projection_fwd_bwd_ms"] = round(timed(projection), 4)
        out["projection_torch_transform_fwd_bwd_ms"] = round(timed(projection_torch_transform), 4)
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="config2",
                    help="benchmark configuration (default config2, the one the metric is quoted on)")
    ap.add_argument("--cpu-rows", type=int, default=None,
                    help="rows of the CPU-baseline sample (default: per workload)")
    ap.add_argument("--nccl-priority", choices=["high", "normal"], default="high",
                    help="stream priority of the NCCL process group (N > 1)")
    ap.add_argument("--hidden-reduce", choices=["peer", "nccl", "rsag"], default="peer",
                    help="N > 1: sum of the partial d_hidden over NVLink peer memory (packed "
                         "rows only), NCCL all-reduce of all rows in chunks, or per chunk an "
                         "fp32 NCCL reduce-scatter and an all-gather of the parts rounded to "
                         "hidden's dtype (rsag)")
    ap.add_argument("--legs", default="device,e2e,cpu,losses,sparse,transform",
                    help="comma list of legs: device (value), e2e, cpu (baseline), losses "
                         "(training losses on the head's output), sparse (CSR / top-k of "
                         "reps), transform (MLM transform before the head); profiling runs "
                         "use --legs device")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    legs = set(args.legs.split(","))
    if "device" not in legs:
        ap.error("--legs must include device")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        ap.error(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    if args.impl == "reference":
        return run_reference_arm(args, rank)

    import datetime

    import torch.distributed as dist

    from sparton_b200 import _lib
    from sparton_b200.head import VocabShard, _HiddenGradReducer, row_chunks

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    group = None
    if world > 1:
        # High-priority NCCL streams: when a d_hidden chunk finishes, its
        # all-reduce gets SMs ahead of the next chunk's persistent gather kernel,
        # so the collectives overlap the remaining backward kernels.
        opts = dist.ProcessGroupNCCL.Options()
        opts.is_high_priority_stream = args.nccl_priority == "high"
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev,
                                pg_options=opts)
        group = dist.group.WORLD

    c = WORKLOADS[args.workload]
    B, S, D, V = c["B"], c["S"], c["D"], c["V"]
    H, W, b, mask, g, L = make_inputs(c)
    T = int(L.sum())
    shard = VocabShard(V, world, rank)
    Vs = shard.size
    Ws = W[shard.start:shard.stop].contiguous()
    bs = b[shard.start:shard.stop].contiguous() if b is not None else None
    gs = g[:, shard.start:shard.stop].contiguous()

    lib = _lib.load()
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream
    Hd, Wd, md, gd = H.to(dev), Ws.to(dev), mask.to(dev), gs.to(dev)
    bd = bs.to(dev) if bs is not None else None
    reps = torch.empty(B, Vs, dtype=c["dtype"], device=dev)
    idx = torch.empty(B, Vs, dtype=torch.int32, device=dev)
    dh_dtype = torch.float32 if world > 1 else c["dtype"]
    dH = torch.empty(B, S, D, dtype=c["dtype"], device=dev)  # single GPU; sharded: the reducer's
    dW = torch.empty(Vs, D, dtype=c["dtype"], device=dev)
    db = torch.empty(Vs, dtype=c["dtype"], device=dev) if bd is not None else None
    wsf = torch.empty(lib.sparton_fwd_workspace_size(B, S, D, Vs), dtype=torch.uint8, device=dev)
    wsb = torch.empty(lib.sparton_bwd_workspace_size(B, S, D, Vs), dtype=torch.uint8, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    dt = _lib.DTYPE[c["dtype"]]
    chunks = row_chunks(B, S * D * torch.empty((), dtype=dh_dtype).element_size())
    side = torch.cuda.Stream(dev)
    peer = None
    if world > 1 and args.hidden_reduce == "peer":
        from sparton_b200.peer import PeerHiddenReduce

        if not PeerHiddenReduce.usable(group, Hd):
            raise RuntimeError("--hidden-reduce peer needs every rank on one node's GPUs (<= 8)")
        peer = PeerHiddenReduce.get(group, dev, B * S, D, c["dtype"])
    import sparton_b200.head as head_mod

    # the e2e leg's SpartonHead does the same
    head_mod.HIDDEN_REDUCE = "nccl" if args.hidden_reduce == "rsag" else args.hidden_reduce
    head_mod.REDUCE_SCATTER_GATHER = args.hidden_reduce == "rsag"
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731

    # sharded backward phases of the timed steps (events on the streams that run
    # them): dH partial done, d_hidden reduction done, dW / db done
    phase_ev = []

    def step(k0=None, k1=None, ph=None):
        _lib.check(lib.sparton_mask_prepare(md.data_ptr(), 2, B, S, wsf.data_ptr(), wsf.numel(), sh),
                   "mask_prepare")
        if k0 is not None:
            k0.record(stream)
        _lib.check(lib.sparton_fwd_prepared(Hd.data_ptr(), Wd.data_ptr(), _lib.ptr(bd), dt, B, S, D,
                                            Vs, reps.data_ptr(), idx.data_ptr(), wsf.data_ptr(),
                                            wsf.numel(), sh), "fwd")
        if k1 is not None:
            k1.record(stream)
        if world == 1:
            # As the ops' backward does: the dH half on this stream, the dW / db
            # half on a side stream, joined before the step ends.
            side.wait_stream(stream)
            _lib.check(lib.sparton_bwd(gd.data_ptr(), reps.data_ptr(), idx.data_ptr(),
                                       Hd.data_ptr(), Wd.data_ptr(), dt, B, S, D, Vs,
                                       dH.data_ptr(), None, None,
                                       _lib.DTYPE[dh_dtype], dt, wsb.data_ptr(), wsb.numel(), sh),
                       "bwd dH")
            _lib.check(lib.sparton_bwd(gd.data_ptr(), reps.data_ptr(), idx.data_ptr(),
                                       Hd.data_ptr(), Wd.data_ptr(), dt, B, S, D, Vs,
                                       None, dW.data_ptr(), _lib.ptr(db),
                                       _lib.DTYPE[dh_dtype], dt, wsb.data_ptr(), wsb.numel(),
                                       side.cuda_stream), "bwd dW")
            stream.wait_stream(side)
            return
        if peer is not None:
            # SpartonHead's sharded backward with the peer reduction: the fp32
            # partial dH into this rank's peer buffer, then the sum of the
            # packed rows over NVLink into dH while dW / db run on a side stream.
            _lib.check(lib.sparton_bwd(gd.data_ptr(), reps.data_ptr(), idx.data_ptr(),
                                       Hd.data_ptr(), Wd.data_ptr(), dt, B, S, D, Vs,
                                       peer.partial(B, S).data_ptr(), None, None,
                                       _lib.DTYPE[torch.float32], dt, wsb.data_ptr(),
                                       wsb.numel(), sh), "bwd dH")
            if ph is not None:
                ph[0].record(stream)
            side.wait_stream(stream)
            _lib.check(lib.sparton_bwd(gd.data_ptr(), reps.data_ptr(), idx.data_ptr(),
                                       Hd.data_ptr(), Wd.data_ptr(), dt, B, S, D, Vs, None,
                                       dW.data_ptr(), _lib.ptr(db), _lib.DTYPE[dh_dtype], dt,
                                       wsb.data_ptr(), wsb.numel(), side.cuda_stream), "bwd dW")
            if ph is not None:
                ph[2].record(side)
            peer.reduce(wsf, B, S, dH)
            if ph is not None:
                ph[1].record(stream)
            stream.wait_stream(side)
            return
        # Sharded, with SpartonHead's sharded backward schedule: partial dH in
        # chunks of batch rows, each chunk all-reduced (fp32, NCCL's stream)
        # while the next chunk is computed, the last ones overlapping dW / db.
        red = _HiddenGradReducer(Hd, dh_dtype, group)
        for b0, b1 in red.chunks:
            dHp = red.partial
            _lib.check(lib.sparton_bwd(gd[b0:b1].data_ptr(), reps[b0:b1].data_ptr(),
                                       idx[b0:b1].data_ptr(), Hd[b0:b1].data_ptr(), Wd.data_ptr(),
                                       dt, b1 - b0, S, D, Vs, dHp[b0:b1].data_ptr(), None, None,
                                       _lib.DTYPE[dh_dtype], dt, wsb.data_ptr(), wsb.numel(), sh),
                       "bwd dH")
            red.reduce(b0, b1)
        if ph is not None:
            ph[0].record(stream)
        _lib.check(lib.sparton_bwd(gd.data_ptr(), reps.data_ptr(), idx.data_ptr(), Hd.data_ptr(),
                                   Wd.data_ptr(), dt, B, S, D, Vs, None, dW.data_ptr(),
                                   _lib.ptr(db), _lib.DTYPE[dh_dtype], dt, wsb.data_ptr(),
                                   wsb.numel(), sh), "bwd dW")
        if ph is not None:
            ph[2].record(stream)
        red.finish()
        if ph is not None:
            ph[1].record(stream)

    def barrier():
        if world > 1:
            dist.barrier(group=group, device_ids=[local_rank])
        torch.cuda.synchronize(dev)

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        return float(t.item())

    # ------------------------------------------------------------ device-resident
    for _ in range(args.warmup):
        flush.zero_()
        step()
    status = _lib.read_device_status(wsf)
    if status != 0:
        raise RuntimeError(f"forward kernel reported device status {status:#x}")
    step_ev = [(ev(), ev()) for _ in range(args.steps)]
    kern_ev = [(ev(), ev()) for _ in range(args.steps)]
    sampler = ClockSampler(dev)
    barrier()
    if world > 1:
        phase_ev = [(ev(), ev(), ev()) for _ in range(args.steps)]
    with sampler:
        for i in range(args.steps):
            flush.zero_()
            step_ev[i][0].record(stream)
            step(*kern_ev[i], ph=phase_ev[i] if phase_ev else None)
            step_ev[i][1].record(stream)
        barrier()
    bwd_phases = None
    if phase_ev:
        # from the end of the forward kernel: dH partial (dH gather and sort) done;
        # then from that point: the d_hidden reduction done, dW / db done
        n = args.steps
        bwd_phases = {
            "dh_partial_ms": round(max_over_ranks(
                sum(kern_ev[i][1].elapsed_time(phase_ev[i][0]) for i in range(n)) / n), 4),
            "reduce_after_dh_ms": round(max_over_ranks(
                sum(phase_ev[i][0].elapsed_time(phase_ev[i][1]) for i in range(n)) / n), 4),
            "dw_after_dh_ms": round(max_over_ranks(
                sum(phase_ev[i][0].elapsed_time(phase_ev[i][2]) for i in range(n)) / n), 4),
        }
    step_ms = max_over_ranks(sum(a.elapsed_time(e) for a, e in step_ev) / args.steps)
    kern_ms = sum(a.elapsed_time(e) for a, e in kern_ev) / args.steps
    kern_ms_max = max_over_ranks(kern_ms)
    # forward part (mask + pack prepare + forward kernel) and backward part
    # (sort, gathers [, all-reduce]) of the same timed steps
    fwd_part_ms = max_over_ranks(
        sum(step_ev[i][0].elapsed_time(kern_ev[i][1]) for i in range(args.steps)) / args.steps)
    bwd_part_ms = max_over_ranks(
        sum(kern_ev[i][1].elapsed_time(step_ev[i][1]) for i in range(args.steps)) / args.steps)
    # mask_prepare + pack_prepare + forward; backward: sort, dH gather, dW list,
    # dW gather (db, when there is a bias, is summed inside the dW gather);
    # sharded, a sort and a dH gather per chunk of batch rows.
    # sort: 3 kernels; dH and dW gathers; dW list; peer reduction: 4
    if world == 1:
        launches_per_step = 3 + 3 + 1 + 2
    elif peer is not None:
        launches_per_step = 3 + 3 + 1 + 2 + 4
    else:
        launches_per_step = 3 + len(chunks) * 4 + 2

    # ------------------------------------------------------------ inference forward
    # mask prepare + the forward without the argmax output (what SpartonHead
    # runs under no_grad), same inputs, L2 flushed before each call.
    inf_ev = [(ev(), ev()) for _ in range(args.steps)]
    for i in range(args.warmup + args.steps):
        flush.zero_()
        if i >= args.warmup:
            inf_ev[i - args.warmup][0].record(stream)
        _lib.check(lib.sparton_fwd(Hd.data_ptr(), Wd.data_ptr(), _lib.ptr(bd), md.data_ptr(), 2,
                                   dt, B, S, D, Vs, reps.data_ptr(), None, wsf.data_ptr(),
                                   wsf.numel(), sh), "fwd (inference)")
        if i >= args.warmup:
            inf_ev[i - args.warmup][1].record(stream)
    barrier()
    inf_ms = max_over_ranks(sum(a.elapsed_time(e) for a, e in inf_ev) / args.steps)

    # ------------------------------------------------------------ end to end
    e2e_ms = None
    if "e2e" in legs:
        e2e_ms = run_e2e(args, c, dev, group, W, b, H, mask, gs, Vs, flush, stream, barrier,
                         max_over_ranks)
        h2d, d2h = e2e_bytes(H, mask, gs, B, Vs, c["dtype"])

    losses_out = None
    if "losses" in legs:
        losses_out = run_losses(args, c, dev, group, world, Vs, flush, stream, barrier,
                                max_over_ranks)

    sparse_out = None
    if "sparse" in legs:
        sparse_out = run_sparse(args, c, dev, group, world, Vs, flush, stream, barrier,
                                max_over_ranks)

    transform_out = None
    if "transform" in legs:
        transform_out = run_transform(args, c, dev, group, world, Vs, flush, stream, barrier,
                                      max_over_ranks)

    # ------------------------------------------------------------ report
    peaks, peaks_src = load_peaks()
    fl = nominal_flops(c)
    value = fl / (step_ms * 1e-3) / 1e12
    alg_fwd = 2.0 * D * Vs * T  # this rank's forward launch
    alg_step = 2.0 * D * V * T + 4.0 * D * B * V  # the whole job's step
    achieved = alg_fwd / (kern_ms * 1e-3) / 1e12
    peak = float(peaks["bf16_tflops"])
    traffic = profile_traffic(args.workload) if world == 1 else None
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": DTYPE_NAME[c["dtype"]],
        "data": f"synthetic (seeded; benchmark {c['name'].split(' (')[0]} distributions)",
        "config": {"workload": workload_desc(c),
                   "B": B, "S": S, "D": D, "V": V, "valid_tokens": T,
                   "parallelism": f"vocab-sharded x{world}" if world > 1 else "single GPU",
                   "dh_reduce": (None if world == 1 else
                                 "peer (NVLink loads, packed rows)" if peer is not None else
                                 f"nccl all-reduce, {len(chunks)} chunks"),
                   "nccl_stream_priority": args.nccl_priority if world > 1 else None,
                   "l2": "flushed (256 MiB write) before every timed step"},
        "tokens_per_s": round(B * S / (step_ms * 1e-3), 1),
        "valid_tokens_per_s": round(T / (step_ms * 1e-3), 1),
        "algorithmic_tflops": round(alg_step / (step_ms * 1e-3) / 1e12, 2),
        # the whole step's algorithmic rate (valid tokens, 2·D·V·T forward +
        # 4·D·B·V backward) over the measured peak: north_star's "fwd+bwd
        # fraction of dense bf16 peak"; frac_of_bf16_peak_nominal counts padded
        # tokens and a dense backward and so exceeds 1
        "step_frac": round(alg_step / (step_ms * 1e-3) / 1e12 / peak, 4),
        "frac_of_bf16_peak_nominal": round(value / peak, 4),
        "fwd_kernel_ms": round(kern_ms_max, 4),
        "fwd_ms": round(fwd_part_ms, 4),
        "bwd_ms": round(bwd_part_ms, 4),
        "bwd_phases": bwd_phases,
        "fwd_inference_ms": round(inf_ms, 4),
        "roofline": {"kernel": "fwd_tc_kernel", "bound": "tensor", "achieved": round(achieved, 2),
                     "peak": peak, "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                     "frac_of_sustained": round(achieved / float(peaks["bf16_tflops_sustained"]), 4),
                     "peak_source": f"{peaks_src} bf16_tflops (burst)",
                     "algorithmic_flops_per_launch": alg_fwd, "traffic": traffic},
        "e2e": None if e2e_ms is None else {
            "value": round(fl / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
            "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "path": "SpartonHead forward + autograd backward; pinned host inputs copied in and reps copied out every step, double-buffered on copy streams"},
        "losses": losses_out,
        "sparse": sparse_out,
        "transform": transform_out,
        "gpu_launches": launches_per_step * args.steps + 2 * args.steps,
        "clocks": sampler.summary(),
    }
    if rank == 0 and world == 1 and "cpu" in legs:
        try:
            # A bounded run of the same per-step work as the reference arm
            # (--impl reference): whole batch where it fits, same inputs.
            # Three warm-up steps, as the reference arm takes at its minimum
            # --warmup: the first steps of the CPU head fault in its buffers.
            res = cpu_baseline(c, cpu_rows_for(c, args.cpu_rows), steps=3, warmup=3)
            line["cpu_baseline"] = {k: res[k] for k in ("value", "unit", "cores", "kind", "sample",
                                                        "cpu_model")}
        except Exception as e:  # pragma: no cover
            line["cpu_baseline"] = {"error": repr(e)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(group=group, device_ids=[local_rank])
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

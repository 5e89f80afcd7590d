"""Benchmark of the quantized DiT linear path on B200 - one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload dit|gemm|fp8|elementwise] [--impl ours|reference]

Workloads (synthetic, seeded; the reference publishes no dataset for this path):
  dit          BASELINE config 5: one denoise step of a 40-block Hy-Nomas-style DiT (hidden 4096, 32 x 128
               heads, MLP 16384, adaLN modulation, W8A8 int8 linears with per-channel weight scales), L =
               20240 tokens, batch 1, sequence-parallel over the ranks (per-block K/V all-gather over NCCL).
               metric: tokens/s of the whole job; roofline: the W8A8 GEMM kernel inside the step.
  gemm         BASELINE config 1 shape: W8A8 int8 linear 4096 x 4096 x 4096 (quantize + GEMM), per-128-group
               activation scales and per-channel weight scales; ranks each run their own rows (replicas).
  fp8          BASELINE config 2: FP8 e4m3 block-scaled GEMM, MLP-up 16384 x 4096 at M = 20240.
  elementwise  BASELINE config 3: LayerNorm + modulate + int8 quantize at M = 20240, D = 4096.

Timing: W warm-up steps, then exactly K steps between a barrier + cuda.synchronize on both sides, CUDA
events on the launching stream, max over ranks. Inputs rotate over buffer sets larger than L2 (126 MB)
so no step reads the previous step's data from L2. `e2e` repeats the step through the public API with
the step's inputs copied from pinned host memory and its result read back inside the timed region.
`--impl reference` times the reference's own CPU path for the same workload (the torch arithmetic it runs
when the input is not on CUDA, restated in oracle/torch_ref.py) on this host's cores.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "comfyui-hy-nomas_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

L2_BYTES = 126 * 2 ** 20


# --------------------------------------------------------------------------------------------------------
# infrastructure


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while the timed region runs."""
    FIELDS = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_ids):
        self.bus_ids = {b.lower()[-12:] for b in bus_ids}
        self.rows = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 10:
                self.rows.append(parts)

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = [r for r in self.rows if not self.bus_ids or r[1].lower()[-12:] in self.bus_ids] or self.rows
        if not rows:
            return None
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[6 + i].lower().startswith("active")})
        loaded = [s for s in sm if mx and s > 0.3 * max(mx)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def init_dist(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        import datetime
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=120))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        dist.barrier()


def max_over_ranks(value, world):
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value, world):
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def timed_steps(step, steps, warmup, world, stream):
    """Warm up, then time exactly `steps` calls of step(i) with CUDA events on `stream` (ms, max over ranks)."""
    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(steps):
        step(warmup + i)
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    return max_over_ranks(start.elapsed_time(end), world)


class KernelTimer:
    """CUDA events around individual launches of one kernel inside the timed region."""

    def __init__(self, stream):
        self.stream = stream
        self.pairs = []
        self.active = False

    def wrap(self, fn):
        if not self.active:
            return fn()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(self.stream)
        out = fn()
        b.record(self.stream)
        self.pairs.append((a, b))
        return out

    def mean_ms(self):
        if not self.pairs:
            return None
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in self.pairs) / len(self.pairs)


def cpu_threads():
    return len(os.sched_getaffinity(0)), torch.get_num_threads()


# --------------------------------------------------------------------------------------------------------
# workloads


def make_int8_weight(n, k, gen, device, per_channel=True):
    """Random int8 codes uniform in [-127, 127] and per-output-channel scales U[1e-3, 5e-3] (BASELINE config
    1), broadcast to the reference's [N, K/128] layout when per_channel is False."""
    q = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    s = torch.rand(n, generator=gen) * 4e-3 + 1e-3
    if not per_channel:
        s = s[:, None].expand(n, k // 128).contiguous()
    return q.to(device), s.to(device)


def outlier_activations(m, k, gen):
    """x ~ N(0, 1) with 1% of the channels scaled x20."""
    x = torch.randn(m, k, generator=gen)
    x[:, torch.randperm(k, generator=gen)[: max(1, k // 100)]] *= 20.0
    return x.bfloat16()


def workload_gemm(args, world, rank, stream, pk):
    from hy_nomas_b200 import kernels
    m, n, k = 4096, 4096, 4096
    gen = torch.Generator().manual_seed(1234 + rank)
    dev = torch.device("cuda")
    set_bytes = m * k * 2 + m * k + n * k + m * n * 2   # x, codes, weight, out
    nsets = max(2, -(-3 * L2_BYTES // set_bytes))
    xs = [outlier_activations(m, k, gen).to(dev) for _ in range(nsets)]
    ws = [make_int8_weight(n, k, gen, dev) for _ in range(nsets)]
    bias = (torch.randn(n, generator=gen) * 0.02).bfloat16().to(dev)
    timer = KernelTimer(stream)

    def step(i):
        x = xs[i % nsets]
        qw, sw = ws[i % nsets]
        qa, sa = kernels.quantize_activations(x)
        return timer.wrap(lambda: kernels.block_gemm(qa, sa, qw, sw, bias))

    ms = timed_steps(step, args.steps, args.warmup, world, stream)
    timer.active = True
    timed_steps(step, args.steps, 0, world, stream)
    gemm_ms = timer.mean_ms()
    ops = 2.0 * m * n * k
    total_ops = sum_over_ranks(ops * args.steps, world)
    value = total_ops / (ms * 1e-3) / 1e12
    # e2e through the public API: x from pinned host memory, y read back, every step
    xh = [x.cpu().pin_memory() for x in xs[:2]]
    yh = torch.empty((m, n), dtype=torch.bfloat16).pin_memory()

    def e2e_step(i):
        x = xh[i % 2].to(dev, non_blocking=True)
        qw, sw = ws[i % nsets]
        y = kernels.int8_g128_linear(x, qw, sw, bias)
        yh.copy_(y, non_blocking=True)

    e2e_ms = timed_steps(e2e_step, args.steps, 2, world, stream)
    e2e = {"value": round(total_ops / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TOPS",
           "h2d_bytes_per_step": m * k * 2, "d2h_bytes_per_step": m * n * 2}
    peak = 2.0 * pk["bf16_tflops"]
    achieved = ops / (gemm_ms * 1e-3) / 1e12
    roof = {"kernel": "hn::gemm::k_block_gemm<int8, per-channel weights>", "bound": "tensor",
            "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TOPS", "frac": round(achieved / peak, 4),
            "peak_note": f"int8 dense = 2 x {pk['source']} bf16 burst ({pk['bf16_tflops']} TFLOP/s)",
            "traffic": traffic_for("gemm"), "algorithmic_bytes": m * k + n * k + m * n * 2 + m * 4 * (k // 128)}
    out = dict(metric="W8A8 GEMM TOPS", value=round(value, 2), unit="TOPS", ms_per_step=round(ms / args.steps, 4),
               higher_is_better=True, scaling="weak", dtype="int8",
               config={"workload": "w8a8_linear_4096x4096x4096 (config 1 shape): quantize + block-scaled GEMM",
                       "M": m, "N": n, "K": k, "activation_scales": "per token x 128 channels",
                       "weight_scales": "per output channel", "l2": f"inputs rotate over {nsets} sets > L2",
                       "parallelism": f"replicas x{world}"},
               e2e=e2e, roofline=roof, gpu_launches=2 * args.steps)
    out["config"]["kernel_variants_tops"] = gemm_variants(m, n, k, stream)
    out["cpu_baseline_fn"] = lambda: cpu_baseline_gemm(m, n, k)
    return out


def gemm_variants(m, n, k, stream, iters=20):
    """Context for the roofline (not the headline): the GEMM kernel alone in each scale mode, and cuBLASLt's
    int8 GEMM (torch._int_mm, no scaling) on the same shape."""
    from hy_nomas_b200 import kernels
    gen = torch.Generator().manual_seed(99)
    dev = torch.device("cuda")
    qa = torch.randint(-127, 128, (m, k), generator=gen, dtype=torch.int8).to(dev)
    qw = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8).to(dev)
    sa_g = (torch.rand(m, k // 128, generator=gen) * 0.02).to(dev)
    sa_r = (torch.rand(m, generator=gen) * 0.02).to(dev)
    sw_g = (torch.rand(n, k // 128, generator=gen) * 4e-3).to(dev)
    sw_r = (torch.rand(n, generator=gen) * 4e-3).to(dev)
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev)
    cases = {"a_group_w_group": lambda: kernels.block_gemm(qa, sa_g, qw, sw_g),
             "a_group_w_channel": lambda: kernels.block_gemm(qa, sa_g, qw, sw_r),
             "a_token_w_channel": lambda: kernels.block_gemm(qa, sa_r, qw, sw_r),
             "cublaslt_int8_int32": lambda: torch._int_mm(qa, qw.t())}
    res = {}
    for name, fn in cases.items():
        try:
            fn()
            times = []
            for _ in range(iters):
                flush.zero_()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                fn()
                b.record(stream)
                b.synchronize()
                times.append(a.elapsed_time(b))
            res[name] = round(2.0 * m * n * k / (statistics.median(times) * 1e-3) / 1e12, 1)
        except RuntimeError as e:
            res[name] = f"unavailable: {str(e).splitlines()[0][:80]}"
    return res


def traffic_for(workload):
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            t = json.load(f)
        return t.get(workload)
    return None


def cpu_baseline_gemm(m, n, k, budget_s=10.0):
    """The reference's CPU path (dequantize_g128 + bf16 F.linear, hy_nomas/ops.py:175-176) on a bounded
    sample of rows, on all host threads."""
    from oracle import torch_ref
    gen = torch.Generator().manual_seed(5)
    rows = 512
    x = outlier_activations(rows, k, gen)
    q, s = make_int8_weight(n, k, gen, "cpu", per_channel=False)
    bias = (torch.randn(n, generator=gen) * 0.02).bfloat16()
    torch_ref.int8_linear_cpu(x, q, s, bias)
    t0 = time.perf_counter()
    it = 0
    while True:
        torch_ref.int8_linear_cpu(x, q, s, bias)
        it += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = (time.perf_counter() - t0) / it
    cores, threads = cpu_threads()
    return {"value": round(2.0 * rows * n * k / dt / 1e12, 4), "unit": "TOPS", "cores": threads, "kind": "port",
            "sample": f"{rows} x {k} -> {n} rows of the workload, {it} iterations in {budget_s:.0f}+ s "
                      f"(dequantize_g128 + bf16 F.linear, torch {torch.__version__}, {threads} threads on "
                      f"{cores} cores)"}


WORKLOADS = {"gemm": workload_gemm}


def run_reference(args, world, rank):
    """The reference's CPU path for the same workload and metric, rank 0 only."""
    if rank != 0:
        return None
    if args.workload != "gemm":
        raise SystemExit(f"--impl reference: workload {args.workload} not wired yet")
    m, n, k = 4096, 4096, 4096
    from oracle import torch_ref
    gen = torch.Generator().manual_seed(5)
    rows = 1024
    x = outlier_activations(rows, k, gen)
    q, s = make_int8_weight(n, k, gen, "cpu", per_channel=False)
    bias = (torch.randn(n, generator=gen) * 0.02).bfloat16()
    for _ in range(args.warmup):
        torch_ref.int8_linear_cpu(x, q, s, bias)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        torch_ref.int8_linear_cpu(x, q, s, bias)
    dt = time.perf_counter() - t0
    value = 2.0 * rows * n * k * args.steps / dt / 1e12
    cores, threads = cpu_threads()
    sample = f"{rows} of {m} rows per step (dequantize_g128 + bf16 F.linear on CPU, {threads} threads)"
    return dict(metric="W8A8 GEMM TOPS", value=round(value, 4), unit="TOPS", n_gpus=world, steps=args.steps,
                warmup=args.warmup, ms_per_step=round(dt / args.steps * 1e3, 3), higher_is_better=True,
                scaling="weak", vs_baseline=None, dtype="int8", data="synthetic",
                config={"workload": "w8a8_linear_4096x4096x4096 (config 1 shape)", "M": m, "N": n, "K": k},
                impl="reference",
                cpu_baseline={"value": round(value, 4), "unit": "TOPS", "cores": threads, "kind": "port",
                              "sample": sample},
                e2e={"value": round(value, 4), "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="gemm", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = init_dist(args)
    if args.impl == "reference":
        line = run_reference(args, world, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return
    pk = peaks()
    stream = torch.cuda.current_stream()
    props = torch.cuda.get_device_properties(torch.cuda.current_device())
    bus = getattr(props, "pci_bus_id", None)
    sampler = ClockSampler([f"{getattr(props, 'pci_domain_id', 0):08x}:{bus:02x}:00.0"] if bus is not None else [])
    if rank == 0:
        sampler.start()
    res = WORKLOADS[args.workload](args, world, rank, stream, pk)
    clocks = sampler.stop() if rank == 0 else None
    cpu_fn = res.pop("cpu_baseline_fn", None)
    if rank == 0:
        line = {"metric": res["metric"], "value": res["value"], "unit": res["unit"], "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
                "higher_is_better": res["higher_is_better"], "scaling": res["scaling"], "vs_baseline": None,
                "dtype": res["dtype"], "data": "synthetic (seeded)", "config": res["config"], "e2e": res["e2e"],
                "roofline": res["roofline"], "gpu_launches": res["gpu_launches"], "clocks": clocks}
        if world == 1 and cpu_fn is not None and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_fn()
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Benchmark of the quantized DiT linear path on B200 - one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload dit|dit_gemms|attention|gemm|fp8|elementwise]
                    [--impl ours|reference]

Workloads (synthetic, seeded; the reference publishes no dataset for this path):
  dit          (default) benchmark config 5: one denoise step of a 40-block Hy-Nomas-style DiT (hidden 4096,
               32 x 128 heads, MLP 16384, adaLN modulation, W8A8 int8 linears with per-channel weight scales),
               L = 20240 tokens, batch 1, sequence-parallel over the ranks (per-block K/V all-gather over
               NCCL). metric: tokens/s of the whole job (strong scaling); roofline: the W8A8 GEMM kernel
               inside the step.
  dit_gemms    benchmark config 4's linears: the block's five W8A8 GEMMs at M = 20240 (v, q|k, proj, fc1 with
               the GELU + requantization epilogue, fc2); metric TOPS; the profiling target of their ncu summary.
  gemm         benchmark config 1: W8A8 int8 linear 4096 x 4096 x 4096 (quantize + GEMM), per-128-group
               activation scales and per-channel weight scales; every rank runs its own copy (replicas).
  fp8          benchmark config 2: FP8 e4m3 block-scaled linear, MLP-up 16384 x 4096 at M = 20240 (quantize +
               GEMM); the config's 12-shape sweep is reported per kernel in `config`.
  elementwise  benchmark config 3: the fused elementwise chain at M = 20240, D = 4096 (LN + modulate + int8
               quantize; QK-RMSNorm + 3-D RoPE of q and k; gated residual; residual + LN + quantize).

Timing: W warm-up steps, then exactly K steps between a barrier + cuda.synchronize on both sides, CUDA
events on the launching stream, max over ranks. Every step reads more than L2 (126 MB) before it reuses an
input (inputs rotate over sets larger than L2, or - the DiT step - 12 GB of weights stream through between
reuses). `e2e` repeats the step through the public API with the step's inputs copied from pinned host
memory and its result read back inside the timed region. `--impl reference` times the reference's own CPU
path for the same workload (the torch arithmetic it runs when the input is not on CUDA, restated in
oracle/torch_ref.py) on this host's cores, rank 0 only.
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
MB = 1e6


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

    def __init__(self, bus_ids, enabled=True):
        self.bus_ids = {b.lower()[-12:] for b in bus_ids}
        self.rows = []
        self.proc = None
        self.thread = None
        self.enabled = enabled
        self.result = None

    def start(self):
        if not self.enabled:
            return
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
        self.proc = None
        rows = [r for r in self.rows if not self.bus_ids or r[1].lower()[-12:] in self.bus_ids] or self.rows
        if not rows:
            return None
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[6 + i].lower().startswith("active")})
        loaded = [s for s in sm if mx and s > 0.3 * max(mx)] or sm
        self.result = {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                       "reasons": reasons, "samples": len(rows)}
        return self.result


def init_dist():
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


def timed_steps(step, steps, warmup, world, stream, sampler=None):
    """Warm up, then time exactly `steps` calls of step(i) with CUDA events on `stream` (ms, max over ranks).
    `sampler` (rank 0's clock sampler) runs from the warm-up to the end of the timed region."""
    if sampler is not None:
        sampler.start()
    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")   # lets a profiler filter the timed steps (ncu --nvtx-include timed/)
    start.record(stream)
    for i in range(steps):
        step(warmup + i)
    end.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    if sampler is not None:
        sampler.stop()
    barrier(world)
    torch.cuda.synchronize()
    return max_over_ranks(start.elapsed_time(end), world)


class KernelTimer:
    """CUDA events around individual launches inside the timed region, with a per-launch work count."""

    def __init__(self, stream):
        self.stream = stream
        self.pairs = []
        self.active = False

    def wrap(self, fn, work=0.0):
        if not self.active:
            return fn()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(self.stream)
        out = fn()
        b.record(self.stream)
        self.pairs.append((a, b, work))
        return out

    def total_ms(self):
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b, _ in self.pairs)

    def mean_ms(self):
        return self.total_ms() / len(self.pairs) if self.pairs else None

    def work(self):
        return sum(w for _, _, w in self.pairs)


def cpu_threads():
    return len(os.sched_getaffinity(0)), torch.get_num_threads()


def traffic_for(workload):
    """DRAM bytes per launch of the workload's dominant kernel, from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f).get(workload)
    return None


def launch_count(fn):
    """Library calls (kernel launches) made by one call of fn."""
    from hy_nomas_b200 import _lib
    c0 = _lib.calls
    fn()
    return _lib.calls - c0


# --------------------------------------------------------------------------------------------------------
# synthetic inputs


def make_int8_weight(n, k, gen, device, per_channel=True):
    """Random int8 codes uniform in [-127, 127] and per-output-channel scales U[1e-3, 5e-3] (benchmark config
    1), broadcast to the reference's [N, K/128] layout when per_channel is False."""
    q = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    s = torch.rand(n, generator=gen) * 4e-3 + 1e-3
    if not per_channel:
        s = s[:, None].expand(n, k // 128).contiguous()
    return q.to(device), s.to(device)


def outlier_activations(m, k, gen):
    """x ~ N(0, 1) with 1% of the channels scaled x20 (benchmark config 1)."""
    x = torch.randn(m, k, generator=gen)
    x[:, torch.randperm(k, generator=gen)[: max(1, k // 100)]] *= 20.0
    return x.bfloat16()


# --------------------------------------------------------------------------------------------------------
# dit (config 5)


# the benchmark's DiT (config 5), stated here so the CPU reference arm needs nothing from the product package
DIT = dict(hidden=4096, heads=32, mlp=16384, blocks=40, rope_dims=(16, 56, 56), theta=10000.0, grid=(23, 22, 40))
DIT_TOKENS = 23 * 22 * 40
DIT_WARM_TOKENS = 512   # the CPU arm's extra warm-up blocks run on this many tokens


def workload_dit(args, world, rank, stream, pk, sampler):
    from hy_nomas_b200 import kernels
    from hy_nomas_b200.dit import CudaOps, DiTConfig, SyntheticDiT
    from hy_nomas_b200.sequence_parallel import SequenceParallel
    cfg = DiTConfig()
    sp = SequenceParallel()
    model = SyntheticDiT(cfg, device="cuda", seed=0, sp=sp)
    lo, hi = model.token_range
    L, d = cfg.tokens, cfg.hidden
    gen = torch.Generator(device="cuda").manual_seed(1000)
    x_full = torch.randn(1, L, d, generator=gen, device="cuda").to(torch.bfloat16)
    x = x_full[:, lo:hi].contiguous()
    vec = torch.randn(1, d, generator=gen, device="cuda").to(torch.bfloat16)

    def step(i):
        return model(x, vec)

    ms = timed_steps(step, args.steps, args.warmup, world, stream, sampler)

    # one instrumented step: CUDA events around every GEMM and attention call, and the launch count
    gemm_t, attn_t = KernelTimer(stream), KernelTimer(stream)
    gemm_t.active = attn_t.active = True
    orig_gemm, orig_attn = kernels.block_gemm, CudaOps.attention

    def gemm_wrap(qa, sa, qw, sw, *a, **kw):
        return gemm_t.wrap(lambda: orig_gemm(qa, sa, qw, sw, *a, **kw), 2.0 * qa.shape[0] * qw.shape[0] * qa.shape[1])

    def attn_wrap(q, k, v):
        return attn_t.wrap(lambda: orig_attn(q, k, v), 4.0 * q.shape[0] * q.shape[1] * k.shape[1] * q.shape[2] * q.shape[3])

    # the exchange waits (flag waits of the copy-engine exchanges, NCCL handle waits): how long the stream sat
    # waiting for the peers' data in the instrumented step
    from hy_nomas_b200 import sequence_parallel as sp_mod
    wait_t = KernelTimer(stream)
    wait_t.active = world > 1
    restore = []
    for cls in (sp_mod.PeerExchange, sp_mod.HeadExchange, sp_mod.HeadCollective):
        def timed_wait(self, *a, _orig=cls.wait, **kw):
            return wait_t.wrap(lambda: _orig(self, *a, **kw))
        restore.append((cls, "wait", cls.__dict__["wait"]))
        cls.wait = timed_wait
    orig_gather_wait = sp_mod.SequenceParallel.wait
    restore.append((sp_mod.SequenceParallel, "wait", sp_mod.SequenceParallel.__dict__["wait"]))
    sp_mod.SequenceParallel.wait = staticmethod(lambda *h: wait_t.wrap(lambda: orig_gather_wait(*h)))
    kernels.block_gemm, CudaOps.attention = gemm_wrap, staticmethod(attn_wrap)
    try:
        barrier(world)
        launches = launch_count(lambda: step(0))
        torch.cuda.synchronize()
    finally:
        kernels.block_gemm, CudaOps.attention = orig_gemm, staticmethod(orig_attn)
        for cls, name, orig in restore:
            setattr(cls, name, orig)
    gemm_ms, attn_ms = gemm_t.total_ms(), attn_t.total_ms()
    wait_ms = wait_t.total_ms()
    wait_max = max_over_ranks(wait_ms, world)
    gemm_ops, attn_flops = gemm_t.work(), attn_t.work()

    # e2e through the public API: this rank's tokens and vec from pinned host memory, the output read back
    xh, vh = x.cpu().pin_memory(), vec.cpu().pin_memory()
    yh = torch.empty_like(xh).pin_memory()

    def e2e_step(i):
        y = model(xh.to("cuda", non_blocking=True), vh.to("cuda", non_blocking=True))
        yh.copy_(y, non_blocking=True)

    e2e_ms = timed_steps(e2e_step, args.steps, 1, world, stream)
    check = sp_output_check(model, x_full, x, vec, world) if world > 1 else None
    tokens = L * args.steps
    value = tokens / (ms * 1e-3)
    int8_peak = 2.0 * pk["bf16_tflops_sustained"]
    achieved = gemm_ops / (gemm_ms * 1e-3) / 1e12
    step_ms = ms / args.steps
    roof = {"kernel": "hn::gemm::k_block_gemm<int8, group activation scales, per-channel weights> (all GEMMs of a "
                      "step)", "bound": "tensor", "achieved": round(achieved, 1), "peak": round(int8_peak, 1),
            "unit": "TOPS", "frac": round(achieved / int8_peak, 4),
            "peak_note": f"int8 dense = 2 x {pk['source']} bf16 sustained ({pk['bf16_tflops_sustained']} TFLOP/s); "
                         "the GEMMs run inside a long step",
            "traffic": dit_gemm_traffic(cfg, hi - lo), "gemm_ops_per_step_rank": gemm_ops}
    config = {"workload": "dit_step_40x_hidden4096_L20240 (config 5): 40 DiT blocks, SDPA attention, W8A8 linears",
              "model": "synthetic Hy-Nomas-style DiT (random init, seeded)", "global_batch": 1, "seq_len": L,
              "tokens_per_rank": hi - lo, "blocks": cfg.blocks, "hidden": d, "heads": cfg.heads, "mlp": d * cfg.mlp_ratio,
              "activation_scales": "per token x 128 channels", "weight_scales": "per output channel",
              "parallelism": f"sp{world} (sequence-parallel; weights replicated)",
              "sp_exchange": {"tokens-ce": "token split: K/V slices pushed by the copy engines over NVLink into "
                                           "CUDA-IPC-mapped peer buffers, flag-gated",
                              "tokens-nccl": "token split: NCCL all-gather of K/V",
                              "heads-ce": "head split: every rank attends for heads/N heads over all tokens; Q/K/V "
                                          "head groups and the output rows pushed by the copy engines (strided DMA) "
                                          "into CUDA-IPC-mapped peer buffers, flag-gated",
                              "heads-collective": "head split: Q/K/V and output exchanged by NCCL all-to-all",
                              "none": "none (one rank)"}[sp.split_name(cfg.heads)],
              "l2": "12 GB of weights stream through L2 between reuses of a step's input",
              "step_breakdown_ms_rank0": {"gemm": round(gemm_ms, 2), "attention": round(attn_ms, 2),
                                          "other": round(max(step_ms - gemm_ms - attn_ms, 0.0), 2),
                                          "of_other_exchange_wait": round(wait_ms, 2)},
              "exchange_wait_ms_per_step": {"rank0": round(wait_ms, 2), "max_over_ranks": round(wait_max, 2),
                                            "waits": len(wait_t.pairs),
                                            "what": "CUDA events around each wait for the peers' data (flag wait "
                                                    "or NCCL handle) in one instrumented step: exposed exchange "
                                                    "plus the wait for slower ranks"},
              "attention_tflops": round(attn_flops / (attn_ms * 1e-3) / 1e12, 1) if attn_ms else None,
              "floor_ms_rank0": {"gemm_at_int8_peak": round(gemm_ops / (int8_peak * 1e12) * 1e3, 2),
                                 "attention_at_bf16_peak": round(attn_flops / (pk["bf16_tflops_sustained"] * 1e12) * 1e3, 2)},
              "modulation_gemv": modulation_context(model, vec, stream, pk)}
    if check is not None:
        config["sp_output_check"] = check
    if not args.no_context:
        config["segment2_with_int8_history"] = segment2_context(model, vec, world, stream)
    if world == 1 and not args.no_context:
        config["configs_1_to_3"] = path_context(stream, pk)
        config["attention_kernel"] = attention_context(stream, pk)
    sp.close()
    return dict(metric="DiT denoise step tokens/s (40 blocks, 20240 tokens)", value=round(value, 1), unit="tokens/s",
                ms_per_step=round(step_ms, 3), higher_is_better=True, scaling="strong", dtype="int8 (GEMMs), bf16",
                config=config,
                e2e={"value": round(tokens / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                     "h2d_bytes_per_step": int(sum_over_ranks(xh.numel() * 2 + vh.numel() * 2, world)),
                     "d2h_bytes_per_step": int(sum_over_ranks(yh.numel() * 2, world))},
                roofline=roof, gpu_launches=launches * args.steps,
                cpu_baseline_fn=lambda: cpu_baseline_dit())


def sp_output_check(model, x_full, x, vec, world, tol=1e-2):
    """Every rank also runs the whole sequence on its own GPU (no sequence parallelism, the same weights) and
    compares its own tokens of that result with the sequence-parallel output: the largest rel-L2 over ranks and
    the number of ranks whose tokens are bit-identical. Attention over the gathered K/V may pick other kernel
    tilings for fewer queries, and a few quantization codes downstream can move with it, hence a tolerance."""
    from hy_nomas_b200.sequence_parallel import SequenceParallel
    y_sp = model(x, vec)
    single = model.replica(SequenceParallel(local=True))
    y_one = single(x_full, vec)
    lo, hi = model.token_range
    ref = y_one[:, lo:hi].float()
    err = (torch.linalg.vector_norm(y_sp.float() - ref) / torch.linalg.vector_norm(ref).clamp_min(1e-30)).item()
    same = 1.0 if torch.equal(y_sp.view(torch.int16), y_one[:, lo:hi].view(torch.int16)) else 0.0
    finite = 1.0 if bool(torch.isfinite(y_sp).all()) else 0.0
    err_max = max_over_ranks(err, world)
    n_same = int(sum_over_ranks(same, world))
    n_finite = int(sum_over_ranks(finite, world))
    del single, y_one
    torch.cuda.empty_cache()
    return {"against": "the same tokens computed on one GPU without sequence parallelism, on every rank",
            "rel_l2_max_over_ranks": float(f"{err_max:.3e}"), "bit_identical_ranks": n_same, "ranks": world,
            "finite_ranks": n_finite, "tolerance": tol, "pass": bool(err_max <= tol and n_finite == world)}


def segment2_context(model, vec, world, stream, steps=5, history_frames=18):
    """The world model's second segment (hy_nomas/model.py:199-209, world.py:197-204): the 23 latent frames of the
    benchmark grid split into 18 frames of history and 5 current frames. A cache pass over the history frames
    (every block's K quantized inside the QK-norm kernel, V by the KV quantizer) writes the int8 K/V cache of
    each block - on every rank the whole history, as a world's staged history is replicated. The timed step
    runs the 5 current frames (sharded over the ranks), each block dequantizing its history into the front of
    its K/V buffers and attending over history + current."""
    from hy_nomas_b200.sequence_parallel import SequenceParallel
    t, gh, gw = model.cfg.grid
    d = model.cfg.hidden
    cache_model = model.replica(sp=SequenceParallel(local=True), grid=(history_frames, gh, gw), t_offset=0)
    gen = torch.Generator(device="cuda").manual_seed(2000)
    xh = torch.randn(1, cache_model.cfg.tokens, d, generator=gen, device="cuda").to(torch.bfloat16)
    history = []
    cache_model(xh, vec, capture=history)
    del xh, cache_model
    seg = model.replica(grid=(t - history_frames, gh, gw), t_offset=history_frames)
    lo, hi = seg.token_range
    x = torch.randn(1, seg.cfg.tokens, d, generator=gen, device="cuda").to(torch.bfloat16)[:, lo:hi].contiguous()
    ms = timed_steps(lambda i: seg(x, vec, history=history), steps, 3, world, stream)
    lh = history[0][0].shape[0]
    hist_bytes = sum(c[0].numel() + c[2].numel() + 4 * (c[1].numel() + c[3].numel()) for c in history)
    del history
    torch.cuda.empty_cache()
    return {"current_tokens": seg.cfg.tokens, "history_tokens": lh, "ms_per_step": round(ms / steps, 3),
            "current_tokens_per_s": round(seg.cfg.tokens * steps / (ms * 1e-3), 1),
            "int8_history_bytes": hist_bytes,
            "note": "40 blocks; every block attends over its dequantized int8 history followed by the current "
                    "tokens' K/V; the history is built by a cache pass on each rank"}


def modulation_context(model, vec, stream, pk, iters=10):
    """The step's stacked modulation linear (every block's Modulate(vec), one [blocks x 6D, D] int8 linear at
    M = 1): its time and the weight bandwidth it reaches (a GEMV reads every weight byte once)."""
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device="cuda")
    t = _time_kernel(lambda: model.modulations(vec), stream, flush, iters)
    w = model.mod_all
    nbytes = w.q.numel() + w.s.numel() * 4 + w.bias.numel() * 2
    return {"ms": round(t, 4), "weight_bytes": nbytes, "gbs": round(nbytes / (t * 1e-3) / 1e9, 1),
            "frac_of_hbm": round(nbytes / (t * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
            "shape": f"1 x {w.q.shape[0]} x {w.q.shape[1]} (quantize + GEMM, timed together)"}


def dit_gemm_traffic(cfg, tokens):
    """DRAM bytes of all GEMM launches of one step on this rank, from the committed per-shape ncu captures
    (profiles/traffic.json "dit_gemm_shapes": bytes per launch at M = 20240, scaled by tokens / 20240, which
    holds while each tile streams its own A rows once and the weights are re-read per row band)."""
    t = traffic_for("dit_gemm_shapes")
    if not t:
        return None
    per_block = sum(t[name] for name in ("v", "qk", "proj", "fc1", "fc2") if name in t)
    if len([n for n in ("v", "qk", "proj", "fc1", "fc2") if n in t]) != 5:
        return None
    return int(per_block * cfg.blocks * tokens / t.get("tokens", 20240))


def path_context(stream, pk):
    """Benchmark configs 1-3 measured in the same run as the DiT step (context for its roofline): the W8A8 GEMM
    kernel at 4096^3 in every scale mode, the FP8 sweep, and the fused elementwise kernels at M = 20240."""
    int8_burst = 2.0 * pk["bf16_tflops"]
    tops = gemm_variants(4096, 4096, 4096, stream)
    ctx = {"config1_w8a8_4096_kernel": {k: {"tops": v, "frac_of_int8_burst": round(v / int8_burst, 4)}
                                        if isinstance(v, float) else v for k, v in tops.items()},
           "config2_fp8_sweep_kernel_tflops": fp8_sweep(stream),
           "config3_elementwise": elementwise_gbs(stream, pk)}
    torch.cuda.empty_cache()
    return ctx


def _cpu_block_inputs(tokens, gen):
    from oracle import torch_ref
    x = torch.randn(1, tokens, DIT["hidden"], generator=gen).to(torch.bfloat16)
    vec = torch.randn(1, DIT["hidden"], generator=gen).to(torch.bfloat16)
    cos, sin = torch_ref.rope_freqs(DIT["rope_dims"], DIT["theta"], *DIT["grid"])
    return x, vec, (cos[:tokens].contiguous(), sin[:tokens].contiguous())


def cpu_dit_block(w, tokens, gen):
    """One block of the reference's CPU path on `tokens` tokens -> (seconds, attention seconds)."""
    from oracle import torch_ref
    x, vec, rope = _cpu_block_inputs(tokens, gen)
    tm = {}
    t0 = time.perf_counter()
    torch_ref.dit_block_cpu(x, vec, w, rope, DIT["heads"], timings=tm)
    return time.perf_counter() - t0, tm.get("attention", 0.0)


def _cpu_dit_weights(gen):
    from oracle import torch_ref
    return torch_ref.make_block_weights_cpu(DIT["hidden"], DIT["mlp"], DIT["hidden"] // DIT["heads"], gen)


def cpu_baseline_dit():
    """The reference's CPU path on one full-length block (L = 20240: every linear, the norms, RoPE and
    attention) after one 512-token warm-up block; the 40-block step is 40 x that block."""
    gen = torch.Generator().manual_seed(7)
    w = _cpu_dit_weights(gen)
    cpu_dit_block(w, DIT_WARM_TOKENS, gen)
    t, ta = cpu_dit_block(w, DIT_TOKENS, gen)
    cores, threads = cpu_threads()
    step_s = DIT["blocks"] * t
    return {"value": round(DIT_TOKENS / step_s, 2), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"one full-length block of the reference's CPU path (dequantize + bf16 F.linear per linear, "
                      f"torch norms, RoPE and SDPA) at {DIT_TOKENS} tokens: {t:.1f} s ({ta:.1f} s attention); the "
                      f"step is {DIT['blocks']} such blocks ({step_s:.0f} s); {threads} threads on {cores} cores"}


def reference_dit(args):
    """Each timed step is one full-length block (L = 20240: every linear, the norms, RoPE and attention) of the
    reference's CPU path; the 40 blocks of a step are identical in work, so the step takes 40 x the block."""
    gen = torch.Generator().manual_seed(7)
    w = _cpu_dit_weights(gen)
    # untimed: one full-length block (allocator and page-in at full size), then cheap 512-token blocks
    cpu_dit_block(w, DIT_TOKENS, gen)
    for _ in range(args.warmup - 1):
        cpu_dit_block(w, DIT_WARM_TOKENS, gen)
    runs = [cpu_dit_block(w, DIT_TOKENS, gen) for _ in range(args.steps)]
    block_s = sum(r[0] for r in runs) / len(runs)
    attn_s = sum(r[1] for r in runs) / len(runs)
    step_s = DIT["blocks"] * block_s
    cores, threads = cpu_threads()
    sample = (f"each step: one full-length block of the reference's CPU path at {DIT_TOKENS} tokens "
              f"({block_s:.1f} s, {attn_s:.1f} s of it attention); a 40-block step is 40 x the block "
              f"({step_s:.0f} s); {threads} threads")
    return dict(metric="DiT denoise step tokens/s (40 blocks, 20240 tokens)", value=round(DIT_TOKENS / step_s, 2),
                unit="tokens/s", ms_per_step=round(step_s * 1e3, 1), higher_is_better=True, scaling="strong",
                dtype="bf16 (CPU)", config={"workload": "dit_step_40x_hidden4096_L20240 (config 5)", "seq_len": DIT_TOKENS,
                                            "block_seconds": round(block_s, 3), "blocks": DIT["blocks"]},
                kind="port", sample=sample, cores=threads)


# --------------------------------------------------------------------------------------------------------
# dit_gemms (config 4's linears)


DIT_GEMM_SHAPES = [("v", 4096, 4096, None), ("qk", 8192, 4096, None), ("proj", 4096, 4096, None),
                   ("fc1", 16384, 4096, "gelu_quant"), ("fc2", 4096, 16384, None)]


def workload_dit_gemms(args, world, rank, stream, pk, sampler):
    """Benchmark config 4's W8A8 linears at the block's shapes, M = 20240 tokens: v, q|k, proj and fc1 (GELU +
    int8 requantization epilogue) on the block's int8 activations, fc2 on fc1's codes - one step is the five
    GEMM launches of a block (8.15 Top). Weights: int8 codes with per-output-channel scales, as the DiT's."""
    from hy_nomas_b200 import kernels
    m = 20240
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(4242 + rank)
    x = torch.randn(m, 4096, generator=gen, device=dev).to(torch.bfloat16)
    qa, sa = kernels.quantize_activations(x)
    ws = {}
    for name, n, k, _ in DIT_GEMM_SHAPES:
        q = torch.randint(-127, 128, (n, k), generator=gen, device=dev, dtype=torch.int8)
        s = (torch.rand(n, generator=gen, device=dev) + 0.5) / (73.6 * k ** 0.5)
        ws[name] = (q, s, (torch.randn(n, generator=gen, device=dev) * 0.02).to(torch.bfloat16))
    h_q, h_s = kernels.block_gemm(qa, sa, *ws["fc1"], epilogue="gelu_quant")
    ops = {name: 2.0 * m * n * k for name, n, k, _ in DIT_GEMM_SHAPES}
    timers = {name: KernelTimer(stream) for name in ops}

    def step(i):
        for name, n, k, epi in DIT_GEMM_SHAPES:
            a, sa_ = (h_q, h_s) if name == "fc2" else (qa, sa)
            timers[name].wrap(lambda: kernels.block_gemm(a, sa_, *ws[name], epilogue=epi), ops[name])

    ms = timed_steps(step, args.steps, args.warmup, world, stream, sampler)
    for t in timers.values():
        t.active = True
    timed_steps(step, args.steps, 0, world, stream)
    per = {name: round(ops[name] / (timers[name].mean_ms() * 1e-3) / 1e12, 1) for name in ops}
    launches = launch_count(lambda: step(0))
    step_ops = sum(ops.values())
    total = sum_over_ranks(step_ops * args.steps, world)
    # e2e: the block's activations from pinned host memory, quantized and run through the five linears by the
    # public API (fc2 on fc1's requantized output), fc2's output read back
    xh = x.cpu().pin_memory()
    yh = torch.empty((m, 4096), dtype=torch.bfloat16).pin_memory()

    def e2e_step(i):
        xd = xh.to(dev, non_blocking=True)
        a, sa_ = kernels.quantize_activations(xd)
        for name in ("v", "qk", "proj"):
            kernels.block_gemm(a, sa_, *ws[name])
        hq, hs = kernels.block_gemm(a, sa_, *ws["fc1"], epilogue="gelu_quant")
        yh.copy_(kernels.block_gemm(hq, hs, *ws["fc2"]), non_blocking=True)

    e2e_ms = timed_steps(e2e_step, args.steps, 1, world, stream)
    peak = 2.0 * pk["bf16_tflops"]
    achieved = step_ops / (sum(t.mean_ms() for t in timers.values()) * 1e-3) / 1e12
    traffic = traffic_for("dit_gemm_shapes")
    roof = {"kernel": "hn::gemm::k_block_gemm<int8, group activation scales, per-channel weights> (the five)",
            "bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TOPS",
            "frac": round(achieved / peak, 4),
            "peak_note": f"int8 dense = 2 x {pk['source']} bf16 burst ({pk['bf16_tflops']} TFLOP/s)",
            "traffic": sum(traffic[n] for n in ops) if traffic else None}
    config = {"workload": "dit_block_linears_M20240 (config 4): v, q|k, proj, fc1 (GELU + requant), fc2",
              "M": m, "shapes": {name: f"{n}x{k}" for name, n, k, _ in DIT_GEMM_SHAPES}, "per_shape_tops": per,
              "activation_scales": "per token x 128 channels", "weight_scales": "per output channel",
              "l2": "weights 16.8-67 MB per shape and activations 83-331 MB stream between reuses",
              "parallelism": f"replicas x{world}"}
    return dict(metric="W8A8 GEMM TOPS (DiT block linears)", value=round(total / (ms * 1e-3) / 1e12, 2), unit="TOPS",
                ms_per_step=round(ms / args.steps, 4), higher_is_better=True, scaling="weak", dtype="int8",
                config=config,
                e2e={"value": round(total / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TOPS",
                     "h2d_bytes_per_step": xh.numel() * 2 * world, "d2h_bytes_per_step": yh.numel() * 2 * world},
                roofline=roof, gpu_launches=launches * args.steps,
                cpu_baseline_fn=lambda: cpu_baseline_gemm(4096, 4096, 4096))


def reference_dit_gemms(args):
    """The reference's CPU path for the block's five linears on 256 of the 20240 rows per step (dequantize +
    bf16 F.linear each, ops.py:175-176)."""
    from oracle import torch_ref
    rows = 256
    gen = torch.Generator().manual_seed(5)
    lin = {}
    for name, n, k, _ in DIT_GEMM_SHAPES:
        x, q, s, bias = cpu_gemm_sample(rows, n, k, gen)
        lin[name] = (x, q, s, bias)

    def run():
        for name, *_ in DIT_GEMM_SHAPES:
            torch_ref.int8_linear_cpu(*lin[name])
    for _ in range(args.warmup):
        run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run()
    dt = time.perf_counter() - t0
    ops = sum(2.0 * rows * n * k for _, n, k, _ in DIT_GEMM_SHAPES)
    cores, threads = cpu_threads()
    return dict(metric="W8A8 GEMM TOPS (DiT block linears)", value=round(ops * args.steps / dt / 1e12, 4), unit="TOPS",
                ms_per_step=round(dt / args.steps * 1e3, 3), higher_is_better=True, scaling="weak", dtype="int8",
                kind="port", cores=threads,
                config={"workload": "dit_block_linears_M20240 (config 4)", "M": 20240},
                sample=f"{rows} of 20240 rows per step for each of the five linears (dequantize_g128 + bf16 F.linear, "
                       f"{threads} threads)")


# --------------------------------------------------------------------------------------------------------
# gemm (config 1)


def workload_gemm(args, world, rank, stream, pk, sampler):
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

    ms = timed_steps(step, args.steps, args.warmup, world, stream, sampler)
    timer.active = True
    timed_steps(step, args.steps, 0, world, stream)
    gemm_ms = timer.mean_ms()
    launches = launch_count(lambda: step(0))
    ops = 2.0 * m * n * k
    total_ops = sum_over_ranks(ops * args.steps, world)
    value = total_ops / (ms * 1e-3) / 1e12
    xh = [x.cpu().pin_memory() for x in xs[:2]]
    yh = torch.empty((m, n), dtype=torch.bfloat16).pin_memory()

    def e2e_step(i):
        x = xh[i % 2].to(dev, non_blocking=True)
        qw, sw = ws[i % nsets]
        y = kernels.int8_g128_linear(x, qw, sw, bias)
        yh.copy_(y, non_blocking=True)

    e2e_ms = timed_steps(e2e_step, args.steps, 2, world, stream)
    e2e = {"value": round(total_ops / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TOPS",
           "h2d_bytes_per_step": m * k * 2 * world, "d2h_bytes_per_step": m * n * 2 * world}
    peak = 2.0 * pk["bf16_tflops"]
    achieved = ops / (gemm_ms * 1e-3) / 1e12
    roof = {"kernel": "hn::gemm::k_block_gemm<int8, group activation scales, per-channel weights>", "bound": "tensor",
            "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TOPS", "frac": round(achieved / peak, 4),
            "peak_note": f"int8 dense = 2 x {pk['source']} bf16 burst ({pk['bf16_tflops']} TFLOP/s)",
            "traffic": traffic_for("gemm"), "algorithmic_bytes": m * k + n * k + m * n * 2 + m * 4 * (k // 128) + n * 4}
    config = {"workload": "w8a8_linear_4096x4096x4096 (config 1): quantize + block-scaled GEMM",
              "M": m, "N": n, "K": k, "activation_scales": "per token x 128 channels",
              "weight_scales": "per output channel", "l2": f"inputs rotate over {nsets} sets > L2",
              "parallelism": f"replicas x{world}", "kernel_variants_tops": gemm_variants(m, n, k, stream)}
    return dict(metric="W8A8 GEMM TOPS", value=round(value, 2), unit="TOPS", ms_per_step=round(ms / args.steps, 4),
                higher_is_better=True, scaling="weak", dtype="int8", config=config, e2e=e2e, roofline=roof,
                gpu_launches=launches * args.steps, cpu_baseline_fn=lambda: cpu_baseline_gemm(m, n, k))


def _time_kernel(fn, stream, flush, iters):
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
    return statistics.median(times)


def gemm_variants(m, n, k, stream, iters=20):
    """Context for the roofline (not the headline): the GEMM kernel alone in each scale mode, config 1's literal
    linear (per-token round-half-even quantization of x, then the per-token x per-channel GEMM, timed together),
    and cuBLASLt's int8 GEMM (torch._int_mm, no scaling) on the same shape."""
    from hy_nomas_b200 import kernels
    gen = torch.Generator().manual_seed(99)
    dev = torch.device("cuda")
    qa = torch.randint(-127, 128, (m, k), generator=gen, dtype=torch.int8).to(dev)
    qw = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8).to(dev)
    sa_g = kernels.quantize_activations(torch.randn(m, k, generator=gen).bfloat16().to(dev))[1]
    sa_r = (torch.rand(m, generator=gen) * 0.02).to(dev)
    sw_g = (torch.rand(n, k // 128, generator=gen) * 4e-3).to(dev)
    sw_r = (torch.rand(n, generator=gen) * 4e-3).to(dev)
    x = torch.randn(m, k, generator=gen).bfloat16().to(dev)
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev)

    def literal_config1():
        qt, st = kernels.quantize_activations(x, per_token=True, round_half_even=True)
        return kernels.block_gemm(qt, st, qw, sw_r)
    sw_gm = sw_g.t().contiguous().t()   # [N, K/128] view of group-major storage (the layout weights.py loads)
    cases = {"a_group_w_group_rowmajor": lambda: kernels.block_gemm(qa, sa_g, qw, sw_g),
             "a_group_w_group_groupmajor": lambda: kernels.block_gemm(qa, sa_g, qw, sw_gm),
             "a_group_w_channel": lambda: kernels.block_gemm(qa, sa_g, qw, sw_r),
             "a_token_w_channel": lambda: kernels.block_gemm(qa, sa_r, qw, sw_r),
             "quantize_token_rne_and_gemm": literal_config1,
             "cublaslt_int8_int32": lambda: torch._int_mm(qa, qw.t())}
    res = {}
    for name, fn in cases.items():
        try:
            res[name] = round(2.0 * m * n * k / (_time_kernel(fn, stream, flush, iters) * 1e-3) / 1e12, 1)
        except RuntimeError as e:
            res[name] = f"unavailable: {str(e).splitlines()[0][:80]}"
    return res


def cpu_gemm_sample(rows, n, k, gen):
    x = outlier_activations(rows, k, gen)
    q, s = make_int8_weight(n, k, gen, "cpu", per_channel=False)
    bias = (torch.randn(n, generator=gen) * 0.02).bfloat16()
    return x, q, s, bias


def cpu_baseline_gemm(m, n, k, budget_s=10.0):
    """The reference's CPU path (dequantize_g128 + bf16 F.linear, hy_nomas/ops.py:175-176) on a bounded
    sample of rows, on all host threads."""
    from oracle import torch_ref
    rows = 512
    x, q, s, bias = cpu_gemm_sample(rows, n, k, torch.Generator().manual_seed(5))
    torch_ref.int8_linear_cpu(x, q, s, bias)
    t0 = time.perf_counter()
    it = 0
    while time.perf_counter() - t0 < budget_s:
        torch_ref.int8_linear_cpu(x, q, s, bias)
        it += 1
    dt = (time.perf_counter() - t0) / it
    cores, threads = cpu_threads()
    return {"value": round(2.0 * rows * n * k / dt / 1e12, 4), "unit": "TOPS", "cores": threads, "kind": "port",
            "sample": f"{rows} x {k} -> {n} rows of the workload, {it} iterations in {budget_s:.0f}+ s "
                      f"(dequantize_g128 + bf16 F.linear, torch {torch.__version__}, {threads} threads on "
                      f"{cores} cores)"}


def reference_gemm(args):
    from oracle import torch_ref
    m, n, k = 4096, 4096, 4096
    rows = 1024
    x, q, s, bias = cpu_gemm_sample(rows, n, k, torch.Generator().manual_seed(5))
    for _ in range(args.warmup):
        torch_ref.int8_linear_cpu(x, q, s, bias)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        torch_ref.int8_linear_cpu(x, q, s, bias)
    dt = time.perf_counter() - t0
    value = 2.0 * rows * n * k * args.steps / dt / 1e12
    cores, threads = cpu_threads()
    return dict(metric="W8A8 GEMM TOPS", value=round(value, 4), unit="TOPS", ms_per_step=round(dt / args.steps * 1e3, 3),
                higher_is_better=True, scaling="weak", dtype="int8", kind="port", cores=threads,
                config={"workload": "w8a8_linear_4096x4096x4096 (config 1)", "M": m, "N": n, "K": k},
                sample=f"{rows} of {m} rows per step (dequantize_g128 + bf16 F.linear on CPU, {threads} threads)")


# --------------------------------------------------------------------------------------------------------
# fp8 (config 2)


FP8_SHAPES = {"qkv": (12288, 4096), "mlp_up": (16384, 4096), "mlp_down": (4096, 16384)}
FP8_M = (1024, 4096, 16384, 20240)


def fp8_weight(n, k, gen, dev):
    """fp32 N(0, 0.02) quantized per 128 x 128 block (pixelumm.py:77-82) by the product's quantizer."""
    from hy_nomas_b200 import ops
    w = torch.randn(n, k, generator=gen, device=dev) * 0.02
    return ops.quantize_fp8_block(w)


def workload_fp8(args, world, rank, stream, pk, sampler):
    from hy_nomas_b200 import kernels
    m, (n, k) = 20240, FP8_SHAPES["mlp_up"]
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(77 + rank)
    nsets = 2
    xs = [torch.randn(m, k, generator=gen, device=dev).to(torch.bfloat16) for _ in range(nsets)]
    ws = [fp8_weight(n, k, gen, dev) for _ in range(nsets)]
    bias = (torch.randn(n, generator=gen, device=dev) * 0.02).to(torch.bfloat16)
    timer = KernelTimer(stream)
    ops_ = 2.0 * m * n * k

    def step(i):
        qw, sw = ws[i % nsets]
        qa, sa = kernels.quantize_activations(xs[i % nsets], "fp8")
        return timer.wrap(lambda: kernels.block_gemm(qa, sa, qw, sw, bias, kind="fp8"), ops_)

    ms = timed_steps(step, args.steps, args.warmup, world, stream, sampler)
    timer.active = True
    timed_steps(step, args.steps, 0, world, stream)
    gemm_ms = timer.mean_ms()
    launches = launch_count(lambda: step(0))
    total = sum_over_ranks(ops_ * args.steps, world)
    xh = [x.cpu().pin_memory() for x in xs]
    yh = torch.empty((m, n), dtype=torch.bfloat16).pin_memory()

    def e2e_step(i):
        qw, sw = ws[i % nsets]
        y = kernels.block_linear(xh[i % nsets].to(dev, non_blocking=True), qw, sw, bias, kind="fp8")
        yh.copy_(y, non_blocking=True)

    e2e_ms = timed_steps(e2e_step, args.steps, 1, world, stream)
    peak = 2.0 * pk["bf16_tflops"]
    achieved = ops_ / (gemm_ms * 1e-3) / 1e12
    roof = {"kernel": "hn::gemm::k_block_gemm<e4m3, 1x128 activation blocks, 128x128 weight blocks>",
            "bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4),
            "peak_note": f"fp8 dense = 2 x {pk['source']} bf16 burst ({pk['bf16_tflops']} TFLOP/s)",
            "traffic": traffic_for("fp8"), "algorithmic_bytes": m * k + n * k + m * n * 2 + m * 4 * (k // 128)}
    config = {"workload": "fp8_block_linear_M20240_N16384_K4096 (config 2, MLP-up): quantize + GEMM",
              "M": m, "N": n, "K": k, "activation_scales": "1 x 128 blocks (e4m3)", "weight_scales": "128 x 128 blocks",
              "l2": "inputs rotate over 2 sets of 166 MB activations + 67 MB weights (> L2)",
              "parallelism": f"replicas x{world}", "sweep_kernel_tflops": fp8_sweep(stream)}
    return dict(metric="FP8 block GEMM TFLOP/s", value=round(total / (ms * 1e-3) / 1e12, 2), unit="TFLOP/s",
                ms_per_step=round(ms / args.steps, 4), higher_is_better=True, scaling="weak", dtype="fp8 e4m3",
                config=config,
                e2e={"value": round(total / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                     "h2d_bytes_per_step": m * k * 2 * world, "d2h_bytes_per_step": m * n * 2 * world},
                roofline=roof, gpu_launches=launches * args.steps,
                cpu_baseline_fn=lambda: cpu_baseline_fp8(m, n, k))


def fp8_sweep(stream, iters=5):
    """The config's 3 weight shapes x 4 token counts, GEMM kernel alone (L2 flushed before each launch)."""
    from hy_nomas_b200 import kernels
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(5)
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev)
    res = {}
    for name, (n, k) in FP8_SHAPES.items():
        qw, sw = fp8_weight(n, k, gen, dev)
        for m in FP8_M:
            qa, sa = kernels.quantize_activations(torch.randn(m, k, generator=gen, device=dev).to(torch.bfloat16), "fp8")
            t = _time_kernel(lambda: kernels.block_gemm(qa, sa, qw, sw, kind="fp8"), stream, flush, iters)
            res[f"{name}_{n}x{k}_M{m}"] = round(2.0 * m * n * k / (t * 1e-3) / 1e12, 1)
        del qw, sw
    return res


def cpu_fp8_sample(rows, n, k, gen):
    from oracle import torch_ref
    x = torch.randn(rows, k, generator=gen).to(torch.bfloat16)
    q, s = torch_ref.fp8_block_quantize(torch.randn(n, k, generator=gen) * 0.02)
    bias = (torch.randn(n, generator=gen) * 0.02).to(torch.bfloat16)
    return x, q, s, bias


def cpu_baseline_fp8(m, n, k, budget_s=10.0):
    """The reference's CPU path for the FP8 linear (dequantize_fp8_block + bf16 F.linear, pixelumm.py:154-155)."""
    from oracle import torch_ref
    rows = 256
    x, q, s, bias = cpu_fp8_sample(rows, n, k, torch.Generator().manual_seed(5))
    torch_ref.fp8_linear_cpu(x, q, s, bias)
    t0 = time.perf_counter()
    it = 0
    while time.perf_counter() - t0 < budget_s:
        torch_ref.fp8_linear_cpu(x, q, s, bias)
        it += 1
    dt = (time.perf_counter() - t0) / it
    cores, threads = cpu_threads()
    return {"value": round(2.0 * rows * n * k / dt / 1e12, 4), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{rows} of {m} rows, {it} iterations in {budget_s:.0f}+ s (dequantize_fp8_block + bf16 "
                      f"F.linear, {threads} threads on {cores} cores)"}


def reference_fp8(args):
    from oracle import torch_ref
    m, (n, k) = 20240, FP8_SHAPES["mlp_up"]
    rows = 512
    x, q, s, bias = cpu_fp8_sample(rows, n, k, torch.Generator().manual_seed(5))
    for _ in range(args.warmup):
        torch_ref.fp8_linear_cpu(x, q, s, bias)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        torch_ref.fp8_linear_cpu(x, q, s, bias)
    dt = time.perf_counter() - t0
    cores, threads = cpu_threads()
    return dict(metric="FP8 block GEMM TFLOP/s", value=round(2.0 * rows * n * k * args.steps / dt / 1e12, 4),
                unit="TFLOP/s", ms_per_step=round(dt / args.steps * 1e3, 3), higher_is_better=True, scaling="weak",
                dtype="fp8 e4m3", kind="port", cores=threads,
                config={"workload": "fp8_block_linear_M20240_N16384_K4096 (config 2)", "M": m, "N": n, "K": k},
                sample=f"{rows} of {m} rows per step (dequantize_fp8_block + bf16 F.linear, {threads} threads)")


# --------------------------------------------------------------------------------------------------------
# elementwise (config 3)


def elementwise_bytes(m, d, h, hd):
    """Algorithmic HBM bytes per kernel (each tensor read or written once)."""
    act = m * d * 2
    codes, scales = m * d, m * (d // 128) * 4
    tables = 2 * m * hd * 4
    return {"adaln_quant": act + codes + scales + 2 * d * 2,
            "qk_norm_rope2": 4 * m * h * hd * 2 + tables + 2 * hd * 2,
            "gated_residual": 3 * act + d * 2,
            "gated_residual_adaln_quant": 3 * act + codes + scales + 3 * d * 2}


def workload_elementwise(args, world, rank, stream, pk, sampler):
    from hy_nomas_b200 import fused, kernels
    from hy_nomas_b200.dit import rope_freqs
    m, d, h, hd = 20240, 4096, 32, 128
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(31 + rank)
    bf = lambda *s, std=1.0: (torch.randn(*s, generator=gen, device=dev) * std).to(torch.bfloat16)  # noqa: E731
    nsets = 2
    sets = [dict(x=bf(1, m, d), y=bf(1, m, d), q=bf(1, m, h, hd), k=bf(1, m, h, hd)) for _ in range(nsets)]
    shift, scale, gate = bf(1, d, std=0.1), bf(1, d, std=0.1), bf(1, d, std=0.1)
    wq, wk = bf(hd, std=0.1) + 1, bf(hd, std=0.1) + 1
    rope = rope_freqs((16, 56, 56), 10000.0, 23, 22, 40, device=dev)
    nbytes = elementwise_bytes(m, d, h, hd)
    timers = {name: KernelTimer(stream) for name in nbytes}

    def step(i):
        s = sets[i % nsets]
        timers["adaln_quant"].wrap(lambda: kernels.adaln_quant(s["x"], shift, scale))
        timers["qk_norm_rope2"].wrap(lambda: fused.qk_norm_rope2(s["q"], s["k"], wq, wk, rope))
        timers["gated_residual"].wrap(lambda: fused.gated_residual(s["x"], s["y"], gate))
        timers["gated_residual_adaln_quant"].wrap(
            lambda: fused.gated_residual_adaln_quant(s["x"], s["y"], gate, shift, scale))

    ms = timed_steps(step, args.steps, args.warmup, world, stream, sampler)
    for t in timers.values():
        t.active = True
    timed_steps(step, args.steps, 0, world, stream)
    per_kernel = {name: t.mean_ms() for name, t in timers.items()}
    launches = launch_count(lambda: step(0))
    step_bytes = sum(nbytes.values())
    total = sum_over_ranks(step_bytes * args.steps, world)
    gbs = {name: round(nbytes[name] / (per_kernel[name] * 1e-3) / 1e9, 1) for name in nbytes}
    top = max(per_kernel, key=per_kernel.get)
    peak = pk["hbm_gbs"]
    roof = {"kernel": f"{top} (largest time share of the chain)", "bound": "hbm", "achieved": gbs[top],
            "peak": peak, "unit": "GB/s", "frac": round(gbs[top] / peak, 4),
            "peak_note": f"{pk['source']} HBM copy bandwidth", "traffic": (traffic_for("elementwise") or {}).get(top),
            "algorithmic_bytes": nbytes[top],
            "per_kernel_gbs": gbs, "per_kernel_frac": {k: round(v / peak, 4) for k, v in gbs.items()}}
    # e2e through the public API: the chain's inputs from pinned host memory, every output a caller consumes
    # (the codes and scales of both quantizing kernels, the normalized q and k, the new residual) read back
    hsets = [{k_: v.cpu().pin_memory() for k_, v in s.items()} for s in sets]
    outs_h = dict(q1=torch.empty((m, d), dtype=torch.int8).pin_memory(),
                  s1=torch.empty((m, d // 128), dtype=torch.float32).pin_memory(),
                  yq=torch.empty((1, m, h, hd), dtype=torch.bfloat16).pin_memory(),
                  yk=torch.empty((1, m, h, hd), dtype=torch.bfloat16).pin_memory(),
                  x2=torch.empty((1, m, d), dtype=torch.bfloat16).pin_memory(),
                  q2=torch.empty((m, d), dtype=torch.int8).pin_memory(),
                  s2=torch.empty((m, d // 128), dtype=torch.float32).pin_memory())

    def e2e_step(i):
        s = {k_: v.to(dev, non_blocking=True) for k_, v in hsets[i % nsets].items()}
        q1, s1 = kernels.adaln_quant(s["x"], shift, scale)
        yq, yk = fused.qk_norm_rope2(s["q"], s["k"], wq, wk, rope)
        fused.gated_residual(s["x"], s["y"], gate)
        x2, q2, s2 = fused.gated_residual_adaln_quant(s["x"], s["y"], gate, shift, scale)
        for name, t in dict(q1=q1, s1=s1, yq=yq, yk=yk, x2=x2, q2=q2, s2=s2).items():
            outs_h[name].copy_(t, non_blocking=True)

    e2e_ms = timed_steps(e2e_step, args.steps, 1, world, stream)
    e2e_total = sum_over_ranks(step_bytes * args.steps, world)
    h2d = sum(v.numel() * v.element_size() for v in hsets[0].values())
    d2h = sum(v.numel() * v.element_size() for v in outs_h.values())
    others = other_elementwise_kernels(m, d, h, hd, stream, sets, shift, scale, wq, rope)
    config = {"workload": "dit_elementwise_chain_M20240_D4096 (config 3): adaln_quant, qk_norm_rope2 (q and k, "
                          "3-D RoPE 16/56/56), gated_residual, gated_residual_adaln_quant",
              "M": m, "D": d, "heads": h, "head_dim": hd, "bytes_per_step": step_bytes,
              "l2": "inputs rotate over 2 sets (each tensor 166 MB > L2)", "parallelism": f"replicas x{world}",
              "other_kernels_gbs": others}
    return dict(metric="fused DiT elementwise chain GB/s", value=round(total / (ms * 1e-3) / 1e9, 1), unit="GB/s",
                ms_per_step=round(ms / args.steps, 4), higher_is_better=True, scaling="weak", dtype="bf16 -> int8",
                config=config,
                e2e={"value": round(e2e_total / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                     "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world},
                roofline=roof, gpu_launches=launches * args.steps,
                cpu_baseline_fn=lambda: cpu_baseline_elementwise(m, d, h, hd))


def other_elementwise_kernels(m, d, h, hd, stream, sets, shift, scale, w, rope, iters=20):
    """The path's remaining bandwidth-bound kernels at the same shapes (not part of the chain's value), GB/s
    of algorithmic bytes: K1 quantize_activations (int8 and e4m3, per 128 and per token), K4 adaln, K5 on one
    tensor, K7 pixelumm_qk (the FP8 decoder's QK norm: 32 heads x 128, split T/HW halves), and the int8 KV
    cache: quantize_kv, dequantize_kv and K5 with the KV quantizer fused (the cache pass)."""
    from hy_nomas_b200 import fused, kernels, world
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device="cuda")
    x2d = [s["x"].view(m, d) for s in sets]
    half = hd // 2
    wt = torch.ones(half, dtype=torch.bfloat16, device="cuda")
    whw = torch.ones(half, dtype=torch.bfloat16, device="cuda")
    kv = [world.quantize_kv(s["q"].view(m, h, hd)) for s in sets]
    dec_w = torch.ones(d, dtype=torch.bfloat16, device="cuda")
    gu = [torch.randn(m, 2 * 12288, device="cuda").to(torch.bfloat16) for _ in range(2)]
    cases = {
        "quantize_activations_int8_g128": (lambda i: kernels.quantize_activations(x2d[i % 2]), m * d * 3 + m * (d // 128) * 4),
        "quantize_activations_e4m3_g128": (lambda i: kernels.quantize_activations(x2d[i % 2], "fp8"), m * d * 3 + m * (d // 128) * 4),
        "quantize_activations_int8_token": (lambda i: kernels.quantize_activations(x2d[i % 2], per_token=True), m * d * 3 + m * 4),
        "adaln": (lambda i: fused.adaln(sets[i % 2]["x"], shift, scale), m * d * 4),
        "qk_norm_rope_one_tensor": (lambda i: fused.qk_norm_rope(sets[i % 2]["q"], w, rope), 2 * m * h * hd * 2 + 2 * m * hd * 4),
        "pixelumm_qk": (lambda i: fused.pixelumm_qk(sets[i % 2]["q"], wt, whw, *rope), 2 * m * h * hd * 2 + 2 * m * hd * 4),
        "quantize_kv": (lambda i: world.quantize_kv(sets[i % 2]["q"].view(m, h, hd)), m * h * hd * 3 + m * h * 4),
        "dequantize_kv": (lambda i: world.dequantize_kv(*kv[i % 2]), m * h * hd * 3 + m * h * 4),
        "qk_norm_rope_kv": (lambda i: fused.qk_norm_rope_kv(sets[i % 2]["q"], w, rope),
                            m * h * hd * 5 + m * h * 4 + 2 * m * hd * 4),
        # the PixelUMM decoder fusions at its shapes (hidden 4096, intermediate 12288): RMSNorm + e4m3 quantizer,
        # and silu(gate) * up + e4m3 quantizer over the halves of a [M, 2 x 12288] gate|up output
        "decoder_rmsnorm_quant_e4m3": (lambda i: fused.rmsnorm_quant(x2d[i % 2], dec_w, 1e-6, "fp8"),
                                       m * d * 3 + m * (d // 128) * 4 + d * 2),
        "decoder_silu_mul_quant_e4m3": (lambda i: fused.silu_mul_quant(gu[i % 2][:, :12288], gu[i % 2][:, 12288:], "fp8"),
                                        m * 12288 * 5 + m * 96 * 4),
    }
    res = {}
    for name, (fn, nbytes) in cases.items():
        fn(0)
        times = []
        for i in range(iters):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn(i)
            b.record(stream)
            b.synchronize()
            times.append(a.elapsed_time(b))
        res[name] = round(nbytes / (statistics.median(times) * 1e-3) / 1e9, 1)
    return res


def elementwise_gbs(stream, pk, iters=20):
    """Config 3's kernels (and the path's other bandwidth-bound kernels) at M = 20240, D = 4096, 32 x 128 heads,
    each alone with L2 flushed before every launch: GB/s of algorithmic bytes and the fraction of the measured
    HBM copy bandwidth."""
    from hy_nomas_b200 import fused, kernels
    from hy_nomas_b200.dit import rope_freqs
    m, d, h, hd = 20240, 4096, 32, 128
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(31)
    bf = lambda *s, std=1.0: (torch.randn(*s, generator=gen, device=dev) * std).to(torch.bfloat16)  # noqa: E731
    sets = [dict(x=bf(1, m, d), y=bf(1, m, d), q=bf(1, m, h, hd), k=bf(1, m, h, hd)) for _ in range(2)]
    shift, scale, gate = bf(1, d, std=0.1), bf(1, d, std=0.1), bf(1, d, std=0.1)
    wq, wk = bf(hd, std=0.1) + 1, bf(hd, std=0.1) + 1
    rope = rope_freqs((16, 56, 56), 10000.0, 23, 22, 40, device=dev)
    nb = elementwise_bytes(m, d, h, hd)
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev)
    chain = {"adaln_quant": lambda i: kernels.adaln_quant(sets[i % 2]["x"], shift, scale),
             "qk_norm_rope2": lambda i: fused.qk_norm_rope2(sets[i % 2]["q"], sets[i % 2]["k"], wq, wk, rope),
             "gated_residual": lambda i: fused.gated_residual(sets[i % 2]["x"], sets[i % 2]["y"], gate),
             "gated_residual_adaln_quant": lambda i: fused.gated_residual_adaln_quant(
                 sets[i % 2]["x"], sets[i % 2]["y"], gate, shift, scale)}
    gbs = {}
    for name, fn in chain.items():
        fn(0)
        times = []
        for i in range(iters):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn(i)
            b.record(stream)
            b.synchronize()
            times.append(a.elapsed_time(b))
        gbs[name] = round(nb[name] / (statistics.median(times) * 1e-3) / 1e9, 1)
    gbs.update(other_elementwise_kernels(m, d, h, hd, stream, sets, shift, scale, wq, rope, iters))
    del sets, flush
    return {name: {"gbs": v, "frac_of_hbm": round(v / pk["hbm_gbs"], 4)} for name, v in gbs.items()}


def cpu_elementwise_chain(rows, d, h, hd, gen):
    """The reference's CPU arithmetic for the chain on `rows` tokens (model.py:103-138, 280-284, ops.py:41-52)."""
    from oracle import torch_ref
    rope_freqs = torch_ref.rope_freqs
    bf = lambda *s, std=1.0: (torch.randn(*s, generator=gen) * std).to(torch.bfloat16)  # noqa: E731
    x, y, q, k = bf(1, rows, d), bf(1, rows, d), bf(1, rows, h, hd), bf(1, rows, h, hd)
    shift, scale, gate = bf(1, d, std=0.1), bf(1, d, std=0.1), bf(1, d, std=0.1)
    w = bf(hd, std=0.1) + 1
    cos, sin = rope_freqs((16, 56, 56), 10000.0, 23, 22, 40)
    cos, sin = cos[:rows], sin[:rows]

    def run():
        xm = torch_ref.modulate(torch_ref.layer_norm(x), shift, scale).to(torch.bfloat16)
        torch_ref.quantize_g128(xm[0])
        torch_ref.apply_rope(torch_ref.rms_norm(q, w), cos, sin)
        torch_ref.apply_rope(torch_ref.rms_norm(k, w), cos, sin)
        x1 = x + y * gate.unsqueeze(1)
        x2 = x + y * gate.unsqueeze(1)
        torch_ref.quantize_g128(torch_ref.modulate(torch_ref.layer_norm(x2), shift, scale).to(torch.bfloat16)[0])
        return x1
    return run


def cpu_baseline_elementwise(m, d, h, hd, budget_s=10.0):
    rows = 1024
    run = cpu_elementwise_chain(rows, d, h, hd, torch.Generator().manual_seed(3))
    run()
    t0 = time.perf_counter()
    it = 0
    while time.perf_counter() - t0 < budget_s:
        run()
        it += 1
    dt = (time.perf_counter() - t0) / it
    cores, threads = cpu_threads()
    b = sum(elementwise_bytes(rows, d, h, hd).values())
    return {"value": round(b / dt / 1e9, 2), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"the chain on {rows} of {m} tokens, {it} iterations in {budget_s:.0f}+ s (torch layer_norm, "
                      f"modulate, quantize_g128, RMSNorm, apply_rope, x + y*gate on CPU; {threads} threads on "
                      f"{cores} cores); GB/s = the same algorithmic bytes per token"}


def reference_elementwise(args):
    m, d, h, hd = 20240, 4096, 32, 128
    rows = 2048
    run = cpu_elementwise_chain(rows, d, h, hd, torch.Generator().manual_seed(3))
    for _ in range(args.warmup):
        run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run()
    dt = time.perf_counter() - t0
    cores, threads = cpu_threads()
    b = sum(elementwise_bytes(rows, d, h, hd).values())
    return dict(metric="fused DiT elementwise chain GB/s", value=round(b * args.steps / dt / 1e9, 3), unit="GB/s",
                ms_per_step=round(dt / args.steps * 1e3, 3), higher_is_better=True, scaling="weak",
                dtype="bf16 -> int8", kind="port", cores=threads,
                config={"workload": "dit_elementwise_chain_M20240_D4096 (config 3)", "M": m, "D": d},
                sample=f"the chain on {rows} of {m} tokens per step (torch CPU arithmetic, {threads} threads)")


# --------------------------------------------------------------------------------------------------------


# --------------------------------------------------------------------------------------------------------
# attention (configs 4 and 5's attention, hy_nomas/model.py:145-151)

ATTN_L, ATTN_H = 20240, 32


def attn_inputs(lq, lk, gen, dev):
    q = torch.randn(1, lq, ATTN_H, 128, generator=gen, device=dev).to(torch.bfloat16)
    k = torch.randn(1, lk, ATTN_H, 128, generator=gen, device=dev).to(torch.bfloat16)
    v = torch.randn(1, lk, ATTN_H, 128, generator=gen, device=dev).to(torch.bfloat16)
    return q, k, v


def workload_attention(args, world, rank, stream, pk, sampler):
    """The block's attention at the DiT shape (20240 queries x 20240 keys x 32 heads x 128) on the library's
    sm_100a kernel with the projection's input quantizer fused (attention.attention_quant, the path the block
    takes with HN_ATTENTION=native); torch's cuDNN SDPA on the same inputs, the one-rank-of-eight shape and the
    key-piece merge of the sequence-parallel step are reported beside it."""
    import torch.nn.functional as F
    from hy_nomas_b200 import attention as attn
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(77 + rank)
    q, k, v = attn_inputs(ATTN_L, ATTN_L, gen, dev)
    flops = 4.0 * ATTN_L * ATTN_L * ATTN_H * 128
    timer = KernelTimer(stream)

    def step(i):
        timer.wrap(lambda: attn.attention_quant(q, k, v), flops)

    ms = timed_steps(step, args.steps, args.warmup, world, stream, sampler)
    timer.active = True
    timed_steps(step, args.steps, 0, world, stream)
    kernel_ms = timer.mean_ms()
    launches = launch_count(lambda: step(0))

    def bench_ms(fn, it=5):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(it):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / it

    sdpa = lambda qq, kk, vv: F.scaled_dot_product_attention(qq.transpose(1, 2), kk.transpose(1, 2), vv.transpose(1, 2))
    sdpa_ms = bench_ms(lambda: sdpa(q, k, v))
    plain_ms = bench_ms(lambda: attn.attention(q, k, v))
    lr = ATTN_L // 8
    qr = q[:, :lr].contiguous()
    rank_native = bench_ms(lambda: attn.attention_quant(qr, k, v))
    rank_sdpa = bench_ms(lambda: sdpa(qr, k, v))
    rank_pieces = bench_ms(lambda: attn.merge([attn.attention_lse(qr, k[:, i * lr:(i + 1) * lr], v[:, i * lr:(i + 1) * lr])
                                               for i in range(8)]))
    rflops = 4.0 * lr * ATTN_L * ATTN_H * 128
    # e2e: q, k, v from pinned host memory through the public API, the quantized projection input read back
    qh, kh, vh = q.cpu().pin_memory(), k.cpu().pin_memory(), v.cpu().pin_memory()
    ch = torch.empty((ATTN_L, ATTN_H * 128), dtype=torch.int8).pin_memory()
    sh = torch.empty((ATTN_L, ATTN_H), dtype=torch.float32).pin_memory()

    def e2e_step(i):
        c, sc = attn.attention_quant(qh.to(dev, non_blocking=True), kh.to(dev, non_blocking=True),
                                     vh.to(dev, non_blocking=True))
        ch.copy_(c, non_blocking=True)
        sh.copy_(sc, non_blocking=True)

    e2e_ms = timed_steps(e2e_step, args.steps, 1, world, stream)
    total = sum_over_ranks(flops * args.steps, world)
    achieved = flops / (kernel_ms * 1e-3) / 1e12
    roof = {"kernel": "hn::attn::k_attention (fused int8 output quantizer)", "bound": "tensor",
            "achieved": round(achieved, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
            "frac": round(achieved / pk["bf16_tflops"], 4),
            "peak_note": f"{pk['source']} bf16 dense burst (the kernel is timed alone)", "traffic": None}
    config = {"workload": f"attention_L{ATTN_L}_H{ATTN_H}_D128 (configs 4/5): softmax(q k^T / sqrt(128)) v + the "
                          "projection's int8 input quantizer",
              "q_k_v": f"bf16 [1, {ATTN_L}, {ATTN_H}, 128] each (166 MB; 498 MB together, above L2)",
              "native_fused_quant_ms": round(kernel_ms, 3), "native_bf16_out_ms": round(plain_ms, 3),
              "torch_cudnn_sdpa_ms": round(sdpa_ms, 3),
              "torch_cudnn_sdpa_tflops": round(flops / (sdpa_ms * 1e-3) / 1e12, 1),
              "one_rank_of_8": {"queries": lr, "native_quant_ms": round(rank_native, 3),
                                "native_tflops": round(rflops / (rank_native * 1e-3) / 1e12, 1),
                                "cudnn_sdpa_ms": round(rank_sdpa, 3),
                                "cudnn_8_key_pieces_plus_merge_ms": round(rank_pieces, 3)},
              "parallelism": f"replicas x{world}"}
    return dict(metric="attention TFLOP/s (20240 x 20240 x 32 heads x 128)", value=round(total / (ms * 1e-3) / 1e12, 1),
                unit="TFLOP/s", ms_per_step=round(ms / args.steps, 3), higher_is_better=True, scaling="weak",
                dtype="bf16 (fp32 softmax and accumulators)", config=config,
                e2e={"value": round(total / (e2e_ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s",
                     "h2d_bytes_per_step": 3 * q.numel() * 2 * world,
                     "d2h_bytes_per_step": (ch.numel() + sh.numel() * 4) * world},
                roofline=roof, gpu_launches=launches * args.steps,
                cpu_baseline_fn=lambda: cpu_baseline_attention())


def attention_context(stream, pk):
    """The library's attention kernel (fused projection quantizer) against cuDNN SDPA at the step's shape, for
    the default line (the step itself runs cuDNN)."""
    import torch.nn.functional as F
    from hy_nomas_b200 import attention as attn
    gen = torch.Generator(device="cuda").manual_seed(78)
    q, k, v = attn_inputs(ATTN_L, ATTN_L, gen, torch.device("cuda"))
    flops = 4.0 * ATTN_L * ATTN_L * ATTN_H * 128

    def ms(fn, it=5):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(it):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / it

    nat = ms(lambda: attn.attention_quant(q, k, v))
    ref = ms(lambda: F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)))
    return {"shape": f"{ATTN_L} x {ATTN_L} x {ATTN_H} heads x 128", "kernel": "hn::attn::k_attention",
            "native_fused_quant_ms": round(nat, 3), "native_tflops": round(flops / (nat * 1e-3) / 1e12, 1),
            "native_frac_of_bf16_burst": round(flops / (nat * 1e-3) / 1e12 / pk["bf16_tflops"], 3),
            "cudnn_sdpa_ms": round(ref, 3), "cudnn_sdpa_tflops": round(flops / (ref * 1e-3) / 1e12, 1),
            "step_uses": "cudnn_sdpa (faster); HN_ATTENTION=native switches the block to the kernel"}


def attention_cpu_sample(rows, gen):
    q = torch.randn(1, rows, ATTN_H, 128, generator=gen).to(torch.bfloat16)
    k = torch.randn(1, ATTN_L, ATTN_H, 128, generator=gen).to(torch.bfloat16)
    v = torch.randn(1, ATTN_L, ATTN_H, 128, generator=gen).to(torch.bfloat16)
    return q, k, v


def attention_cpu(q, k, v):
    """The reference's attention through torch SDPA (ComfyUI's pytorch backend, hy_nomas/model.py:145-151)."""
    import torch.nn.functional as F
    return F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)).transpose(1, 2)


def cpu_baseline_attention(budget_s=10.0):
    rows = 64
    q, k, v = attention_cpu_sample(rows, torch.Generator().manual_seed(6))
    attention_cpu(q, k, v)
    t0 = time.perf_counter()
    it = 0
    while time.perf_counter() - t0 < budget_s:
        attention_cpu(q, k, v)
        it += 1
    dt = (time.perf_counter() - t0) / it
    cores, threads = cpu_threads()
    return {"value": round(4.0 * rows * ATTN_L * ATTN_H * 128 / dt / 1e12, 4), "unit": "TFLOP/s", "cores": threads,
            "kind": "reference",
            "sample": f"{rows} of {ATTN_L} queries against all keys, {it} iterations in {budget_s:.0f}+ s (torch "
                      f"{torch.__version__} SDPA on bf16, {threads} threads on {cores} cores)"}


def reference_attention(args):
    """The reference's attention on the host: torch SDPA (its pytorch backend) on 64 of the 20240 queries per
    step against all keys."""
    rows = 64
    q, k, v = attention_cpu_sample(rows, torch.Generator().manual_seed(6))
    for _ in range(args.warmup):
        attention_cpu(q, k, v)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        attention_cpu(q, k, v)
    dt = time.perf_counter() - t0
    cores, threads = cpu_threads()
    return dict(metric="attention TFLOP/s (20240 x 20240 x 32 heads x 128)",
                value=round(4.0 * rows * ATTN_L * ATTN_H * 128 * args.steps / dt / 1e12, 4), unit="TFLOP/s",
                ms_per_step=round(dt / args.steps * 1e3, 3), higher_is_better=True, scaling="weak",
                dtype="bf16 (fp32 softmax and accumulators)", kind="reference", cores=threads,
                config={"workload": f"attention_L{ATTN_L}_H{ATTN_H}_D128 (configs 4/5)"},
                sample=f"{rows} of {ATTN_L} queries per step (torch SDPA on bf16, {threads} threads)")


WORKLOADS = {"dit": (workload_dit, reference_dit), "dit_gemms": (workload_dit_gemms, reference_dit_gemms),
             "attention": (workload_attention, reference_attention),
             "gemm": (workload_gemm, reference_gemm),
             "fp8": (workload_fp8, reference_fp8), "elementwise": (workload_elementwise, reference_elementwise)}


def run_reference(args, world, rank):
    """The reference's CPU path for the same workload and metric, rank 0 only (other ranks do no work and start
    no process group, so nothing else competes for the host's cores). Nothing of the product package is
    imported: the reference arm loads only torch and oracle/torch_ref.py."""
    if rank != 0:
        return None
    # all of the host's threads, pinned (torchrun sets OMP_NUM_THREADS=1 for its workers)
    torch.set_num_threads(len(os.sched_getaffinity(0)))
    r = WORKLOADS[args.workload][1](args)
    sample, kind, cores = r.pop("sample"), r.pop("kind"), r.pop("cores")
    line = {"metric": r["metric"], "value": r["value"], "unit": r["unit"], "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": r["higher_is_better"],
            "scaling": r["scaling"], "vs_baseline": None, "dtype": r["dtype"], "data": "synthetic (seeded)",
            "config": r["config"], "impl": "reference",
            "cpu_baseline": {"value": r["value"], "unit": r["unit"], "cores": cores, "kind": kind, "sample": sample},
            "e2e": {"value": r["value"], "unit": r["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    return line


def main():
    # the JSON line goes to the real stdout; everything else written to file descriptor 1 (NCCL's version
    # banner, library messages) is redirected to stderr so stdout carries exactly one line
    json_out = os.fdopen(os.dup(1), "w")
    sys.stdout.flush()
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default: 10 for dit, 50 otherwise; "
                                                            "3 for --impl reference)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="dit", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-context", action="store_true", help="dit: skip the configs 1-3 kernel measurements")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.steps is None:
        args.steps = 3 if args.impl == "reference" else (10 if args.workload == "dit" else 50)
    if args.impl == "reference":
        # the CPU arm: rank 0 alone works; no GPU and no process group are touched
        world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
        line = run_reference(args, world, rank)
        if line is not None:
            print(json.dumps(line), file=json_out, flush=True)
        return
    world, rank, local = init_dist()
    try:
        pk = peaks()
        stream = torch.cuda.current_stream()
        props = torch.cuda.get_device_properties(torch.cuda.current_device())
        bus = getattr(props, "pci_bus_id", None)
        sampler = ClockSampler([f"{getattr(props, 'pci_domain_id', 0):08x}:{bus:02x}:00.0"] if bus is not None else [],
                               enabled=(rank == 0))
        res = WORKLOADS[args.workload][0](args, world, rank, stream, pk, sampler)
        cpu_fn = res.pop("cpu_baseline_fn", None)
        if rank == 0:
            line = {"metric": res["metric"], "value": res["value"], "unit": res["unit"], "n_gpus": world,
                    "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
                    "higher_is_better": res["higher_is_better"], "scaling": res["scaling"], "vs_baseline": None,
                    "dtype": res["dtype"], "data": "synthetic (seeded)", "config": res["config"], "e2e": res["e2e"],
                    "roofline": res["roofline"], "gpu_launches": res["gpu_launches"], "clocks": sampler.result}
            if world == 1 and cpu_fn is not None and not args.no_cpu_baseline:
                line["cpu_baseline"] = cpu_fn()
            print(json.dumps(line), file=json_out, flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

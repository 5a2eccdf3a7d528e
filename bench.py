"""Benchmark of the optimizer-step path on B200 (and of the reference's CPU path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: one full TritonMuonSRWithAuxAdam(batch_ns=True) step on
Llama-3-8B-shaped synthetic tensors -- 224 hidden matrices in the Muon group (lr 0.02,
momentum 0.95, Nesterov, ns_steps 5, wd 0.01), embedding, head and 65 RMSNorm vectors in
the AdamW group -- bf16 params ~N(0, 0.02), grads ~N(0, 1e-3), seeded. Every tensor is far
larger than the 126 MB L2, so timed steps stream from HBM without an explicit flush.
The same run also times the 8-bit blockwise AdamW step on the same tensors.

``value`` is the device time of one full step (max over ranks, CUDA events), ``e2e`` the
same step through the public API with the step's gradients copied in from pinned host
memory and the updated weights copied back out (``HostStaging``: copies overlapped with the
step chunk by chunk; ``e2e_serial``: all uploads, then the step, then all downloads).
``--impl reference`` times the reference's pure-PyTorch MuonSR / AdamW-SR step (restated in
``oracle/``) on the host cores on a bounded sample and scales it to a full step.
"""
import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
# The sharded step's peer copies run on 2 streams per peer next to the compute stream; with
# CUDA's default 8 hardware queues a copy stream waiting on a peer's event can hold up the
# compute stream that shares its queue. Must be set before CUDA initialises.
os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "Llama-3-8B hybrid optimizer step ms; NS TFLOP/s; 8-bit AdamW HBM GB/s"
# dram__bytes_read.sum + dram__bytes_write.sum of one adamw8bit_kernel launch on 2^28 elements
# (block 256), from the capture summarised in profiles/adamw8bit_kernel_256M.md
A8_DRAM_BYTES_PER_ELEMENT = (1.619793e9 + 1.024948e9) / (1 << 28)
N_LAYERS, D, KV, FF, VOCAB = 32, 4096, 1024, 14336, 128256


def llama_shapes():
    muon = []
    for _ in range(N_LAYERS):
        muon += [(D, D), (KV, D), (KV, D), (D, D), (FF, D), (FF, D), (D, FF)]
    adam = [(VOCAB, D), (VOCAB, D)] + [(D,)] * (2 * N_LAYERS + 1)
    return muon, adam


def ns_flops(shape, steps=5):
    m, n = min(shape), max(shape)
    return steps * (4 * m * m * n + 2 * m ** 3)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], p["bf16_tflops_sustained"], "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


# ---------------------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except Exception:
            self.proc.kill()
            return None
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------
class Timers:
    """CUDA-event timers around the kernel wrappers (current stream), summed per name."""

    def __init__(self):
        self.events = {}
        self.enabled = False

    def wrap(self, mod, name):
        fn = getattr(mod, name)
        timers = self

        def timed(*a, **k):
            if not timers.enabled:
                return fn(*a, **k)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            out = fn(*a, **k)
            e.record()
            timers.events.setdefault(name, []).append((s, e))
            return out

        setattr(mod, name, timed)

    def totals_ms(self):
        return {k: sum(s.elapsed_time(e) for s, e in v) for k, v in self.events.items()}

    def counts(self):
        return {k: len(v) for k, v in self.events.items()}


def build_tensors(device, seed=0):
    muon_shapes, adam_shapes = llama_shapes()
    g = torch.Generator(device=device).manual_seed(seed)

    def mk(shape, std):
        t = torch.empty(shape, dtype=torch.bfloat16, device=device)
        t.normal_(0.0, std, generator=g)
        return torch.nn.Parameter(t)

    muon = [mk(s, 0.02) for s in muon_shapes]
    adam = [mk(s, 0.02) for s in adam_shapes]
    for p in muon + adam:
        p.grad = torch.empty_like(p).normal_(0.0, 1e-3, generator=g)
    return muon, adam


def time_steps(step_fn, steps, warmup, world):
    for _ in range(warmup):
        step_fn()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        step_fn()
    end.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end) / steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t)
    return ms


def run_ours(args, rank, world, local_rank):
    from muon_sr_b200 import Sharder, TritonAdamW8bit, TritonMuonSRWithAuxAdam, _lib
    from muon_sr_b200 import kernels as K

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    lib = _lib.load()
    hbm_gbs, tf_burst, tf_sus, peak_kind = peaks()
    muon, adam = build_tensors(device)
    shard = Sharder(reserve_sms=args.reserve_sms) if world > 1 else None
    opt = TritonMuonSRWithAuxAdam([
        dict(params=muon, use_muon=True, lr=0.02, momentum=0.95, weight_decay=0.01),
        dict(params=adam, use_muon=False, lr=3e-4, betas=(0.9, 0.95), eps=1e-10, weight_decay=0.01),
    ], batch_ns=True, shard=shard)

    timers = Timers()
    for name in ("newton_schulz", "muon_prepare", "muon_apply", "adamw_sr"):
        timers.wrap(K, name)
    if shard is not None:
        timers.wrap(Sharder, "sync_params")  # end of step: waits for the weight exchange
    # the optimizer module imported the wrappers by module reference (K.<name>), so the
    # wrapped functions are the ones it calls

    sampler = ClockSampler(local_rank)
    sampler.start()
    l0 = lib.msr_launch_count()
    timers.enabled = True
    for _ in range(args.warmup):
        opt.step()
    torch.cuda.synchronize()
    timers.events.clear()
    l0 = lib.msr_launch_count()
    ms = time_steps(opt.step, args.steps, 0, world)
    launches = lib.msr_launch_count() - l0
    clocks = sampler.stop()
    tot = timers.totals_ms()
    timers.enabled = False
    # host time to issue one step (the device still works on the previous one)
    host = []
    for _ in range(2):
        t0 = time.perf_counter()
        opt.step()
        host.append((time.perf_counter() - t0) * 1e3)
    torch.cuda.synchronize()
    host_ms = min(host)
    assert K.device_error() == 0, "device wait timed out in a kernel"

    # Newton-Schulz roofline: algorithmic FLOPs of the matrices this rank owned
    owned_flops = 0
    if shard is None:
        owned_flops = sum(ns_flops(tuple(p.shape)) for p in muon)
    else:
        owned_flops = sum(ns_flops(tuple(p.shape)) for p in muon if shard._owner[id(p)] == shard.rank)
    ns_ms_step = tot.get("newton_schulz", 0.0) / args.steps
    ns_tflops = owned_flops / (ns_ms_step * 1e-3) / 1e12 if ns_ms_step > 0 else None
    total_flops = sum(ns_flops(tuple(p.shape)) for p in muon)

    # elementwise bytes (per step, whole job)
    n_muon = sum(p.numel() for p in muon)
    n_adam = sum(p.numel() for p in adam)
    breakdown = {k: v / args.steps for k, v in tot.items()}
    breakdown["host_issue"] = host_ms
    per_rank = [breakdown]
    if world > 1:
        per_rank = [None] * world
        dist.all_gather_object(per_rank, breakdown)

    # elementwise kernels' algorithmic HBM rate (this rank's tensors)
    if shard is None:
        own_muon, own_adam = n_muon, n_adam
    else:
        own_muon = sum(p.numel() for p in muon if shard._owner[id(p)] == shard.rank)
        own_adam = sum(p.numel() for p in adam if shard._owner[id(p)] == shard.rank)

    def ew_rates(bd):
        out = {}
        for name, nbytes in (("muon_prepare", 8 * own_muon), ("muon_apply", 6 * own_muon), ("adamw_sr", 14 * own_adam)):
            if bd.get(name, 0) > 0 and nbytes:
                out[name] = nbytes / (bd[name] * 1e-3) / 1e9
        return out

    # ---- the same step with the opt-in fast noise stream (not the reference's bits) ----
    K.set_sr_noise("fast")
    timers.events.clear()
    timers.enabled = True
    fast_ms = time_steps(opt.step, args.steps, 1, world)
    timers.enabled = False
    fast_bd = {k: v / (args.steps + 1) for k, v in timers.totals_ms().items()}
    K.set_sr_noise("reference")
    fast_noise = {"value": fast_ms, "unit": "ms", "breakdown_ms_per_step": fast_bd,
                  "elementwise_hbm_gbs": ew_rates(fast_bd),
                  "note": "set_sr_noise('fast'): one Philox4x32-10 call per 8 rounded values; unbiased SR, "
                          "different bits than the reference; not the headline"}

    # ---- 8-bit blockwise AdamW on the same tensors ----
    params = muon + adam
    opt8 = TritonAdamW8bit([dict(params=params, optim_bits=8)], lr=1e-3, betas=(0.9, 0.999), eps=1e-8,
                           weight_decay=0.01, block_size=256, shard=shard)
    a8_timers = Timers()
    a8_timers.wrap(K, "adamw8bit")
    a8_timers.enabled = True
    for _ in range(args.warmup):
        opt8.step()
    torch.cuda.synchronize()
    a8_timers.events.clear()
    a8_step_ms = time_steps(opt8.step, args.steps, 0, world)
    a8_kernel_ms = a8_timers.totals_ms().get("adamw8bit", 0.0) / args.steps
    a8_timers.enabled = False
    n_all = n_muon + n_adam
    a8_bytes = n_all * 10 + 2 * 8 * math.ceil(n_all / 256)
    if shard is not None:
        owned = sum(p.numel() for p in params if shard._owner[id(p)] == shard.rank)
        a8_bytes_rank = owned * 10 + 16 * owned / 256
        a8_elems_rank = owned
    else:
        a8_bytes_rank = a8_bytes
        a8_elems_rank = n_all
    a8_gbs = a8_bytes_rank / (a8_kernel_ms * 1e-3) / 1e9 if a8_kernel_ms > 0 else None
    # the same 8-bit step with the opt-in fast noise stream
    K.set_sr_noise("fast")
    a8_timers.events.clear()
    a8_timers.enabled = True
    a8_fast_step_ms = time_steps(opt8.step, args.steps, 1, world)
    a8_fast_kernel_ms = a8_timers.totals_ms().get("adamw8bit", 0.0) / (args.steps + 1)
    a8_timers.enabled = False
    K.set_sr_noise("reference")
    fast_noise["adamw8bit_step_ms"] = a8_fast_step_ms
    fast_noise["adamw8bit_hbm_gbs"] = a8_bytes_rank / (a8_fast_kernel_ms * 1e-3) / 1e9 if a8_fast_kernel_ms else None
    del opt8
    torch.cuda.empty_cache()

    # ---- SR gradient accumulation (one micro-batch into every tensor through the
    # accumulator hook, after the first) and configs[1]: TritonAdamW on the GPT-2 AdamW set ----
    extra = {}
    if rank == 0:
        from muon_sr_b200 import TritonAdamW, TritonSRAccumulator
        grads = [p.grad for p in params]

        def micro_batch():
            for p, g in zip(params, grads):
                p.grad = g
                TritonSRAccumulator._accum_hook(p)

        micro_batch()  # first micro-batch creates the buffers
        acc_ms = time_steps(micro_batch, 3, 1, 1)
        for p, g in zip(params, grads):
            del p.acc_grad
            p.grad = g
        gg = torch.Generator(device=device).manual_seed(1)
        gpt2 = [torch.nn.Parameter(torch.empty(s, dtype=torch.bfloat16, device=device).normal_(0, 0.02, generator=gg))
                for s in [(50257, 768)] + [(768,)] * 24]
        for p in gpt2:
            p.grad = torch.empty_like(p).normal_(0, 1e-3, generator=gg)
        opt_a = TritonAdamW(gpt2, lr=3e-4, betas=(0.9, 0.95), eps=1e-10, weight_decay=0.01)
        aw_ms = time_steps(opt_a.step, 50, 5, 1)
        n_gpt2 = sum(p.numel() for p in gpt2)
        extra = {"sr_accum_ms_per_microbatch": acc_ms,
                 "sr_accum_hbm_gbs": 6 * n_all / (acc_ms * 1e-3) / 1e9,
                 "adamw_sr_gpt2_ms": aw_ms,
                 "adamw_sr_gpt2_hbm_gbs": 14 * n_gpt2 / (aw_ms * 1e-3) / 1e9}
        # configs[0] matrices + configs[1] vectors as one GPT-2-small hybrid step, eager and
        # replayed from a StepGraph: a short step, where the host's launch work shows
        from muon_sr_b200 import StepGraph
        mats = [torch.nn.Parameter(torch.empty(s, dtype=torch.bfloat16, device=device).normal_(0, 0.02, generator=gg))
                for _ in range(12) for s in ((768, 2304), (768, 768), (768, 3072), (3072, 768))]
        for p in mats:
            p.grad = torch.empty_like(p).normal_(0, 1e-3, generator=gg)
        opt_h = TritonMuonSRWithAuxAdam([
            dict(params=mats, use_muon=True, lr=0.02, momentum=0.95, weight_decay=0.01),
            dict(params=gpt2, use_muon=False, lr=3e-4, betas=(0.9, 0.95), eps=1e-10, weight_decay=0.01),
        ], batch_ns=True)

        def host_ms(fn, n=20):
            """Host time to issue one step, each call made with the GPU idle (no back-pressure)."""
            total = 0.0
            for _ in range(n):
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                fn()
                total += time.perf_counter() - t0
            torch.cuda.synchronize()
            return total * 1e3 / n

        eager_ms = time_steps(opt_h.step, 20, 3, 1)
        eager_host = host_ms(opt_h.step)
        extra.update({"gpt2_hybrid_step_ms": eager_ms, "gpt2_hybrid_host_issue_ms": eager_host,
                      "gpt2_hybrid_ns_tflops": sum(ns_flops(p.shape) for p in mats) / (eager_ms * 1e-3) / 1e12})
        # single-process runs only: a stream capture in global mode while an NCCL process group
        # is alive could make the communicator's background threads' CUDA calls fail
        if world == 1:
            try:
                sg = StepGraph(opt_h)
                extra.update({"gpt2_hybrid_step_ms_graph": time_steps(sg.step, 20, 3, 1),
                              "gpt2_hybrid_host_issue_ms_graph": host_ms(sg.step)})
                del sg
            except RuntimeError as exc:  # reported, not fatal: the headline does not use graphs
                extra["gpt2_hybrid_graph_error"] = str(exc)[:300]
        del opt_h, mats
        del opt_a, gpt2
        torch.cuda.empty_cache()

    # ---- end to end through the public API with host buffers ----
    # HostStaging: each step uploads the gradients it reads from pinned host memory and
    # downloads the weights it updates, overlapped with the step chunk by chunk; the step's
    # stream waits for both copy streams, so the events bracket every copy. e2e_serial is the
    # same step with all uploads before it and all downloads after it.
    e2e = e2e_serial = None
    if not args.no_e2e:
        from muon_sr_b200 import HostStaging
        pin_g = [torch.empty(p.shape, dtype=torch.bfloat16, pin_memory=True) for p in params]
        for h, p in zip(pin_g, params):
            h.copy_(p.grad)
        owned = [shard is None or shard._owner[id(p)] == shard.rank for p in params]
        pin_p = [torch.empty(p.shape, dtype=torch.bfloat16, pin_memory=True) if o else None
                 for p, o in zip(params, owned)]
        staged_error = None
        try:
            staged = HostStaging(opt, params, pin_g, pin_p)
            e2e_ms = time_steps(staged.step, max(2, args.steps // 2), 1, world)
            moved = torch.tensor([staged.h2d_bytes, staged.d2h_bytes], dtype=torch.float64, device="cuda")
            if world > 1:
                dist.all_reduce(moved)
            e2e = {"value": e2e_ms, "unit": "ms", "h2d_bytes_per_step": int(moved[0]),
                   "d2h_bytes_per_step": int(moved[1]),
                   "api": "HostStaging(optimizer, params, pinned host grads, pinned host weights).step()"}
            del staged
        except RuntimeError as exc:  # fall back to the serial copies below, and say so
            staged_error = str(exc)[:300]
            torch.cuda.synchronize()

        def serial_step():
            for h, p in zip(pin_g, params):
                p.grad.copy_(h, non_blocking=True)
            opt.step()
            for h, p in zip(pin_p, params):
                if h is not None:
                    h.copy_(p.detach(), non_blocking=True)

        serial_ms = time_steps(serial_step, max(2, args.steps // 2), 1, world)
        e2e_serial = {"value": serial_ms, "unit": "ms",
                      "h2d_bytes_per_step": sum(p.numel() * 2 for p in params) * world,
                      "d2h_bytes_per_step": sum(p.numel() * 2 for p in params)}
        if e2e is None:
            e2e = dict(e2e_serial, api="opt.step() between host copies", staged_error=staged_error)
        del pin_g, pin_p

    result = None
    if rank == 0:
        peak_ns = tf_sus
        result = {
            "metric": METRIC, "value": ms, "unit": "ms", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,0.02) params, N(0,1e-3) grads)",
            "config": {"workload": "configs[3]: TritonMuonSRWithAuxAdam(batch_ns=True) step, Llama-3-8B shapes",
                       "muon_matrices": len(muon), "adamw_tensors": len(adam), "elements": n_all,
                       "parallelism": f"param-sharded x{world}" if world > 1 else "single GPU",
                       "l2": "inputs > L2 (126 MB), no flush"},
            "ns_tflops": ns_tflops, "ns_tflop_per_step": total_flops / 1e12,
            "adamw8bit_hbm_gbs": a8_gbs, "adamw8bit_step_ms": a8_step_ms, "adamw8bit_kernel_ms": a8_kernel_ms,
            "breakdown_ms_per_step": breakdown,
            "elementwise_hbm_gbs": ew_rates(breakdown),
            "fast_noise": fast_noise,
            "breakdown_ms_per_step_per_rank": per_rank if world > 1 else None,
            "roofline": {"bound": "tensor", "kernel": "gemm_pair_kernel (Newton-Schulz chain)",
                         "achieved": ns_tflops, "peak": peak_ns, "unit": "TFLOP/s",
                         "frac": (ns_tflops / peak_ns) if ns_tflops else None,
                         "peak_kind": f"bf16_tflops_sustained ({peak_kind})", "traffic": None,
                         "traffic_note": "tensor-bound chain of mixed shapes; per-launch DRAM bytes equal the "
                                         "algorithmic operand bytes (profiles/gemm_pair_kernel_ns_4x4096.md)"},
            "roofline_8bit": {"bound": "hbm", "kernel": "adamw8bit_kernel", "achieved": a8_gbs, "peak": hbm_gbs,
                              "unit": "GB/s", "frac": (a8_gbs / hbm_gbs) if a8_gbs else None,
                              "algorithmic_bytes": a8_bytes,
                              "traffic": A8_DRAM_BYTES_PER_ELEMENT * a8_elems_rank,
                              "traffic_note": "DRAM bytes per element of a 2^28-element ncu capture "
                                              "(profiles/adamw8bit_kernel_256M.md) scaled to the elements "
                                              "this rank updates per step, like achieved"},
            "other_configs": extra,
            "gpu_launches": int(launches),
            "clocks": clocks,
            "e2e": e2e,
            "e2e_serial": e2e_serial,
        }
    return result


# ---------------------------------------------------------------------------------------
# CPU (reference) arm -- the reference's pure-PyTorch MuonSR / AdamW-SR restated in oracle/
# ---------------------------------------------------------------------------------------
CPU_SAMPLE = ("per step: three MuonSR parameter steps (oracle.muon_cpu, restating muon_sr/muon_sr.py) for each "
              "of the four distinct Llama-3-8B matrix shapes, scaled by that shape's count, plus an AdamW-SR "
              "step on a 2^23-element slice scaled by elements to the 1.05G-element AdamW group")


def cpu_sample_step(threads):
    """One bounded sample of the full Llama step on the host cores: MuonSR parameter steps
    for three matrices of each distinct shape (q/o, k/v, gate/up, down), scaled by that
    shape's count, and an AdamW-SR step on a 2^23-element slice scaled by elements.
    Returns (extrapolated milliseconds per full step, seconds of CPU work in the sample)."""
    from oracle.muon_cpu import adamw_sr_step, muon_sr_step
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    muon_shapes, adam_shapes = llama_shapes()
    counts = {}
    for s in muon_shapes:
        counts[s] = counts.get(s, 0) + 1
    full = 0.0
    work = 0.0
    per_shape = 3  # matrices sampled per distinct shape
    for shape, count in counts.items():
        for _ in range(per_shape):
            p = (torch.randn(*shape, generator=g) * 0.02).bfloat16()
            gr = (torch.randn(*shape, generator=g) * 1e-3).bfloat16()
            b = torch.zeros_like(p)
            t0 = time.perf_counter()
            muon_sr_step([p], [gr], [b], lr=0.02, weight_decay=0.01)
            dt = time.perf_counter() - t0
            full += dt * count / per_shape
            work += dt
    n_slice = 1 << 23
    pa = (torch.randn(n_slice, generator=g) * 0.02).bfloat16()
    ga = (torch.randn(n_slice, generator=g) * 1e-3).bfloat16()
    ea, eb = torch.zeros_like(pa), torch.zeros_like(pa)
    t0 = time.perf_counter()
    adamw_sr_step([pa], [ga], [ea], [eb], 1, weight_decay=0.01)
    dt = time.perf_counter() - t0
    full += dt * sum(math.prod(s) for s in adam_shapes) / n_slice
    work += dt
    return full * 1e3, work


def run_reference(args, rank):
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    sample = CPU_SAMPLE
    for _ in range(args.warmup):
        cpu_sample_step(threads)
    vals = [cpu_sample_step(threads)[0] for _ in range(args.steps)]
    v = statistics.median(vals)
    return {"impl": "reference", "metric": METRIC, "value": v, "unit": "ms", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": v, "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "configs[3]: hybrid Muon+AdamW SR step, Llama-3-8B shapes (CPU, sampled)"},
            "cpu_baseline": {"value": v, "unit": "ms", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_kernel_case(args):
    """Single-kernel cases for profiling (``--kernel``): a few GB on the device, inputs larger
    than L2, each kernel launched warmup + steps times; prints per-launch times."""
    from muon_sr_b200 import kernels as K
    from muon_sr_b200.adamw8bit import create_dynamic_map
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    out = {"kernel": args.kernel}
    if args.kernel == "ns":
        shape = (4, D, D) if args.small else (16, D, D)
        x = torch.empty(shape, dtype=torch.bfloat16, device=dev).normal_(0, 1e-3, generator=g)
        fn = lambda: K.newton_schulz(x, 5)
        work = shape[0] * ns_flops(shape[1:]) / 1e12
        unit = "TFLOP/s"
    else:
        n = (1 << 28) if args.small else (1 << 30)
        p = torch.empty(n, dtype=torch.bfloat16, device=dev).normal_(0, 0.02, generator=g)
        gr = torch.empty_like(p).normal_(0, 1e-3, generator=g)
        if args.kernel == "adamw8bit":
            s1 = torch.full((n,), 127, dtype=torch.uint8, device=dev)
            s2 = torch.zeros(n, dtype=torch.uint8, device=dev)
            a1 = torch.zeros(n // 256, device=dev)
            a2 = torch.zeros_like(a1)
            q1, q2 = create_dynamic_map(True).to(dev), create_dynamic_map(False).to(dev)
            qt = K.quant_tables(q1, q2)
            fn = lambda: K.adamw8bit([(p, gr, s1, s2, a1, a2, 1, 7, True)], q1, q2, 1e-3, 0.9, 0.999, 1e-8, 0.01, 256,
                                     qtables=qt)
            work = (n * 10 + n // 256 * 16) / 1e9
        elif args.kernel == "adamw":
            m, v = torch.zeros_like(p), torch.zeros_like(p)
            fn = lambda: K.adamw_sr([(p, gr, m, v, 1, 7)], 3e-4, 0.9, 0.95, 1e-10, 0.01)
            work = n * 14 / 1e9
        elif args.kernel == "prepare":
            buf, upd = torch.zeros_like(p), torch.empty_like(p)
            fn = lambda: K.muon_prepare([(gr, buf, upd, 0, 7)], 0.95, True)
            work = n * 8 / 1e9
        else:  # apply
            upd = torch.empty_like(p).normal_(0, 0.1, generator=g)
            fn = lambda: K.muon_apply([(p, upd, 1.0, 7)], 0.02, 0.01)
            work = n * 6 / 1e9
        unit = "GB/s"
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        fn()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / args.steps
    out.update({"ms_per_call": ms, "rate": work / (ms * 1e-3), "unit": unit, "small": bool(args.small)})
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernel", choices=["ns", "adamw8bit", "adamw", "prepare", "apply"],
                    help="time one kernel alone (profiling cases) instead of the optimizer step")
    ap.add_argument("--small", action="store_true", help="with --kernel: the few-GB profiling size")
    ap.add_argument("--reserve-sms", type=int, default=int(os.environ.get("MSR_RESERVE_SMS", "0")),
                    help="N>1: SMs the GEMMs leave to the concurrent weight broadcasts")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.kernel:
        run_kernel_case(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        out = run_reference(args, rank)
        if out is not None:
            print(json.dumps(out), flush=True)
        return

    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        out = run_ours(args, rank, world, local_rank)
        if rank == 0:
            if world == 1 and not args.no_cpu_baseline:
                v, secs = cpu_sample_step(os.cpu_count() or 1)
                out["cpu_baseline"] = {"value": v, "unit": "ms", "cores": os.cpu_count() or 1, "kind": "port",
                                       "sample": f"{CPU_SAMPLE} ({secs:.1f} s of CPU work)"}
            print(json.dumps(out), flush=True)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

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
``--impl reference`` times the reference's own pure-PyTorch ``MuonSRWithAuxAdam`` step (the
unmodified package installed in ``baseline/_ref``; the ``oracle/`` restatement only if that
install is missing) on the host cores, on a bounded sample scaled to a full step
(``extrapolated`` in the line says so).

With one GPU the line also carries ``reference_gpu``: the reference's own Triton kernels and
torch/cuBLAS Newton-Schulz (``baseline/_ref``) timed on the same GPU on the same synthetic
inputs, beside this engine's numbers for the same work, and ``cpu_reference_configs0``: the
reference's ``MuonSR.step()`` on the whole GPT-2-small matrix set on the host
cores, not extrapolated. With several GPUs, ``sharded_bit_identical`` reports whether a small
sharded hybrid step and 8-bit step wrote the same bits as the unsharded step on every rank.
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
# (block 256), from an ncu capture of ``bench.py --kernel adamw8bit --small``
A8_DRAM_BYTES_PER_ELEMENT = (1.619793e9 + 1.024948e9) / (1 << 28)
REF_DIR = os.path.join(ROOT, "baseline", "_ref")
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
    shard = Sharder(reserve_sms=args.reserve_sms, transport=args.transport) if world > 1 else None
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

    # ---- N > 1: the gradients' reduce-scatter onto their owners (Sharder.reduce_grads) ----
    grad_rs = None
    if world > 1:
        lay = shard.reduce_grads(opt)  # first call packs the gradients and makes them views (untimed)
        rs_ms = time_steps(lambda: shard.reduce_grads(opt), 3, 1, world)
        nbytes = world * lay["chunk_elements"] * 2
        grad_rs = {"ms": rs_ms, "collective": "one NCCL reduce-scatter (AVG) over the owner-ordered packed bf16 "
                                              "gradient buffer, in place",
                   "buffer_bytes": nbytes, "padding": lay["padding"], "tensors": lay["tensors"],
                   "bus_gbs": nbytes / (rs_ms * 1e-3) / 1e9 * (world - 1) / world}

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

    # ---- after the measurements: the reference's GPU path (1 GPU), sharded parity (N > 1) ----
    del opt
    torch.cuda.empty_cache()
    ref_gpu = sharded = None
    if world == 1 and not args.no_reference_gpu:
        try:
            ref_gpu = reference_gpu(args, device, muon, adam)
        except Exception as exc:  # reported in the line; the engine's numbers above stand
            ref_gpu = {"error": f"{type(exc).__name__}: {exc}"[:400]}
        torch.cuda.empty_cache()
    if world > 1:
        sharded = sharded_bit_check(device, args.transport)

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
                       "weight_exchange": shard.transport if shard is not None else None,
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
                                         "algorithmic operand bytes (ncu capture of bench.py --kernel ns --small)"},
            "roofline_8bit": {"bound": "hbm", "kernel": "adamw8bit_kernel", "achieved": a8_gbs, "peak": hbm_gbs,
                              "unit": "GB/s", "frac": (a8_gbs / hbm_gbs) if a8_gbs else None,
                              "algorithmic_bytes": a8_bytes,
                              "traffic": A8_DRAM_BYTES_PER_ELEMENT * a8_elems_rank,
                              "traffic_note": "DRAM bytes per element of a 2^28-element ncu capture "
                                              "(bench.py --kernel adamw8bit --small) scaled to the elements "
                                              "this rank updates per step, like achieved"},
            "other_configs": extra,
            "gpu_launches": int(launches),
            "clocks": clocks,
            "e2e": e2e,
            "e2e_serial": e2e_serial,
        }
        if ref_gpu is not None:
            result["reference_gpu"] = ref_gpu
        if sharded is not None:
            result["sharded_bit_identical"] = sharded
        if grad_rs is not None:
            result["grad_reduce_scatter"] = grad_rs
    return result


def sharded_bit_check(device, transport):
    """N > 1: the sharded step writes the single-GPU bits. A small hybrid Muon + AdamW step
    (batch_ns, two steps) and an 8-bit AdamW step run twice from the same weights and
    gradients on every rank -- once sharded over all ranks (``Sharder``), once unsharded on
    this rank's GPU -- and every weight is compared bit for bit; the mismatch count is
    summed over ranks."""
    from muon_sr_b200 import Sharder, TritonAdamW8bit, TritonMuonSRWithAuxAdam
    g = torch.Generator().manual_seed(123)
    mshapes = [(256, 512)] * 6 + [(512, 256)] * 4 + [(384, 384)] * 3 + [(1024, 256)] * 2
    shapes = mshapes + [(2000, 256), (256,), (256,), (512,)]
    init = [(torch.randn(shp, generator=g) * 0.02).bfloat16() for shp in shapes]
    grads = [[(torch.randn(shp, generator=g) * 1e-3).bfloat16().to(device) for shp in shapes] for _ in range(2)]
    nm = len(mshapes)

    def hybrid(ps, sh):
        return TritonMuonSRWithAuxAdam([
            dict(params=ps[:nm], use_muon=True, lr=0.02, momentum=0.95, weight_decay=0.01),
            dict(params=ps[nm:], use_muon=False, lr=3e-4, betas=(0.9, 0.95), eps=1e-10, weight_decay=0.01)],
            batch_ns=True, shard=sh)

    def eight_bit(ps, sh):
        return TritonAdamW8bit([dict(params=ps, optim_bits=8)], lr=1e-3, weight_decay=0.01, shard=sh)

    bad = compared = 0
    for make in (hybrid, eight_bit):
        pa = [torch.nn.Parameter(t.to(device)) for t in init]
        pb = [torch.nn.Parameter(t.to(device)) for t in init]
        oa, ob = make(pa, Sharder(transport=transport)), make(pb, None)
        for gs in grads:
            for p, q, gr in zip(pa, pb, gs):
                p.grad = gr.clone()
                q.grad = gr.clone()
            oa.step()
            ob.step()
        torch.cuda.synchronize()
        bad += sum(int(not torch.equal(p.detach().view(torch.int16), q.detach().view(torch.int16)))
                   for p, q in zip(pa, pb))
        compared += len(pa)
        del oa, ob
    t = torch.tensor([bad], dtype=torch.int64, device=device)
    dist.all_reduce(t)
    return {"identical": int(t.item()) == 0, "mismatched_tensors_all_ranks": int(t.item()),
            "tensors_per_rank": compared,
            "what": "hybrid Muon+AdamW (batch_ns, 2 steps) and 8-bit AdamW (2 steps), 19 tensors each, "
                    "sharded over all ranks vs unsharded on each rank"}


# ---------------------------------------------------------------------------------------
# the reference itself (baseline/_ref): CPU arm, configs[0] on the CPU, GPU path on this GPU
# ---------------------------------------------------------------------------------------
def reference_module():
    """(the unmodified reference package installed in baseline/_ref, None) or (None, why not)."""
    if not os.path.isdir(os.path.join(REF_DIR, "muon_sr")):
        return None, "baseline/_ref is not installed"
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    try:
        import muon_sr
    except Exception as exc:  # e.g. triton missing: the reference imports it at module load
        return None, f"importing the reference failed: {type(exc).__name__}: {exc}"[:300]
    return muon_sr, None


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


CPU_SAMPLE = ("per step: one MuonSRWithAuxAdam(batch_ns=True) step per distinct Llama-3-8B matrix shape (one "
              "matrix each: q/o 4096x4096, k/v 1024x4096, gate/up 14336x4096, down 4096x14336) scaled by that "
              "shape's count, plus the AdamW group's step on a 2^22-element slice scaled by elements to the "
              "1.05G-element AdamW group")
_cpu_opts = {}


def cpu_sample_step(threads):
    """One bounded sample of the full Llama step on the host cores: the reference's own
    ``MuonSRWithAuxAdam(batch_ns=True)`` (baseline/_ref; the oracle's restatement if the
    install is missing) on one matrix of each distinct shape, each timed on its own and scaled
    by that shape's count, and on an AdamW-group slice scaled by elements. The optimizers are
    built once and reused, so warm-up steps create their state and timed steps are steady.
    Returns (extrapolated ms per full step, seconds of CPU work actually timed, kind)."""
    torch.set_num_threads(threads)
    ref, _ = reference_module()
    muon_shapes, adam_shapes = llama_shapes()
    counts = {}
    for shp in muon_shapes:
        counts[shp] = counts.get(shp, 0) + 1
    n_slice = 1 << 22
    n_adam = sum(math.prod(shp) for shp in adam_shapes)
    if not _cpu_opts:
        g = torch.Generator().manual_seed(0)

        def param(shape):
            p = torch.nn.Parameter((torch.randn(*shape, generator=g) * 0.02).bfloat16())
            p.grad = (torch.randn(*shape, generator=g) * 1e-3).bfloat16()
            return p
        for shape in counts:
            p = param(shape)
            if ref is not None:
                opt = ref.MuonSRWithAuxAdam([dict(params=[p], use_muon=True, lr=0.02, momentum=0.95,
                                                  weight_decay=0.01)], batch_ns=True)
                _cpu_opts[shape] = (opt.step, counts[shape])
            else:
                from oracle.muon_cpu import muon_sr_step
                buf = torch.zeros_like(p)
                _cpu_opts[shape] = ((lambda p=p, b=buf: muon_sr_step([p], [p.grad], [b], lr=0.02,
                                                                      weight_decay=0.01)), counts[shape])
        pa = param((n_slice,))
        if ref is not None:
            opt = ref.MuonSRWithAuxAdam([dict(params=[pa], use_muon=False, lr=3e-4, betas=(0.9, 0.95), eps=1e-10,
                                              weight_decay=0.01)], batch_ns=True)
            _cpu_opts["adamw"] = (opt.step, n_adam / n_slice)
        else:
            from oracle.muon_cpu import adamw_sr_step
            ea, eb = torch.zeros_like(pa), torch.zeros_like(pa)
            _cpu_opts["adamw"] = ((lambda: adamw_sr_step([pa], [pa.grad], [ea], [eb], 1, weight_decay=0.01)),
                                  n_adam / n_slice)
    full = work = 0.0
    for fn, scale in _cpu_opts.values():
        t0 = time.perf_counter()
        fn()
        dt = time.perf_counter() - t0
        full += dt * scale
        work += dt
    return full * 1e3, work, ("reference" if ref is not None else "port")


def cpu_reference_configs0(threads):
    """configs[0] on the host cores, whole and unextrapolated: the reference's ``MuonSR``
    (baseline/_ref) on the GPT-2-small matrix set -- 12 x {768x2304, 768x768, 768x3072,
    3072x768} bf16 params N(0, 0.02), grads N(0, 1e-3), momentum 0.95, Nesterov, ns_steps 5,
    lr 0.02, wd 0.01 -- one warm-up step and the best of 3, with batch_ns False and True."""
    ref, why = reference_module()
    if ref is None:
        return {"unavailable": why}
    torch.set_num_threads(threads)
    out = {"cores": threads, "cpu_model": cpu_model(), "unit": "ms", "matrices": 48,
           "ns_tflop_per_step": 12 * sum(ns_flops(shp) for shp in GPT2_MATS) / 1e12}
    for batch in (False, True):
        g = torch.Generator().manual_seed(0)
        ps = []
        for _ in range(12):
            for shp in GPT2_MATS:
                p = torch.nn.Parameter((torch.randn(*shp, generator=g) * 0.02).bfloat16())
                p.grad = (torch.randn(*shp, generator=g) * 1e-3).bfloat16()
                ps.append(p)
        opt = ref.MuonSR(ps, lr=0.02, weight_decay=0.01, momentum=0.95, nesterov=True, ns_steps=5, batch_ns=batch)
        opt.step()
        best = float("inf")
        for _ in range(3):
            t0 = time.perf_counter()
            opt.step()
            best = min(best, time.perf_counter() - t0)
        out[f"batch_ns_{str(batch).lower()}_ms"] = best * 1e3
    return out


GPT2_MATS = ((768, 2304), (768, 768), (768, 3072), (3072, 768))


def run_reference(args, rank):
    """The reference arm: the reference's CPU path on the host cores (rank 0 only)."""
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        cpu_sample_step(threads)
    samples = [cpu_sample_step(threads) for _ in range(args.steps)]
    v = statistics.median(x[0] for x in samples)
    kind = samples[0][2]
    timed_s = sum(x[1] for x in samples)
    sample = CPU_SAMPLE + (" (the reference's own classes from baseline/_ref)" if kind == "reference" else
                           " (the oracle's restatement: baseline/_ref is not installed)")
    return {"impl": "reference", "metric": METRIC, "value": v, "unit": "ms", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": v, "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "configs[3]: MuonSRWithAuxAdam(batch_ns=True) step, Llama-3-8B shapes, on the "
                                   "host cores (sampled, extrapolated)"},
            "extrapolated": True, "cpu_seconds_timed": timed_s,
            "cpu_baseline": {"value": v, "unit": "ms", "cores": threads, "kind": kind, "sample": sample,
                             "cpu_model": cpu_model(), "extrapolated": True},
            "e2e": {"value": v, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def reference_gpu(args, device, muon, adam):
    """The reference's own GPU path (baseline/_ref: its Triton kernels and its torch/cuBLAS
    Newton-Schulz, unmodified, through its public classes) on this GPU, on the same synthetic
    tensors, next to this engine on the same work. CUDA events on the current stream, the
    reference's steps after its own warm-up (Triton compiles on the first call)."""
    ref, why = reference_module()
    if ref is None:
        return {"unavailable": why}
    from muon_sr_b200 import TritonAdamW, TritonAdamW8bit, TritonMuonSR, TritonMuonSRWithAuxAdam, TritonSRAccumulator
    from muon_sr_b200 import kernels as K
    from muon_sr.muon_sr import _newton_schulz as ref_ns
    steps, warm = min(args.steps, 5), 3
    out = {"steps": steps, "warmup": warm, "unit": "ms", "source": "baseline/_ref (pip install of the reference)"}

    def pair(name, ours_fn, ref_fn, st=steps, wu=warm):
        o = time_steps(ours_fn, st, wu, 1)
        r = time_steps(ref_fn, st, wu, 1)
        out[name] = {"reference_ms": r, "ours_ms": o, "speedup": r / o}
        torch.cuda.empty_cache()

    groups = lambda m, a: [dict(params=m, use_muon=True, lr=0.02, momentum=0.95, weight_decay=0.01),
                           dict(params=a, use_muon=False, lr=3e-4, betas=(0.9, 0.95), eps=1e-10, weight_decay=0.01)]
    # the full hybrid step
    ours = TritonMuonSRWithAuxAdam(groups(muon, adam), batch_ns=True)
    theirs = ref.TritonMuonSRWithAuxAdam(groups(muon, adam), batch_ns=True)
    pair("configs3_hybrid_step", ours.step, theirs.step)
    del ours, theirs
    torch.cuda.empty_cache()
    # 8-bit blockwise AdamW on the same tensors
    params = muon + adam
    kw = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, block_size=256)
    ours = TritonAdamW8bit([dict(params=params, optim_bits=8)], **kw)
    theirs = ref.TritonAdamW8bit([dict(params=params, optim_bits=8)], **kw)
    pair("configs2_adamw8bit_step", ours.step, theirs.step)
    out["configs2_adamw8bit_step"]["algorithmic_gb"] = (10 * sum(p.numel() for p in params)
                                                        + 16 * sum(math.ceil(p.numel() / 256) for p in params)) / 1e9
    del ours, theirs
    torch.cuda.empty_cache()
    # one SR-accumulation micro-batch (after the first) through each one's hook
    grads = [p.grad for p in params]

    def micro(hook):
        def run():
            for p, g in zip(params, grads):
                p.grad = g
                hook(p)
        return run
    for hook in (TritonSRAccumulator._accum_hook, ref.TritonSRAccumulator._accum_hook):
        micro(hook)()
        o = time_steps(micro(hook), steps, 1, 1)
        out.setdefault("configs4_sr_accum_microbatch", {})["ours_ms" if hook is TritonSRAccumulator._accum_hook
                                                          else "reference_ms"] = o
        for p, g in zip(params, grads):
            del p.acc_grad
            p.grad = g
    c4 = out["configs4_sr_accum_microbatch"]
    c4["speedup"] = c4["reference_ms"] / c4["ours_ms"]
    torch.cuda.empty_cache()
    # TritonAdamW on the GPT-2 AdamW set; configs[0]'s matrices as a TritonMuonSR step
    gg = torch.Generator(device=device).manual_seed(1)
    mk = lambda shp, std: torch.empty(shp, dtype=torch.bfloat16, device=device).normal_(0, std, generator=gg)
    gpt2 = [torch.nn.Parameter(mk(shp, 0.02)) for shp in [(50257, 768)] + [(768,)] * 24]
    mats = [torch.nn.Parameter(mk(shp, 0.02)) for _ in range(12) for shp in GPT2_MATS]
    for p in gpt2 + mats:
        p.grad = mk(p.shape, 1e-3)
    kw = dict(lr=3e-4, betas=(0.9, 0.95), eps=1e-10, weight_decay=0.01)
    ours, theirs = TritonAdamW(gpt2, **kw), ref.TritonAdamW(gpt2, **kw)
    pair("configs1_adamw_step", ours.step, theirs.step, st=50, wu=5)
    ours = TritonMuonSR(mats, lr=0.02, weight_decay=0.01, batch_ns=True)
    theirs = ref.TritonMuonSR(mats, lr=0.02, weight_decay=0.01, batch_ns=True)
    pair("configs0_gpt2_muon_step", ours.step, theirs.step, st=20, wu=3)
    del ours, theirs, gpt2, mats
    torch.cuda.empty_cache()
    # Newton-Schulz per shape: the stacks one chunk of each configuration's step holds
    ns = {}
    for name, shape in (("q/o", (16, D, D)), ("k/v", (64, KV, D)), ("gate/up", (4, FF, D)), ("down", (4, D, FF)),
                        ("gpt2 768x2304", (12, 768, 2304)), ("gpt2 768x768", (12, 768, 768)),
                        ("gpt2 768x3072", (12, 768, 3072)), ("gpt2 3072x768", (12, 3072, 768))):
        x = torch.empty(shape, dtype=torch.bfloat16, device=device).normal_(0, 1e-3, generator=gg)
        flops = shape[0] * ns_flops(shape[1:]) / 1e12
        o = time_steps(lambda: K.newton_schulz(x, 5), steps, warm, 1)
        r = time_steps(lambda: ref_ns(x, 5, None), steps, warm, 1)
        ns[name] = {"shape": list(shape), "ours_tflops": flops / (o * 1e-3), "reference_tflops": flops / (r * 1e-3),
                    "speedup": r / o}
        del x
        torch.cuda.empty_cache()
    out["newton_schulz_effective_tflops"] = ns
    return out


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
        if args.ns_shape:
            shape = tuple(int(v) for v in args.ns_shape.split("x"))
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
        elif args.kernel == "centralize":
            rows = n // 4096  # [rows, 4096]: one mean per row, the row read twice (the second from cache)
            gm = gr.view(rows, 4096)
            fn = lambda: K.centralize(gm, 0.5)
            work = n * 4 / 1e9
        elif args.kernel == "accum":
            acc = torch.empty_like(p).normal_(0, 1e-3, generator=g)
            fn = lambda: K.grad_accum_(acc, gr, 1234)
            work = n * 6 / 1e9
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
    out.update({"ms_per_call": ms, "rate": work / (ms * 1e-3), "unit": unit, "small": bool(args.small),
                "noise": args.noise})
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's own GPU path (baseline/_ref) next to the engine")
    ap.add_argument("--kernel", choices=["ns", "adamw8bit", "adamw", "prepare", "apply", "accum", "centralize"],
                    help="time one kernel alone (profiling cases) instead of the optimizer step")
    ap.add_argument("--small", action="store_true", help="with --kernel: the few-GB profiling size")
    ap.add_argument("--ns-shape", default=None,
                    help="with --kernel ns: the stack as BATCHxROWSxCOLS (e.g. 12x768x3072)")
    ap.add_argument("--noise", choices=["reference", "fast", "none"], default="reference",
                    help="with --kernel: the stochastic-rounding noise stream")
    ap.add_argument("--transport", choices=["auto", "multicast", "p2p", "nccl"], default="auto",
                    help="N>1: how the sharded step shares the updated weights (Sharder transport)")
    ap.add_argument("--reserve-sms", type=int, default=int(os.environ.get("MSR_RESERVE_SMS", "0")),
                    help="N>1: SMs the GEMMs leave to the concurrent weight broadcasts")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.kernel:
        from muon_sr_b200 import kernels as K
        K.set_sr_noise(args.noise)
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
                threads = os.cpu_count() or 1
                cpu_sample_step(threads)  # builds the sampled optimizers' state (untimed)
                v, secs, kind = cpu_sample_step(threads)
                out["cpu_baseline"] = {"value": v, "unit": "ms", "cores": threads, "kind": kind,
                                       "cpu_model": cpu_model(), "extrapolated": True,
                                       "cpu_seconds_timed": secs, "sample": CPU_SAMPLE}
                out["cpu_reference_configs0"] = cpu_reference_configs0(threads)
            print(json.dumps(out), flush=True)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

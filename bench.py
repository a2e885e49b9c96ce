#!/usr/bin/env python
"""Optimizer-step benchmark (BASELINE.json metric: NorMuon+AdamW step ms, L14 d1024).

    python bench.py [--gpus N --steps K --warmup W] [--impl engine|reference] [--device cpu|cuda]

engine arm (default): the L14/d1024/d_ff 5632/V 32768 recipe parameter set
on seeded synthetic bf16 tensors resident in HBM; one
step = muon.step(); adamw.step(); ema.update() through the drop-in API
(build_optimizers + EmaWeights). Prints one JSON line with the step time, the
Gram Newton-Schulz GEMM roofline (denominator chosen from the clocks of the
run it is measured in), the end-to-end time through the same API with host
gradients copied in and a result read back; at N = 1 also the configs[2] /
configs[3] micro-benchmarks, the reference's step run by torch on the same
GPU and the CPU baseline. With N > 1 (torchrun), the step is sharded by
matrices / table rows, the updated bf16 weights are exchanged over NVLink
(copy-engine pushes and NCCL), time = max over ranks, and the line carries a
bitwise comparison of every rank's results with the unsharded engine.

reference arm: the reference's own optimizer math (the CPU oracle, bit-exact
with transformer_lm.sol_modules on CPU) on the host cores, on a 1/14 sample of
the same workload (one layer's matrices and 1/14 of every vocabulary table)
scaled to a full step. ``--device cuda`` runs the same torch code on the GPU
over the full workload (the reference's GPU step with its quintic fallback).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "cs336-a1-sol_b200"))

from sol_b200 import EmaWeights, _lib, build_optimizers, synth  # noqa: E402
from sol_b200.sharding import ShardedStep  # noqa: E402

RECIPE = dict(muon_lr=8e-3, adam_lr=1.2e-2, embed_lr=2.4e-2, weight_decay=0.1, cautious_wd=True, bf16_master=True)
MOM_WARMUP = 300
# dram__bytes_read.sum + dram__bytes_write.sum per tensor-core GEMM launch,
# averaged over the 30 launches of one L14 step, from a one-pass ncu capture
# of this benchmark's default configuration on one GPU (not measured by the
# run that prints it; reported for that configuration only).
GEMM_TRAFFIC_BYTES_PER_LAUNCH = 2.163e8


def peaks():
    """(bf16 burst TF/s, bf16 sustained TF/s, HBM GB/s, "measured" | "fallback")."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        burst = float(d["bf16_tflops"])
        return burst, float(d.get("bf16_tflops_sustained", burst)), float(d["hbm_gbs"]), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """SM clock and clock-event (throttle) reasons during the timed region,
    read through NVML (reads only) every few milliseconds from a thread, so
    that short timed regions (a sharded step on 8 GPUs takes ~1.5 ms) still
    get samples. The device is matched by UUID / PCI bus id, not by index."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, index, period_s=0.004):
        self.index = index
        self.period = period_s
        self.samples = []
        self.nvml = None
        self.t0 = 0.0

    def _handle(self, nv):
        props = torch.cuda.get_device_properties(self.index)
        uuid = str(getattr(props, "uuid", ""))
        for cand in (uuid, "GPU-" + uuid):
            try:
                return nv.nvmlDeviceGetHandleByUUID(cand.encode() if isinstance(cand, str) else cand)
            except Exception:  # noqa: BLE001
                pass
        try:
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            return nv.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:  # noqa: BLE001
            return nv.nvmlDeviceGetHandleByIndex(self.index)

    def start(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nvml = nv
            self.handle = self._handle(nv)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(self.handle, nv.NVML_CLOCK_SM))
        except Exception as e:  # noqa: BLE001
            self.nvml = None
            self.error = f"NVML unavailable: {type(e).__name__}"
            return
        self.stop_flag = threading.Event()

        def poll():
            while not self.stop_flag.is_set():
                try:
                    sm = self.nvml.nvmlDeviceGetClockInfo(self.handle, self.nvml.NVML_CLOCK_SM)
                    rs = self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                    self.samples.append((time.time(), float(sm), int(rs)))
                except Exception:  # noqa: BLE001
                    pass
                self.stop_flag.wait(self.period)

        self.thread = threading.Thread(target=poll, daemon=True)
        self.thread.start()

    def mark(self):
        """Start of the timed region (samples before it are warm-up)."""
        self.t0 = time.time()

    def stop(self):
        if self.nvml is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [getattr(self, "error", "NVML unavailable")]}
        self.stop_flag.set()
        self.thread.join(timeout=2)
        timed = [x for x in self.samples if x[0] >= self.t0]
        window = "timed region"
        if len(timed) < 2:  # fewer than two polls fell inside: include the warm-up ones
            timed, window = self.samples, "warm-up + timed region"
        reasons = sorted({nm for _, _, rs in timed for nm, bit in self.REASONS if rs & bit})
        sm = [x[1] for x in timed]
        try:
            self.nvml.nvmlShutdown()
        except Exception:  # noqa: BLE001
            pass
        low = sorted(sm)[len(sm) // 10] if sm else None
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_mhz_p10": low, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(sm), "window": window, "source": "NVML"}


def gram_flops(m, n, T=5, resets=(2,), mode="gram"):
    """Algorithmic FLOPs of the orthogonaliser's GEMM list for one matrix
    (symmetric outputs counted at half of the dense product)."""
    if mode == "quintic":
        return T * (m * m * n + m ** 3 + 2 * m * m * n)
    f = m * m * n  # first Gram matrix
    q_is_identity = True
    for t in range(T):
        if t > 0 and t in resets:
            f += 2 * m * m * n + m * m * n  # X = Q X, R = X X^T
            q_is_identity = True
        f += m ** 3  # R^2 (symmetric)
        if not q_is_identity:
            f += m ** 3  # Q P (symmetric: Q and P are polynomials in one Gram matrix)
        q_is_identity = False
        if t < T - 1 and (t + 1) not in resets:
            f += 2 * m ** 3  # P R and (P R) P (both symmetric)
    return f + 2 * m * m * n  # out = Q X


def step_flops(model, muon, mode, min_m=1):
    """Orthogonaliser FLOPs of one step over this rank's matrices with min(r, c) >= min_m."""
    tot = 0
    for g in muon.param_groups:
        for p in g["params"]:
            if muon._owned is not None and id(p) not in muon._owned:
                continue
            r, c = p.shape
            if min(r, c) >= min_m:
                tot += gram_flops(min(r, c), max(r, c), mode=mode)
    return tot


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        backend = "nccl" if args.device == "cuda" else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
        else:
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    elif args.device == "cuda":
        torch.cuda.set_device(local)
    return world, rank, local


def max_over_ranks(x, world, device):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ------------------------------------------------------------- CPU legs ---
def sample_config(cfg):
    """One layer of cfg with 1/L of every vocabulary table: 1/L of a full step."""
    from dataclasses import replace
    return replace(cfg, name=cfg.name + "_sample", n_layers=1, vocab=cfg.vocab // cfg.n_layers)


def run_oracle_steps(cfg, device, steps, warmup, threads=None):
    from oracle import ref_step  # the checker / reference arm only
    if threads:
        torch.set_num_threads(threads)
    model = synth.SyntheticLM(cfg, device=device, seed=0)
    grads = synth.make_grads(model, 0, seed=0)
    synth.set_grads(model, grads)
    step = ref_step.RefStep(model, **RECIPE)
    times = []
    for it in range(warmup + steps):
        mom = 0.85 + 0.10 * min(1.0, it / MOM_WARMUP)
        step.muon.group["momentum"] = mom
        if device == "cuda":
            torch.cuda.synchronize()
        t0 = time.perf_counter()
        step.step()
        if device == "cuda":
            torch.cuda.synchronize()
        if it >= warmup:
            times.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(times), times


def cpu_baseline(cfg, steps=2, warmup=1):
    scfg = sample_config(cfg)
    threads = os.cpu_count() or 1
    ms, _ = run_oracle_steps(scfg, "cpu", steps, warmup, threads)
    return {"value": ms * cfg.n_layers, "unit": "ms", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"one layer of {cfg.name} (5 NorMuon matrices) + 1/{cfg.n_layers} of every vocabulary "
                      f"table, median of {steps} steps after {warmup} warm-up, scaled x{cfg.n_layers}"}


def reference_arm(args, world, rank):
    cfg = synth.CONFIGS[args.config]
    if rank != 0:
        return None
    if args.device == "cuda":
        ms, _ = run_oracle_steps(cfg, "cuda", min(args.steps, 10), max(1, min(args.warmup, 3)))
        line = {"metric": "optimizer step ms (NorMuon+AdamW+EMA)", "value": ms, "unit": "ms", "impl": "reference",
                "device": "cuda", "n_gpus": 1, "steps": min(args.steps, 10), "higher_is_better": False,
                "dtype": "bf16", "data": "synthetic",
                "config": {"workload": cfg.name, "orthogonalizer": "quintic fallback (torch bf16 matmul)"},
                "note": "reference optimizer math (bit-exact CPU oracle) executed with torch on the GPU"}
        line["e2e"] = {"value": ms, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
        return line
    steps, warm = min(args.steps, 3), min(args.warmup, 1)
    scfg = sample_config(cfg)
    ms, _ = run_oracle_steps(scfg, "cpu", steps, warm, os.cpu_count() or 1)
    value = ms * cfg.n_layers
    cb = {"value": value, "unit": "ms", "cores": torch.get_num_threads(), "kind": "port",
          "sample": f"one layer of {cfg.name} + 1/{cfg.n_layers} of every vocabulary table, median of {steps} "
                    f"steps after {warm} warm-up, scaled x{cfg.n_layers}"}
    return {"metric": "optimizer step ms (NorMuon+AdamW+EMA)", "value": value, "unit": "ms", "impl": "reference",
            "n_gpus": args.gpus, "steps": steps, "warmup": warm, "ms_per_step": value, "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": cfg.name, "orthogonalizer": "quintic fallback (reference, GNS absent)"},
            "cpu_baseline": cb, "e2e": {"value": value, "unit": "ms", "h2d_bytes_per_step": 0,
                                        "d2h_bytes_per_step": 0}}


# ------------------------------------------------------------ engine arm ---
def engine_arm(args, world, rank, local):
    cfg = synth.CONFIGS[args.config]
    dev = torch.device("cuda", local)
    _lib.load()
    model = synth.SyntheticLM(cfg, device=dev, seed=0)
    named = list(model.named_parameters())
    # gradients live in one flat buffer so the end-to-end leg copies them in with
    # one H2D copy; each view starts on a 256-byte boundary, as separately
    # allocated gradients do
    total = sum(p.numel() for _, p in named)
    pad = lambda n: (n + 127) // 128 * 128  # noqa: E731
    flat_grad = torch.empty(sum(pad(p.numel()) for _, p in named), dtype=cfg.dtype, device=dev)
    grads = synth.make_grads(model, 0, seed=0)
    off = 0
    grad_offsets = []
    for (_, p), g in zip(named, grads):
        n = p.numel()
        view = flat_grad[off:off + n].view_as(p)
        view.copy_(g)
        p.grad = view
        grad_offsets.append(off)
        off += pad(n)
    del grads
    muon, adamw = build_optimizers(model, orthogonalizer=args.orthogonalizer, coefficients=args.coefficients,
                                   adam_master="bf16_mt", **RECIPE)
    ema = EmaWeights(model, 0.999)
    sharded = ShardedStep(model, muon, adamw, ema, world=world, rank=rank, exchange=args.exchange,
                          push_streams=args.push_streams, waves=args.waves, assignment=args.assignment,
                          adamw_between_waves=args.adamw_between_waves) if world > 1 else None
    stream = torch.cuda.current_stream(dev)
    ortho_events = []
    adam_ev = []
    shard_marks = []

    def one_step(it, record=False, before=None):
        """One optimizer step; before(name), when given, runs right before the
        NorMuon ("normuon") and AdamW ("adamw") steps (the e2e leg waits there
        for the gradients each of them reads)."""
        before = before or (lambda name: None)
        mom = 0.85 + 0.10 * min(1.0, it / MOM_WARMUP)
        for g in muon.param_groups:
            g["momentum"] = mom
        if sharded is not None:
            # AdamW, table gathers overlapped with NorMuon, EMA, arena gather
            if record:
                marks = [("start", torch.cuda.Event(enable_timing=True))]
                marks[0][1].record(stream)

                def mark(name):
                    ev = torch.cuda.Event(enable_timing=True)
                    ev.record(stream)
                    marks.append((name, ev))
                sharded.step(mark, before=before)
                shard_marks.append(marks)
            else:
                sharded.step(before=before)
            return
        before("normuon")
        muon.step()
        if record:
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        before("adamw")
        adamw.step()
        if record:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record(stream)
            adam_ev.append((e0, e1))
        ema.update()

    sampler = ClockSampler(local)
    sampler.start()  # samples from the warm-up on, so short timed regions still get clock readings
    for it in range(args.warmup):
        one_step(it)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    sampler.mark()
    launches0 = _lib.launch_count()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    host_t = 0.0
    for k in range(args.steps):
        h0 = time.perf_counter()
        one_step(args.warmup + k)
        host_t += time.perf_counter() - h0
    end.record(stream)
    torch.cuda.synchronize()
    launches = _lib.launch_count() - launches0
    clocks = sampler.stop()
    # Phase timing: a second timed run of the same steps with CUDA events on
    # the launching stream around each orthogonaliser call and the AdamW pass.
    # The events sit between library calls, not between the GEMM launches of
    # one call, so the GEMM chain keeps its programmatic dependent launches.
    # The dominant kernel's figure is the tensor-core GEMM chain: the calls of
    # the m > 32 classes, whose launches are all tcgen05 GEMMs in the default
    # Gram mode (the m <= 32 gates run in one CUDA-core kernel of their own).
    torch.cuda.synchronize()
    gsampler = ClockSampler(local)  # clocks of this second run, where the GEMM figure comes from
    gsampler.start()
    gsampler.mark()
    muon._timing_events = ortho_events
    for k in range(args.steps):
        one_step(args.warmup + args.steps + k, record=True)
    torch.cuda.synchronize()
    muon._timing_events = None
    gclocks = gsampler.stop()
    err = _lib.device_error()
    if err:
        raise RuntimeError(f"device error word {err}")
    ms_local = start.elapsed_time(end) / args.steps
    ms = max_over_ranks(ms_local, world, dev)
    ortho_ms = sum(a.elapsed_time(b) for a, b, _, _ in ortho_events) / args.steps
    gemm_ms = sum(a.elapsed_time(b) for a, b, m, _ in ortho_events if m > 32) / args.steps
    per_step = [a.elapsed_time(b) for a, b, m, _ in ortho_events if m > 32]
    per_class = max(1, len(per_step) // max(1, args.steps))
    per_step = [sum(per_step[i:i + per_class]) for i in range(0, len(per_step), per_class)]
    gemm_n = sum(n for _, _, m, n in ortho_events if m > 32) / args.steps
    adam_ms = sum(a.elapsed_time(b) for a, b in adam_ev) / args.steps
    shard_phases = {}
    for marks in shard_marks:
        for (_, a), (name, b) in zip(marks, marks[1:]):
            shard_phases[name] = shard_phases.get(name, 0.0) + a.elapsed_time(b) / args.steps
    if shard_phases:
        adam_ms = shard_phases["adamw"]
    mode = "quintic" if args.orthogonalizer == "quintic" else "gram"
    flops = step_flops(model, muon, mode)
    gemm_flops = step_flops(model, muon, mode, min_m=33)
    peak_burst, peak_sus, peak_gbs, peak_kind = peaks()
    # dominant kernel: the tensor-core GEMM chain, algorithmic FLOPs (symmetric
    # outputs at half) over its device time in the step. Denominator: the burst
    # bf16 peak when the SM clock held its maximum through the timed region,
    # the sustained (power-capped) one when the clock samples show it lowered.
    # the peak follows the clocks of the run the GEMM figure comes from: the
    # burst figure when neither its clock median nor its power-cap flags show
    # the GPU below its maximum clock, else the sustained (power-capped) one
    sm, smax = gclocks.get("sm_mhz"), gclocks.get("sm_max_mhz")
    capped = "sw_power_cap" in (gclocks.get("reasons") or [])
    at_max = bool(sm and smax and sm >= 0.97 * smax) and not capped
    peak_tf = peak_burst if at_max or not sm else peak_sus
    peak_label = (f"{peak_kind} bf16 burst (SM clock median {sm} of max {smax} MHz in the GEMM-timing run, no "
                  "power cap seen)" if peak_tf == peak_burst else
                  f"{peak_kind} bf16 sustained (SM clock median {sm} of max {smax} MHz in the GEMM-timing run, "
                  f"power cap {'seen' if capped else 'not seen'})")
    achieved = gemm_flops / (gemm_ms * 1e-3) / 1e12 if gemm_ms > 0 else None
    # AdamW+EMA streaming bytes: p 2+2, rem 2+2, g 2, m 4+4, v 4+4, fp32 EMA 4+4 = 34 B/elem
    adam_elems = sum(p.numel() for g in adamw.param_groups for p in g["params"])
    adam_bytes = adam_elems * 34 / (world if sharded else 1)

    e2e = None
    if not args.no_e2e:
        e2e = e2e_leg(args, model, muon, adamw, ema, sharded, flat_grad, one_step, world, dev, grad_offsets)
    line = {
        "metric": "optimizer step ms (NorMuon+AdamW+EMA)", "value": ms, "unit": "ms", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": cfg.name, "params": total, "muon_matrices": sum(len(g["params"]) for g in
                                                                            muon.param_groups),
                   "orthogonalizer": f"{args.orthogonalizer}/{args.coefficients if mode == 'gram' else 'quintic'}",
                   "adamw": "bf16 + bf16 remainder, fp32 moments", "ema": "fp32, folded",
                   "l2": "working set > L2 (126 MB); no flush",
                   "parallelism": f"shard{world}" if world > 1 else "single",
                   "exchange": sharded.exchange if sharded is not None else None,
                   "push_streams": sharded.push_streams if sharded is not None else None,
                   "waves": sharded.waves if sharded is not None else None,
                   "adamw_between_waves": sharded.adamw_between_waves if sharded is not None else None,
                   "assignment": sharded.assignment if sharded is not None else None},
        "phases_ms": {"orthogonalize": ortho_ms, "adamw": adam_ms,
                      "normuon_other+ema+gather": ms_local - ortho_ms - adam_ms},
        "sharded_phases_ms": shard_phases or None,
        "adamw_gbs": adam_bytes / (adam_ms * 1e-3) / 1e9 if adam_ms > 0 else None,
        "roofline": {"bound": "tensor", "kernel": "gemm_tc_kernel (every tensor-core GEMM of the step)",
                     "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                     "frac": (achieved / peak_tf) if achieved else None,
                     "traffic": GEMM_TRAFFIC_BYTES_PER_LAUNCH if (args.config == "c2_L14_d1024" and world == 1)
                     else None,
                     "traffic_source": "ncu one-pass capture of this configuration's GEMM launches (DRAM read + "
                                       "write per launch), not measured by this run",
                     "launches_per_step": gemm_n, "gemm_ms_per_step": gemm_ms, "flops_per_step": gemm_flops,
                     "flops_per_launch": gemm_flops / max(1, gemm_n),
                     "timing": "CUDA events on the launching stream around the orthogonaliser calls of the "
                               "tensor-core classes (30 GEMM launches each, nothing else; replayed from a "
                               "launch graph), second timed run",
                     "peak_kind": peak_label,
                     "frac_of_burst_peak": (achieved / peak_burst) if achieved else None,
                     "frac_of_sustained_peak": (achieved / peak_sus) if achieved else None,
                     "gemm_ms_first_last_min": [per_step[0], per_step[-1], min(per_step)] if per_step else None,
                     "clocks": gclocks},
        "orthogonalizer": {"ms_per_step": ortho_ms, "flops_per_step": flops,
                           "tflops": flops / (ortho_ms * 1e-3) / 1e12 if ortho_ms > 0 else None},
        "host_enqueue_ms_per_step": host_t * 1e3 / args.steps,
        "clocks": clocks, "gpu_launches": launches,
        "launch_graphs": _lib.launch_graph_stats(),
    }
    if e2e:
        line["e2e"] = e2e
    if sharded is not None:
        sharded.close()
    return line


def single_gpu_extras(args, cfg, dev):
    """Measurements printed beside the N = 1 headline, each outside the engine's
    timed regions: BASELINE configs[2] (Gram-NS TFLOP/s per shape) and
    configs[3] (AdamW+EMA GB/s) through the engine, and the reference's own
    optimizer step executed by torch on the same GPU (its quintic fallback:
    the gram-newton-schulz package it would import is absent, so its GNS path
    cannot run; the step is the reference's math, bit-exact with it on the CPU)."""
    out = {}
    if not args.no_micro:
        ns = argparse.Namespace(shape="1024x1024,3072x1024,5632x1024,1024x5632", steps=10, warmup=3,
                                orthogonalizer=args.orthogonalizer, coefficients=args.coefficients, tables=7)
        g = micro_gram(ns, dev)
        out["gram_ns_micro"] = {"per_shape": g["per_shape"], "peak": g["peak"], "peak_kind": g["peak_kind"]}
        torch.cuda.empty_cache()
        a = micro_adamw(ns, dev)
        out["adamw_micro"] = {"gbs": a["value"], "ms": a["ms_per_step"], "frac": a["roofline"]["frac"],
                              "elements": a["config"]["elements"], "bytes_per_element": 34}
        torch.cuda.empty_cache()
    if not args.no_reference_gpu:
        steps, warm = 5, 2
        ms, _ = run_oracle_steps(cfg, "cuda", steps, warm)
        out["reference_gpu"] = {"ms": ms, "steps": steps, "warmup": warm, "gns_installed": False,
                                "orthogonalizer": "quintic fallback (zeropower_via_newtonschulz5, torch bf16 "
                                                  "matmul on cuBLAS)",
                                "timing": "median of host-synchronised steps, after the engine's timed regions"}
        torch.cuda.empty_cache()
    return out


def sharded_parity(args, cfg, world, rank, dev, steps=3):
    """Bit-identity of the sharded step with the single-GPU engine, checked on
    every rank after the timed regions: a fresh sharded engine and a fresh
    unsharded one on the same seeded parameters and gradients take the same
    steps; every parameter and (after gather_ema) every EMA shadow must be
    equal bit for bit on every rank. Every rank takes the same collectives."""
    import torch.distributed as dist
    kw = dict(orthogonalizer=args.orthogonalizer, coefficients=args.coefficients, adam_master="bf16_mt", **RECIPE)
    model = synth.SyntheticLM(cfg, device=dev, seed=0)
    muon, adamw = build_optimizers(model, **kw)
    ema = EmaWeights(model, 0.999)
    sh = ShardedStep(model, muon, adamw, ema, world=world, rank=rank, exchange=args.exchange,
                     push_streams=args.push_streams, waves=args.waves, assignment=args.assignment,
                     adamw_between_waves=args.adamw_between_waves)
    ref = synth.SyntheticLM(cfg, device=dev, seed=0)
    rmuon, radamw = build_optimizers(ref, **kw)
    rema = EmaWeights(ref, 0.999)
    try:
        for it in range(steps):
            mom = 0.85 + 0.10 * min(1.0, it / MOM_WARMUP)
            for opt in (muon, rmuon):
                for g in opt.param_groups:
                    g["momentum"] = mom
            grads = synth.make_grads(model, it, seed=0)
            synth.set_grads(model, [g.clone() for g in grads])
            synth.set_grads(ref, grads)
            del grads
            sh.step()
            rmuon.step()
            radamw.step()
            rema.update()
        torch.cuda.synchronize()
        named, rnamed = list(model.named_parameters()), list(ref.named_parameters())
        bad_p = sum(0 if torch.equal(p.data, r.data) else 1 for (_, p), (_, r) in zip(named, rnamed))
        sh.gather_ema()
        torch.cuda.synchronize()
        bad_e = sum(0 if torch.equal(a, b) else 1 for a, b in zip(ema.shadow, rema.shadow))
        err = _lib.device_error()
    finally:
        sh.close()
    t = torch.tensor([bad_p, bad_e, 1 if err else 0], dtype=torch.int64, device=dev)
    dist.all_reduce(t)
    bad_p, bad_e, errs = (int(x) for x in t.tolist())
    return {"equal": bad_p == 0 and bad_e == 0 and errs == 0, "mismatched_params": bad_p,
            "mismatched_ema": bad_e, "ranks_with_device_error": errs, "steps": steps,
            "checked": f"{len(named)} parameters and EMA shadows on each of {world} ranks, bitwise, against "
                       "the unsharded engine on the same GPU"}


def e2e_leg(args, model, muon, adamw, ema, sharded, flat_grad, one_step, world, dev, grad_offsets):
    """Same step through the public API, with the step's gradients copied in
    from pinned host memory and a result read back every step. A sharded rank
    copies in only the gradients its optimizer shard reads (its NorMuon
    matrices, its rows of the split tables and the small replicated tensors),
    as a rank does after a gradient reduce-scatter. The copies overlap the
    step: the optimizer that runs first waits only for its own gradients."""
    host = torch.empty(flat_grad.numel(), dtype=flat_grad.dtype, pin_memory=True)
    host.copy_(flat_grad.cpu())
    # gradient ranges each optimizer reads, copied in the order the step
    # consumes them (NorMuon first on one GPU, AdamW first in the sharded step)
    muon_ids = {id(p) for g in muon.param_groups for p in g["params"]}
    ranges = {"normuon": [], "adamw": []}
    for (_, p), off in zip(model.named_parameters(), grad_offsets):
        n = p.numel()
        which = "normuon" if id(p) in muon_ids else "adamw"
        if sharded is None:
            ranges[which].append((off, n))
        elif id(p) in sharded.owner:
            if sharded.owner[id(p)] == sharded.rank:
                ranges[which].append((off, n))
        else:
            start, cnt = adamw._owned_slices.get(id(p), (0, n))
            ranges[which].append((off + start, cnt))

    def merge(rs):
        merged = []
        for off, n in sorted(rs):
            if merged and merged[-1][0] + merged[-1][1] >= off:
                o0, n0 = merged[-1]
                merged[-1] = (o0, max(n0, off + n - o0))
            else:
                merged.append((off, n))
        return merged

    ranges = {k: merge(v) for k, v in ranges.items()}
    if sharded is not None:
        order = [sharded.first_optimizer, "normuon" if sharded.first_optimizer == "adamw" else "adamw"]
    else:
        order = ["normuon", "adamw"]
    h2d = sum(n for v in ranges.values() for _, n in v) * host.element_size()
    probe = next(iter(muon.param_groups[0]["params"]))
    out = torch.empty(256, dtype=probe.dtype, pin_memory=True)
    stream = torch.cuda.current_stream(dev)
    copy_stream = torch.cuda.Stream(dev)

    def step_with_copies(k):
        # the copies of this step start once the previous step is done with
        # the gradient buffer; each optimizer waits only for its own gradients
        copy_stream.wait_stream(stream)
        ready = {}
        with torch.cuda.stream(copy_stream):
            for which in order:
                for off, n in ranges[which]:
                    flat_grad[off:off + n].copy_(host[off:off + n], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy_stream)
                ready[which] = ev
        one_step(k, before=lambda name: stream.wait_event(ready[name]))
        out.copy_(probe.detach().reshape(-1)[:256], non_blocking=True)

    for it in range(2):
        step_with_copies(it)
    torch.cuda.synchronize()
    barrier(world)
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for k in range(args.steps):
        step_with_copies(k)
    e.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(s.elapsed_time(e) / args.steps, world, dev)
    return {"value": ms, "unit": "ms", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": out.numel() * out.element_size(),
            "overlap": "gradients copied on a side stream in the order the step reads them; each optimizer "
                       "waits for its own"}


def micro_gram(args, dev):
    """batched orthogonalisation, 14 matrices per shape,
    5 iterations, N(0,1) inputs scaled to unit spectral norm."""
    from sol_b200 import NorMuonGNS
    shapes = [tuple(int(x) for x in s.split("x")) for s in args.shape.split(",")]
    peak_tf, _, _, peak_kind = peaks()  # kernels timed alone: burst peak
    S = int(getattr(args, "batch", 14))
    out = []
    for (r, c) in shapes:
        g = torch.Generator(device=dev).manual_seed(0)
        U = torch.randn(S, r, c, generator=g, device=dev)
        U = U / torch.linalg.matrix_norm(U, ord=2, keepdim=True)
        U = U.to(torch.bfloat16)
        opt = NorMuonGNS([torch.nn.Parameter(torch.zeros(r, c, device=dev))], orthogonalizer=args.orthogonalizer,
                         coefficients=args.coefficients)
        o = torch.empty_like(U)
        ws = opt._workspace(dev, S, r, c)
        part = ws["partial"].view(S, -1)
        part.zero_()
        part[:, 0] = U.float().pow(2).sum(dim=(1, 2))
        for _ in range(args.warmup):
            opt._ortho(U, ws["partial"], S, r, c, 5, o, ws)
        torch.cuda.synchronize()
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(args.steps):
            opt._ortho(U, ws["partial"], S, r, c, 5, o, ws)
        s1.record()
        torch.cuda.synchronize()
        ms = s0.elapsed_time(s1) / args.steps
        mode = "quintic" if args.orthogonalizer == "quintic" else "gram"
        fl = S * gram_flops(min(r, c), max(r, c), mode=mode)
        tf = fl / (ms * 1e-3) / 1e12
        out.append({"shape": f"{S}x{r}x{c}", "ms": ms, "tflops": tf, "frac": tf / peak_tf})
    return {"metric": "Gram-NS TFLOP/s", "value": statistics.mean(x["tflops"] for x in out), "unit": "TFLOP/s",
            "higher_is_better": True, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "dtype": "bf16/f16",
            "data": "synthetic", "config": {"workload": "configs[2] Gram-NS microbenchmark",
                                             "orthogonalizer": args.orthogonalizer, "coefficients": args.coefficients},
            "per_shape": out, "peak": peak_tf, "peak_kind": f"{peak_kind} bf16 burst"}


def micro_adamw(args, dev):
    """streaming AdamW+EMA over 7 x 32768 x 1024 + 1M scalars,
    bf16 params + bf16 remainder, fp32 moments, fp32 EMA, cautious decay 0.1, step 100."""
    from sol_b200 import AdamW, EmaWeights
    g = torch.Generator(device=dev).manual_seed(0)
    params = [torch.nn.Parameter((torch.randn(32768, 1024, generator=g, device=dev) * 0.02).to(torch.bfloat16))
              for _ in range(args.tables)]
    params.append(torch.nn.Parameter(torch.ones(1 << 20, device=dev, dtype=torch.bfloat16)))
    for p in params:
        p.grad = (torch.randn(p.shape, generator=g, device=dev) * 1e-4).to(torch.bfloat16)
    opt = AdamW(params, lr=2.4e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, master="bf16_mt",
                cautious_wd=True)
    holder = torch.nn.Module()
    for i, p in enumerate(params):
        holder.register_parameter(f"t{i}", p)
    ema = EmaWeights(holder, 0.999)
    for p in params:
        opt._init_state(p)
        opt._steps[id(p)] = 99
    ema.update()  # arms folding
    for _ in range(args.warmup):
        opt.step()
        ema.update()
    torch.cuda.synchronize()
    s0 = torch.cuda.Event(enable_timing=True)
    s1 = torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(args.steps):
        opt.step()
        ema.update()
    s1.record()
    torch.cuda.synchronize()
    ms = s0.elapsed_time(s1) / args.steps
    n = sum(p.numel() for p in params)
    gbs = n * 34 / (ms * 1e-3) / 1e9
    _, _, peak_gbs, peak_kind = peaks()
    return {"metric": "AdamW+EMA GB/s", "value": gbs, "unit": "GB/s", "higher_is_better": True, "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "dtype": "bf16+fp32", "data": "synthetic",
            "config": {"workload": "configs[3] streaming AdamW+EMA", "elements": n,
                       "bytes_per_element": 34, "ema": "fp32 (bf16 shadow underflows at decay 0.999)"},
            "ms_per_step": ms,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak_gbs, "unit": "GB/s", "frac": gbs / peak_gbs,
                         "traffic": None, "peak_kind": f"{peak_kind} copy"}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["engine", "reference"], default="engine")
    ap.add_argument("--device", choices=["cuda", "cpu"], default=None,
                    help="engine: cuda; reference arm: cpu (host cores) unless cuda is given")
    ap.add_argument("--config", default="c2_L14_d1024", choices=sorted(synth.CONFIGS))
    ap.add_argument("--orthogonalizer", default="gram", choices=["gram", "quintic"])
    ap.add_argument("--coefficients", default="polar_express", choices=["polar_express", "quintic"])
    ap.add_argument("--exchange", default="auto", choices=["auto", "ce", "hybrid", "nccl"],
                    help="N>1: copy-engine pushes over CUDA IPC mappings, NCCL all-gathers, or both")
    ap.add_argument("--push-streams", type=int, default=1, help="N>1: streams the copy-engine pushes use")
    ap.add_argument("--waves", type=int, default=None,
                    help="N>1: NorMuon waves per rank (exchange overlaps compute); default 2 from 4 GPUs with at least 16 matrices per rank, else 1")
    ap.add_argument("--assignment", default="lpt", choices=["lpt", "runs"], help="N>1: matrix-to-rank assignment")
    ap.add_argument("--adamw-between-waves", action="store_true",
                    help="N>1 with two or more waves: AdamW after the first NorMuon wave")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-micro", action="store_true", help="N=1: skip the configs[2]/[3] micro-benchmarks")
    ap.add_argument("--no-reference-gpu", action="store_true", help="N=1: skip the reference step on the GPU")
    ap.add_argument("--no-parity", action="store_true", help="N>1: skip the bit-identity check")
    ap.add_argument("--micro", choices=["gram", "adamw"], default=None,
                    help="run a BASELINE micro-benchmark (configs[2] / configs[3]) instead of the full step")
    ap.add_argument("--shape", default="1024x1024,3072x1024,5632x1024,1024x5632")
    ap.add_argument("--tables", type=int, default=7, help="--micro adamw: number of 32768x1024 tables")
    ap.add_argument("--batch", type=int, default=14, help="--micro gram: matrices per shape")
    args = ap.parse_args()
    if args.device is None:
        args.device = "cuda" if args.impl == "engine" else "cpu"
    if args.warmup < 3 and args.impl == "engine":
        args.warmup = 3
    if args.impl == "reference" and args.device == "cpu":
        world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
        if rank == 0:
            print(json.dumps(reference_arm(args, world, rank)), flush=True)
        return
    world, rank, local = dist_setup(args)
    if args.micro:
        dev = torch.device("cuda", local)
        _lib.load()
        line = micro_gram(args, dev) if args.micro == "gram" else micro_adamw(args, dev)
        if rank == 0:
            print(json.dumps(line), flush=True)
        return
    try:
        if args.impl == "reference":
            line = reference_arm(args, world, rank)
        else:
            line = engine_arm(args, world, rank, local)
            cfg = synth.CONFIGS[args.config]
            dev = torch.device("cuda", local)
            torch.cuda.empty_cache()
            if world > 1 and not args.no_parity:
                line["parity_vs_single_gpu"] = sharded_parity(args, cfg, world, rank, dev)
            if world == 1:
                line.update(single_gpu_extras(args, cfg, dev))
                if not args.no_cpu_baseline:
                    line["cpu_baseline"] = cpu_baseline(cfg)
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

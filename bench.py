#!/usr/bin/env python3
"""bench.py -- MoE-layer tokens/s of the Mixtral-8x7B-shaped NF4 MoE block on B200.

Workload (the isolated-block configuration): hidden 4096, 8 experts, top-2,
SwiGLU intermediate 14336, weights N(0, 0.02) seed 2 quantized to NF4 with
riallm's block format (0.625 B/weight, 880.8 MB for the layer), bf16
activations N(0, 1). One step = one MoE block forward over one batch of
tokens (default: a decode batch of 64). The weights are larger than the
126 MB L2, so every step streams them from HBM.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints ONE JSON line on rank 0. Multi-GPU (torchrun, one rank per GPU):
expert parallel -- rank r keeps experts [r E/N, (r+1) E/N), every step
routes its own batch, sends each token row to the ranks that own its
experts and gets the expert outputs back (a token all-to-all inside the
library over NCCL point-to-point), then sums them per token (weak scaling:
64 tokens per GPU); value
is the total tokens of all ranks over the slowest rank's device time.
The single-GPU line also carries a Mixtral-8x7B decode measurement (32
layers, batch 1 and 32; --decode-only runs it alone), a token-count sweep,
the fine-grained block (128 experts, top-8) and layer streaming from pinned
host memory for the Mixtral-8x7B block and a Mixtral-8x22B-shaped one.

--impl reference times the oracle's CPU port of riallm's MoE block
(oracle/riallm_oracle.c, all host threads) on the same workload; the Rust
reference itself cannot be built here.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, I, E, TOP_K = 4096, 14336, 8, 2
NF4_BYTES_PER_WEIGHT = 0.5 + 8.0 / 64.0          # codes + f32 scale and zero per 64
WEIGHTS_PER_EXPERT = 3 * H * I                    # gate, up, down
BYTES_PER_EXPERT = int(WEIGHTS_PER_EXPERT * NF4_BYTES_PER_WEIGHT)  # 110,100,480
METRIC = "MoE-layer tokens/s & Mixtral-8x7B NF4 decode tok/s at 1/2/4/8 B200; % HBM peak"
SWEEP_T = (1, 8, 32, 64, 4096)


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), float(p["bf16_tflops_sustained"]), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


# ------------------------------------------------------------------ clocks

_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
            0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
            0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
            0x100: "display_clock_setting"}


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML in a thread."""

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._period = period_s
        self._dev = device_index
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            except Exception:
                pass
            time.sleep(self._period)

    def __enter__(self):
        if self._nv:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self):
        if not self._nv or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"], "samples": 0}
        reasons = [name for bit, name in _REASONS.items() if self.reasons & bit and bit != 0x1]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples)}


# ------------------------------------------------------------ distributed

def dist_setup():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# ----------------------------------------------------------- reference arm

def run_reference(args, rank, world):
    """Times the CPU port of riallm's MoE block (the oracle) on host cores."""
    if rank != 0:
        return 0
    import numpy as np
    from oracle import oracle as O

    O.build()
    t0 = time.time()
    rng = np.random.default_rng(2)
    layer = {}
    for name, shape in (("gate", (E, H)), ("gate_up_proj", (E, 2 * I, H)), ("down_proj", (E, H, I))):
        a = rng.standard_normal(size=shape, dtype=np.float32)
        a *= np.float32(0.02)
        layer[name] = O.quantize(a, O.FOUR_BIT)
        del a
    w = O.MoeWeights(layer["gate"], layer["gate_up_proj"], layer["down_proj"])
    x = O.synthetic_x(args.tokens, H, seed=3, bf16=True)
    setup_s = time.time() - t0
    threads = os.cpu_count() or 1

    # Size each step's sample so the whole run stays within a few minutes.
    t1 = time.perf_counter()
    O.moe_forward(w, x[:1], 1, H, I, E, TOP_K, n_threads=threads)
    one_token_s = time.perf_counter() - t1
    max_run_s = 150.0
    n_calls = args.warmup + args.steps
    sample_tokens = args.tokens
    est = n_calls * one_token_s * sample_tokens * 0.6  # tokens share dequantized rows
    if est > max_run_s:
        sample_tokens = max(1, int(args.tokens * max_run_s / est))
    xs = x[:sample_tokens]
    for _ in range(args.warmup):
        O.moe_forward(w, xs, sample_tokens, H, I, E, TOP_K, n_threads=threads)
    t2 = time.perf_counter()
    for _ in range(args.steps):
        O.moe_forward(w, xs, sample_tokens, H, I, E, TOP_K, n_threads=threads)
    el = time.perf_counter() - t2
    value = sample_tokens * args.steps / el
    sample = (f"{sample_tokens} of the {args.tokens}-token decode batch per step, full 8-expert "
              f"NF4 Mixtral block, fp32 oracle port, {threads} threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * el / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: N(0,0.02) weights (numpy seed 2) NF4-quantized; N(0,1) bf16 activations",
        "config": config_dict(args, world),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "setup_s": round(setup_s, 1),
    }
    print(json.dumps(line), flush=True)
    return 0


def config_dict(args, world):
    return {"workload": f"mixtral8x7b_moe_block_nf4_decode_T{args.tokens}",
            "hidden": H, "intermediate": I, "experts": E, "top_k": TOP_K,
            "tokens_per_step_per_gpu": args.tokens, "compression": "FourBit (riallm NF4 layout)",
            "parallelism": (f"ep{world} (expert-parallel: {E // max(world, 1)} experts per GPU; "
                            + {"replicated": "tokens all-gathered, partials reduce-scattered over NCCL)",
                               "all_to_all": "token all-to-all over NCCL inside the library)",
                               "all_to_all_peer": "token all-to-all by the library's stores into peer memory)"}[
                                   args.ep_path]) if world > 1 else "single",
            "l2_policy": "inputs larger than L2 (880.8 MB of NF4 weights per step vs 126 MB L2)"}


# ------------------------------------------------------------------ ours

def make_layer(rb, torch, device, seed=2, hidden=H, inter=I, experts=E):
    """Seeded N(0, 0.02) weights quantized to NF4 in riallm's layout (the
    Mixtral-8x7B block by default). Each tensor is generated and quantized
    one expert slice at a time into the full tensor's buffers (64-element
    blocks never straddle experts, so the bytes, scales and zero points equal
    those of quantizing the whole tensor at once); this keeps the device
    footprint near the NF4 data (0.9 GB for Mixtral-8x7B)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    L = rb.lib()
    ctx = rb.Context.get(device.index or 0)
    d = {}
    for name, shape in (("mlp.gate.weight", (experts, hidden)),
                        ("mlp.experts.gate_up_proj", (experts, 2 * inter, hidden)),
                        ("mlp.experts.down_proj", (experts, hidden, inter))):
        numel = 1
        for v in shape:
            numel *= v
        data = torch.empty(numel // 2, dtype=torch.uint8, device=device)
        scales = torch.empty(numel // 64, dtype=torch.float32, device=device)
        zeros = torch.empty(numel // 64, dtype=torch.float32, device=device)
        chunk = numel // shape[0] if len(shape) == 3 else numel
        for c0 in range(0, numel, chunk):
            w = torch.empty(chunk, device=device).normal_(0.0, 0.02, generator=gen)
            ctx.check(L.riallm_cuda_quantize(ctx.ptr, 1, w.data_ptr(), chunk, data.data_ptr() + c0 // 2,
                                             scales.data_ptr() + 4 * (c0 // 64), zeros.data_ptr() + 4 * (c0 // 64),
                                             torch.cuda.current_stream().cuda_stream))
            del w
        d[name] = rb.QuantizedTensor(data, shape, rb.CompressionType.FourBit, scales, zeros, 64)
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return d


class Block:
    """One MoE block call through the C ABI with fixed buffers (so it can be
    captured in a CUDA graph)."""

    def __init__(self, rb, torch, d, T, device):
        self.rb, self.torch = rb, torch
        self.ctx = rb.Context.get(device.index or 0)
        self.w, self.keep, _ = rb._weights(d)
        gen = torch.Generator(device=device).manual_seed(1000 + T)
        self.x = torch.empty(T, H, device=device).normal_(0, 1, generator=gen).to(torch.bfloat16)
        self.out = torch.empty_like(self.x)
        self.T = T
        self.ctx.reserve(T, H, I, E, TOP_K, torch.bfloat16)

    def __call__(self, stream_ptr=None):
        L = self.rb.lib()
        st = stream_ptr if stream_ptr is not None else self.torch.cuda.current_stream().cuda_stream
        rc = L.riallm_cuda_moe_forward(self.ctx.ptr, ctypes.byref(self.w), self.x.data_ptr(),
                                       self.out.data_ptr(), self.T, H, I, E, TOP_K, 1, 0, st)
        if rc:
            self.ctx.check(rc)

    def distinct_experts(self):
        idx, _, counts, _, _ = self.rb.route(self.keep[0], self.x, TOP_K, E)
        return int((counts > 0).sum().item())


def expert_bytes(T, U):
    """Algorithmic bytes of the two expert-GEMM launches of one step."""
    P = T * TOP_K
    return U * BYTES_PER_EXPERT + P * H * 2 + 2 * P * I * 2 + P * H * 4


# DRAM bytes of one step's two expert-GEMM launches (read + written), from
# one ncu capture of the 64-token workload: 625.7 + 10.0 MB (gate_up) and
# 317.9 + 6.4 MB (down), against 891.3 MB algorithmic. ncu flushes the
# caches between kernels, so the down launch's first stages, which gate_up
# prefetches into L2, are counted twice there (~12 MB).
TRAFFIC_T64 = 960.0e6


def expert_flops(T):
    return 2.0 * T * TOP_K * 3 * H * I


def timed(torch, fn, steps, warmup, dist, world):
    for _ in range(warmup):
        fn()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    end.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def phase_profile(torch, blk, steps):
    """Per-phase device time from CUDA events recorded by the library on the
    launching stream. A sleep kernel queued first keeps the GPU busy while the
    host enqueues every step, so no host gap lands inside an event pair."""
    torch.cuda.synchronize()
    blk.ctx.profile(True)
    torch.cuda._sleep(int(2e8))
    for _ in range(steps):
        blk()
    torch.cuda.synchronize()
    blk.ctx.profile(False)
    ph, calls = blk.ctx.profile_read()
    return {k: v / max(calls, 1) for k, v in ph.items()}, calls


def run_ours(args, rank, world, local):
    import torch
    import riallm_b200 as rb

    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    hbm_peak, bf16_peak, bf16_sust, peak_src = load_peaks()

    d = make_layer(rb, torch, device)
    if world > 1:
        return run_ep(args, rank, world, local, rb, torch, dist, d, device, hbm_peak, peak_src)
    blk = Block(rb, torch, d, args.tokens, device)
    U = blk.distinct_experts()

    # Capture one step in a CUDA graph (after a warm-up that sizes the arena).
    for _ in range(3):
        blk()
    torch.cuda.synchronize()
    l0 = blk.ctx.launch_count()
    blk()
    launches_per_step = blk.ctx.launch_count() - l0  # kernels of one step, counted by the library
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            blk(s.cuda_stream)
    torch.cuda.synchronize()

    launches0 = blk.ctx.launch_count()
    with ClockSampler(local) as clk:
        ms = timed(torch, g.replay, args.steps, args.warmup, dist, world)
    per_step_launches = (blk.ctx.launch_count() - launches0)  # graph replays launch nothing through the library
    ms_per_step = ms / args.steps
    value = world * args.tokens * args.steps / (ms / 1000.0)

    # Roofline of the dominant kernel (the tcgen05 expert GEMM: gate_up + down launches).
    ph, _ = phase_profile(torch, blk, max(10, min(args.steps, 50)))
    kern_ms = ph["gate_up"] + ph["down"]
    bytes_step = expert_bytes(args.tokens, U)
    achieved = bytes_step / (kern_ms / 1000.0) / 1e9
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(achieved / hbm_peak, 4),
                "traffic": TRAFFIC_T64 if args.tokens == 64 else None,
                "traffic_source": "dram__bytes_read.sum + dram__bytes_write.sum of the gate_up and down "
                                  "launches, one ncu capture of this 64-token workload" if args.tokens == 64 else None,
                "kernel": "expert_gemm_kernel<NF4> (gate_up + down launches of one step)",
                "algorithmic_bytes_per_step": bytes_step, "distinct_experts": U,
                "kernel_ms_per_step": round(kern_ms, 4),
                "phase_ms_per_step": {k: round(v, 4) for k, v in ph.items()},
                "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured" else peak_src,
                "step_frac": round(U * BYTES_PER_EXPERT / (ms_per_step / 1000.0) / 1e9 / hbm_peak, 4)}

    # End to end through the C ABI with host buffers: every step copies its
    # x from pinned host memory (H2D), runs the block and copies the output
    # back (D2H). The copies run on a second stream, double-buffered, so
    # step i's block overlaps step i+1's H2D and step i-1's D2H; the timed
    # region spans all of them (the copy stream is joined before the end).
    L = rb.lib()
    blks = [blk, Block(rb, torch, d, args.tokens, device)]
    blks[1].x.copy_(blk.x)
    nbytes = blk.x.numel() * 2
    hx = torch.empty_like(blk.x, device="cpu").pin_memory()
    hx.copy_(blk.x.cpu())
    houts = [torch.empty_like(hx).pin_memory() for _ in range(2)]
    comp = torch.cuda.current_stream()
    copy = torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_run(n):
        cs, ks = copy.cuda_stream, comp.cuda_stream
        copy.wait_stream(comp)
        blk.ctx.check(L.riallm_cuda_memcpy_h2d_async(blk.ctx.ptr, blks[0].x.data_ptr(), hx.data_ptr(), nbytes, cs))
        ev_in[0].record(copy)
        for i in range(n):
            b, nb = i % 2, (i + 1) % 2
            if i + 1 < n:
                if i >= 1:
                    copy.wait_event(ev_done[nb])  # step i-1 has read blks[nb].x
                blk.ctx.check(L.riallm_cuda_memcpy_h2d_async(blk.ctx.ptr, blks[nb].x.data_ptr(), hx.data_ptr(),
                                                             nbytes, cs))
                ev_in[nb].record(copy)
            comp.wait_event(ev_in[b])
            if i >= 2:
                comp.wait_event(ev_out[b])  # step i-2's output has been copied out
            blks[b](ks)
            ev_done[b].record(comp)
            copy.wait_event(ev_done[b])
            blk.ctx.check(L.riallm_cuda_memcpy_d2h_async(blk.ctx.ptr, houts[b].data_ptr(), blks[b].out.data_ptr(),
                                                         nbytes, cs))
            ev_out[b].record(copy)
        comp.wait_stream(copy)

    e2e_run(args.warmup)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    e2e_run(args.steps)
    t1.record()
    torch.cuda.synchronize()
    e2e_ms = t0.elapsed_time(t1)
    if not torch.equal(houts[(args.steps - 1) % 2], blks[(args.steps - 1) % 2].out.cpu()):
        raise RuntimeError("end-to-end output differs from the device-resident run")
    e2e = {"value": world * args.tokens * args.steps / (e2e_ms / 1000.0), "unit": "tokens/s",
           "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes,
           "ms_per_step": round(e2e_ms / args.steps, 4),
           "note": "C ABI calls with pinned host buffers; H2D and D2H on a copy stream, double-buffered"}

    # Sweep over the other token counts of the configuration (rank-local).
    sweep = []
    if not args.no_sweep:
        for T in SWEEP_T:
            if T == args.tokens:
                continue
            b2 = Block(rb, torch, d, T, device)
            u2 = b2.distinct_experts()
            for _ in range(2):
                b2()
            steps2 = 5 if T >= 1024 else 20
            ms2 = timed(torch, b2, steps2, 2, dist, world)
            ph2, _ = phase_profile(torch, b2, steps2)
            k2 = ph2["gate_up"] + ph2["down"]
            entry = {"tokens": T, "tokens_per_s": round(world * T * steps2 / (ms2 / 1000.0), 1),
                     "ms_per_step": round(ms2 / steps2, 4), "kernel_ms": round(k2, 4),
                     "distinct_experts": u2}
            if T >= 1024:
                tf = expert_flops(T) / (k2 / 1000.0) / 1e12
                entry.update({"bound": "tensor", "achieved_tflops": round(tf, 1),
                              "frac_of_burst_peak": round(tf / bf16_peak, 4),
                              "frac_of_sustained_peak": round(tf / bf16_sust, 4)})
            else:
                gbs = expert_bytes(T, u2) / (k2 / 1000.0) / 1e9
                entry.update({"bound": "hbm", "achieved_gbs": round(gbs, 1), "frac": round(gbs / hbm_peak, 4)})
            sweep.append(entry)
            del b2

    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu_baseline:
        cpu = cpu_baseline(rb, torch, d, blk)
    streaming = None if args.no_stream else stream_measure(rb, torch, d, blk.x)
    streaming_8x22b = None if args.no_stream else stream_measure_8x22b(rb, torch, device)
    streaming_model = None if args.no_stream else stream_model_measure(rb, torch, device)
    decode = None if args.no_decode else decode_measure(rb, torch, device, decode_batches(args),
                                                        new_tokens=args.decode_new)
    fine_model = None if args.no_decode else decode_measure(
        rb, torch, device, (1, 64), prompt_len=128, new_tokens=32, seed=4, cfg=fine_model_config(),
        bytes_per_expert=FINE_BYTES_PER_EXPERT, name="fine-grained")
    fine = None if args.no_sweep else fine_grained_measure(rb, torch, device)
    quant = None if args.no_sweep else quant_measure(rb, torch, device, d, hbm_peak, peak_src)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: N(0,0.02) weights (torch cuda generator, seed 2) NF4-quantized; N(0,1) bf16 activations",
            "config": config_dict(args, world),
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps,
            "gpu_launches_note": f"{launches_per_step} kernels per step (router, gather, expert gate_up and down GEMMs, combine) replayed from one CUDA graph",
            "captured_launches": per_step_launches,
            "clocks": clk.summary(), "sweep": sweep, "streaming": streaming, "streaming_8x22b": streaming_8x22b,
            "streaming_model": streaming_model,
            "decode": decode, "fine_model_decode": fine_model, "fine_grained": fine, "quant": quant,
        }
        print(json.dumps(line), flush=True)
    del g
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_ep(args, rank, world, local, rb, torch, dist, d, device, hbm_peak, peak_src):
    """Expert parallel over `world` GPUs (weak scaling: args.tokens tokens per
    GPU); rank r keeps experts [r E/W, (r+1) E/W). Two designs are timed on
    the same tokens, each checked against the single-GPU block:

      replicated: all-gather the tokens, every rank runs its experts for all
        of them (riallm_cuda_moe_forward_ep), reduce-scatter the float32
        partials (riallm_b200.ep.ExpertParallelMoE; no host synchronisation);
      all_to_all: each rank routes its own tokens and exchanges only the
        routed rows and their expert outputs (riallm_cuda_moe_forward_ep_a2a,
        NCCL inside the library; one host synchronisation per call for the
        message sizes);
      all_to_all_peer: the same exchange by the library's own kernels,
        storing the rows into the peers' IPC-mapped buffers over NVLink
        (riallm_cuda_moe_forward_ep_peer; no host synchronisation).

    --ep-path picks the one the line's value, roofline and e2e report (the
    replicated one by default: faster at decode batch sizes); the other is
    reported beside it. Phase times come from the library's events; the
    collectives of the replicated path run in torch, so its communication is
    the step time minus the library phases."""
    from riallm_b200.ep import ExpertParallelA2A, ExpertParallelMoE, expert_range
    e_b, e_l = expert_range(E, rank, world)
    local_w = {"mlp.gate.weight": d["mlp.gate.weight"],
               "mlp.experts.gate_up_proj": d["mlp.experts.gate_up_proj"].expert_slice(e_b, e_l),
               "mlp.experts.down_proj": d["mlp.experts.down_proj"].expert_slice(e_b, e_l)}
    gen = torch.Generator(device=device).manual_seed(1000 + args.tokens + 7919 * rank)
    x = torch.empty(args.tokens, H, device=device).normal_(0, 1, generator=gen).to(torch.bfloat16)
    made = {}

    def make(name):
        # Built in the order timed, on every rank alike: the all-to-all
        # handle brings its own NCCL communicator, which need not exist
        # while the other design is timed.
        if name == "replicated":
            ctx_rep = rb.Context(device.index or 0)
            ctx_rep.reserve(world * args.tokens, H, I, E, TOP_K, torch.bfloat16)
            rep = ExpertParallelMoE(local_w, E, TOP_K)
            made[name] = (lambda v: rep(v, ctx=ctx_rep), ctx_rep, ctx_rep.close)
        else:
            a2a = ExpertParallelA2A(local_w, E, TOP_K, device=local,
                                    transport="peer" if name == "all_to_all_peer" else "nccl", max_tokens=args.tokens)
            made[name] = (a2a, a2a.ctx, a2a.close)
        return made[name]
    head = args.ep_path
    order = [head] + ([] if args.no_sweep else
                      [p for p in ("replicated", "all_to_all", "all_to_all_peer") if p != head])
    # The replicated and peer-memory steps have no host synchronisation:
    # they are timed as CUDA-graph replays (collectives and hand-offs
    # included), like the one-GPU block. The NCCL all-to-all needs the
    # message sizes on the host and runs eagerly.
    graphs = []  # released before the handles close and the group ends

    def capture(fn, xin):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                fn(xin)
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            o = fn(xin)
        graphs.append(g)
        return g, o

    res, clk, head_graphs = {}, None, None
    g = gout = None
    for name in order:
        fn, ctx, _ = make(name)
        fn(x)
        l0 = ctx.launch_count()
        fn(x)
        launches = ctx.launch_count() - l0  # library kernels of one step
        graphed = name != "all_to_all"
        if graphed:
            g, gout = capture(fn, x)
            step = g.replay
        else:
            step = (lambda f: (lambda: f(x)))(fn)
        if name == head:
            with ClockSampler(local) as clk:
                ms = timed(torch, step, args.steps, args.warmup, dist, world)
        else:
            ms = timed(torch, step, args.steps, args.warmup, dist, world)
        ph = ep_phases(torch, _EpCall(fn, ctx), x, n=10)
        ctx.synchronize()  # raises if a bounded device wait of the path expired
        lib_ms = sum(ph.values())
        chk = ep_verify(rb, torch, dist, d, fn, x, rank, world)
        if graphed:
            # The replayed step computes what the eager call does, bit for bit.
            g.replay()
            same = torch.tensor([1.0 if torch.equal(gout, fn(x)) else 0.0], device=device)
            dist.all_reduce(same, op=dist.ReduceOp.MIN)
            chk["graph_replay_equals_eager"] = bool(same.item() == 1.0)
            chk["passed"] = chk["passed"] and chk["graph_replay_equals_eager"]
            if name == head:
                xs1 = x.clone()  # the e2e loop's second input buffer
                head_graphs = [(g, gout), capture(fn, xs1)]
        res[name] = {"tokens_per_s": round(world * args.tokens * args.steps / (ms / 1000.0), 1),
                     "ms_per_step": round(ms / args.steps, 4), "launches_per_step": launches,
                     "cuda_graph": graphed, "phase_ms_per_step": ph,
                     "outside_library_ms_per_step": round(max(ms / args.steps - lib_ms, 0.0), 4),
                     "check": chk}
    ms_per_step = res[head]["ms_per_step"]
    value = res[head]["tokens_per_s"]
    launches_per_step = res[head]["launches_per_step"]
    ep_check = res[head]["check"]
    blk = made[head][0]
    ph = res[head]["phase_ms_per_step"]

    # Local expert GEMM phases on this rank (roofline of the dominant kernel).
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x)
    _, _, counts, _, _ = rb.route(d["mlp.gate.weight"], torch.cat(parts, 0), TOP_K, E)
    U_local = int((counts[e_b:e_b + e_l] > 0).sum().item())
    P_local = int(counts[e_b:e_b + e_l].sum().item())
    kern_ms = ph["gate_up"] + ph["down"]
    bytes_step = U_local * BYTES_PER_EXPERT + P_local * (H * 2 + 2 * I * 2 + H * 4)
    achieved = bytes_step / (kern_ms / 1000.0) / 1e9 if kern_ms > 0 else 0.0
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(achieved / hbm_peak, 4), "traffic": None,
                "kernel": f"expert_gemm_kernel<NF4> (rank 0's gate_up + down launches of one {head} step)",
                "algorithmic_bytes_per_step": bytes_step, "distinct_experts": U_local,
                "kernel_ms_per_step": round(kern_ms, 4),
                "phase_ms_per_step": ph,
                "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured" else peak_src}

    # End to end: this rank's tokens from pinned host memory, the block, the
    # output back to the host, every step; the copies run on a second stream,
    # double-buffered, overlapping the neighbouring steps' blocks.
    hx = torch.empty_like(x, device="cpu").pin_memory()
    hx.copy_(x.cpu())
    houts = [torch.empty_like(hx).pin_memory() for _ in range(2)]
    xs = [x, xs1] if head_graphs is not None else [x, torch.empty_like(x)]
    outs = [None, None]
    comp = torch.cuda.current_stream()
    copy = torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def head_step(b):
        if head_graphs is None:
            return blk(xs[b])
        gb, ob = head_graphs[b]
        gb.replay()
        return ob

    def e2e_run(n):
        copy.wait_stream(comp)
        with torch.cuda.stream(copy):
            xs[0].copy_(hx, non_blocking=True)
        ev_in[0].record(copy)
        for i in range(n):
            b, nb = i % 2, (i + 1) % 2
            if i + 1 < n:
                if i >= 1:
                    copy.wait_event(ev_done[nb])
                with torch.cuda.stream(copy):
                    xs[nb].copy_(hx, non_blocking=True)
                ev_in[nb].record(copy)
            comp.wait_event(ev_in[b])
            if i >= 2:
                comp.wait_event(ev_out[b])
            outs[b] = head_step(b)
            ev_done[b].record(comp)
            copy.wait_event(ev_done[b])
            with torch.cuda.stream(copy):
                houts[b].copy_(outs[b], non_blocking=True)
            ev_out[b].record(copy)
        comp.wait_stream(copy)

    e2e_run(args.warmup)
    dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    e2e_run(args.steps)
    t1.record()
    torch.cuda.synchronize()
    tt = torch.tensor([t0.elapsed_time(t1)], device="cuda")
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    e2e_ms = float(tt.item())
    # Graphs that hold NCCL calls go before the communicators do.
    head_graphs = g = gout = step = None
    graphs.clear()
    torch.cuda.synchronize()
    for _, _, close in made.values():
        close()
    fine_ep = None if args.no_sweep else ep_fine_measure(rb, torch, dist, device, rank, world)
    dec_ep = None if args.no_decode else ep_decode_measure(rb, torch, dist, device, rank, world,
                                                           decode_batches(args), new_tokens=min(args.decode_new, 64))
    fine_dec_ep = None if args.no_decode else ep_decode_measure(
        rb, torch, dist, device, rank, world, (64,), prompt_len=128, new_tokens=32, seed=4,
        cfg=fine_model_config(), name="fine-grained")
    nbytes = x.numel() * 2
    e2e = {"value": world * args.tokens * args.steps / (e2e_ms / 1000.0), "unit": "tokens/s",
           "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes,
           "ms_per_step": round(e2e_ms / args.steps, 4),
           "note": "per rank: pinned H2D of its tokens and D2H of its output on a copy stream, double-buffered"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: N(0,0.02) weights (torch cuda generator, seed 2) NF4-quantized; N(0,1) bf16 activations",
            "config": config_dict(args, world),
            "roofline": roofline, "cpu_baseline": None, "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps,
            "gpu_launches_note": f"{launches_per_step} library kernels per step per GPU ({head} path) plus its NCCL collectives",
            "clocks": clk.summary(), "sweep": [], "ep_check": ep_check, "ep_path": head, "ep_paths": res,
            "fine_grained_ep": fine_ep,
            "decode": dec_ep, "fine_model_decode": fine_dec_ep,
        }
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    fine_ok = fine_ep is None or all(r["check"]["passed"] for r in fine_ep["runs"])
    dec_ok = all(r["check"]["passed"] for dd in (dec_ep, fine_dec_ep) if dd for r in dd["runs"] if "check" in r)
    paths_ok = all(r["check"]["passed"] for r in res.values())
    return 0 if paths_ok and fine_ok and dec_ok else 1


EP_TOL = 5e-3


def ep_compare(torch, dist, out, ref):
    """Expert-parallel output against the single-GPU block on the same
    tokens, worst over the ranks. The two sum the same float32 terms in a
    different order and round each output to bf16 once, so an element may
    differ by one bf16 rounding step (up to 2^-7 of its magnitude) where the
    float32 value sits next to a rounding boundary. Passes when every
    element differs by at most one bf16 ulp of the larger of the two values
    plus 1e-3 of max |single| (the float32 reordering itself, which matters
    only for elements near zero): max |ep - single| / max |single| is then
    below 2^-7 + 1e-3, and below EP_TOL when no large element flips."""
    a, b = out.float(), ref.float()
    diff = (a - b).abs()
    _, ex = torch.frexp(torch.maximum(a.abs(), b.abs()))
    ulp = torch.ldexp(torch.ones_like(diff), (ex - 8).to(torch.int32))
    scale = b.abs().max()
    bad = (diff > ulp + 1e-3 * scale).sum().float()
    t = torch.stack([diff.max() / scale, (diff / ulp).max(), (diff > 0).sum().float() / diff.numel(), bad])
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    rel, ulps, frac, nbad = float(t[0]), float(t[1]), float(t[2]), int(t[3])
    return {"max_rel_err": rel, "max_ulps": ulps, "frac_elements_differing": frac, "elements_beyond_bound": nbad,
            "bound": "1 bf16 ulp + 1e-3 * max|single| per element", "passed": nbad == 0}


def ep_phases(torch, blk, x, n=5):
    """Mean per-phase device times (ms) of n expert-parallel steps, from the
    library's events on the launching stream (route, gather, dispatch,
    gate_up, down, return, combine; the counts exchange and its host
    synchronisation are the rest of the step)."""
    torch.cuda.synchronize()
    blk.ctx.profile(True)
    for _ in range(n):
        blk(x)
    torch.cuda.synchronize()
    blk.ctx.profile(False)
    ph, calls = blk.ctx.profile_read()
    return {k: round(v / max(calls, 1), 4) for k, v in ph.items()}


def ep_decode_measure(rb, torch, dist, device, rank, world, batches=(1, 32), prompt_len=512, new_tokens=64,
                      seed=3, cfg=None, name="mixtral-8x7b"):
    """Mixtral-8x7B decoding (32 layers, synthetic weights seed 3 as in
    decode_measure) expert parallel over the ranks: each rank keeps 8 / world
    experts of every layer plus replicated attention, norms, embedding and LM
    head, and decodes its own batch of sequences (prompt of `prompt_len` ids,
    then `new_tokens` teacher-forced steps replayed from the decode graph);
    every MoE block all-gathers the ranks' tokens and reduce-scatters the
    partial sums (ExpertParallelMoE, NCCL, captured in the graph). Times are
    the max over ranks; tok/s counts every rank's sequences. Rank 0 first runs
    its first prefill on the whole model on one GPU and checks the
    expert-parallel prefill logits against it."""
    from riallm_b200 import decoder as D
    from riallm_b200.ep import ExpertParallelMoE, expert_range
    cfg = cfg or D.DecoderConfig.mixtral_8x7b()
    dev = device.index or 0
    t0 = time.perf_counter()
    qw = D.synthetic_model(cfg, seed=seed, device=str(device))
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    g = torch.Generator().manual_seed(seed + 101 * rank)
    prompts = {B: torch.randint(0, cfg.vocab, (B, prompt_len), generator=g).to(device) for B in batches}
    conts = {B: torch.randint(0, cfg.vocab, (new_tokens, B, 1), generator=g).to(device) for B in batches}
    ref_logits = None
    if rank == 0:
        full = D.Decoder(cfg, qw, max_batch=batches[0], max_seq=prompt_len + 1, device=dev)
        ref_logits = full.forward(prompts[batches[0]]).float().cpu().numpy()
        full.close()
        del full
    dist.barrier()
    e_b, e_l = expert_range(cfg.experts, rank, world)
    local = {}
    for key, v in qw.items():
        if ".mlp.experts." in key:
            sl = v.expert_slice(e_b, e_l)
            local[key] = rb.QuantizedTensor(sl.data.clone(), tuple(sl.shape), sl.qtype, sl.scales.clone(),
                                            sl.zero_points.clone(), sl.block_size)
        else:
            local[key] = v
    del qw
    torch.cuda.empty_cache()
    ep = ExpertParallelMoE(None, cfg.experts, cfg.top_k)
    model = D.Decoder(cfg, local, max_batch=max(batches), max_seq=prompt_len + new_tokens + 3, device=dev, ep=ep)
    del local
    out = {"model": f"{name}: {cfg.layers} layers, synthetic weights (seed {seed}), experts NF4 ({e_l} per GPU), "
                    "attention/embedding bf16 replicated", "prompt_tokens": prompt_len, "new_tokens": new_tokens,
           "build_s": round(build_s, 2), "runs": []}

    def ev():
        return torch.cuda.Event(enable_timing=True)
    for B in batches:
        model.generate(prompts[B], 2)  # warm-up: prefill shapes and the decode graph for B
        model.reset()
        p0, p1, d1 = ev(), ev(), ev()
        dist.barrier()
        torch.cuda.synchronize()
        p0.record()
        logits = model.forward(prompts[B])
        p1.record()
        model.decode_forced(conts[B])
        d1.record()
        torch.cuda.synchronize()
        t = torch.tensor([p0.elapsed_time(p1), p1.elapsed_time(d1)], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        pms, dms = float(t[0]), float(t[1])
        run = {"batch_per_gpu": B, "decode_tok_s": round(world * B * new_tokens / (dms / 1000.0), 1),
               "ms_per_decode_step": round(dms / new_tokens, 3), "prefill_ms": round(pms, 2),
               "prefill_tok_s": round(world * B * prompt_len / (pms / 1000.0), 1)}
        if rank == 0 and B == batches[0]:
            lg = logits.float().cpu().numpy()
            e = float(abs(lg - ref_logits).max() / abs(ref_logits).max())
            agree = float((lg.argmax(-1) == ref_logits.argmax(-1)).mean())
            # Both runs sum the same float32 terms in another order and round
            # activations to bf16 at every layer, so an early one-ulp flip
            # can grow over the layers: logits within 2e-2 for 32 layers,
            # 5e-2 for deeper models, and the greedy token of at least 95 % of
            # the sequences unchanged.
            tol = 2e-2 if cfg.layers <= 32 else 5e-2
            run["check"] = {"prefill_logits_rel_err_vs_one_gpu": e, "tol": tol, "greedy_agreement": agree,
                            "passed": e < tol and agree >= 0.95}
        out["runs"].append(run)
    model.close()
    del model
    torch.cuda.empty_cache()
    return out


def ep_fine_measure(rb, torch, dist, device, rank, world, steps=10):
    """The fine-grained block (hidden 2048, 128 experts, top-8, intermediate
    768; N(0, 0.02) weights seed 4 quantized to NF4, as fine_grained_measure
    makes them) expert parallel over the ranks, 128 / world experts each: a
    64-token decode batch and an 8192-token prefill per rank. Step time is
    the max over ranks; phase times are rank 0's; every rank's output is
    checked against the single-GPU block on its own tokens (a token's output
    depends on that token alone), within EP_TOL."""
    from riallm_b200.ep import ExpertParallelA2A, expert_range
    Hf, If, Ef, kf = 2048, 768, 128, 8
    qt = rb.CompressionType.FourBit
    g = torch.Generator(device=device).manual_seed(4)
    d = {"mlp.gate.weight": rb.quantize_tensor(torch.randn(Ef, Hf, device=device, generator=g) * 0.02, qt),
         "mlp.experts.gate_up_proj": rb.quantize_tensor(
             torch.randn(Ef, 2 * If, Hf, device=device, generator=g) * 0.02, qt),
         "mlp.experts.down_proj": rb.quantize_tensor(torch.randn(Ef, Hf, If, device=device, generator=g) * 0.02, qt)}
    e_b, e_l = expert_range(Ef, rank, world)
    local_w = {"mlp.gate.weight": d["mlp.gate.weight"],
               "mlp.experts.gate_up_proj": d["mlp.experts.gate_up_proj"].expert_slice(e_b, e_l),
               "mlp.experts.down_proj": d["mlp.experts.down_proj"].expert_slice(e_b, e_l)}
    out = {"config": f"fine-grained: hidden 2048, 128 experts, top-8, intermediate 768, NF4; {e_l} experts per GPU",
           "runs": []}
    for transport in ("nccl", "peer"):
        blk = ExpertParallelA2A(local_w, Ef, kf, device=device.index or 0, transport=transport, max_tokens=8192)
        for T in (64, 8192):
            gx = torch.Generator(device=device).manual_seed(4000 + T + 7919 * rank)
            x = torch.randn(T, Hf, device=device, generator=gx).to(torch.bfloat16)
            ms = timed(torch, lambda: blk(x), steps, 3, dist, world)
            ph = ep_phases(torch, blk, x)
            chk = ep_compare(torch, dist, blk(x), rb.apply_moe(d, x, kf, Ef))
            blk.ctx.synchronize()  # raises if a bounded wait of the call expired
            out["runs"].append({"transport": transport, "tokens_per_gpu": T,
                                "tokens_per_s": round(world * T * steps / (ms / 1000.0), 1),
                                "ms_per_step": round(ms / steps, 4), "phase_ms_per_step": ph, "check": chk})
        blk.close()
    del d, local_w
    torch.cuda.empty_cache()
    return out


class _EpCall:
    """An expert-parallel step in the shape ep_phases expects."""

    def __init__(self, fn, ctx):
        self.fn, self.ctx = fn, ctx

    def __call__(self, x):
        return self.fn(x)


def ep_verify(rb, torch, dist, d, blk, x, rank, world):
    """Checks the expert-parallel step's output on every rank against the
    single-GPU block run on the same gathered tokens (this rank holds the
    whole layer), with ep_compare; the worst rank's figures are reported."""
    out = blk(x)
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x)
    ref = rb.apply_moe(d, torch.cat(parts, 0), TOP_K, E)[rank * x.shape[0]:(rank + 1) * x.shape[0]]
    chk = ep_compare(torch, dist, out, ref)
    chk["against"] = "single-GPU riallm_cuda_moe_forward on the same gathered tokens, every rank"
    return chk


def stream_measure(rb, torch, d, x, n_layers=4, depth=2, experts=E, top_k=TOP_K, label=None):
    """Streaming mode (ModelOptions.prefetch_layers): one NF4 MoE layer
    packed once into pinned host memory and streamed through a ring of
    `depth` device slots, n_layers layers per pass (the same layer bytes
    n_layers times), the decode batch `x` through each layer. Reports the
    H2D rate of the copies and how much of the copy time the compute hides."""
    from riallm_b200.streaming import LayerStreamer, PackedLayer
    packed = PackedLayer({k: v for k, v in d.items()})
    layers = [packed] * n_layers
    s = LayerStreamer(layers, depth=depth, device=x.device.index or 0)

    def fn(i, t):
        rb.apply_moe(t, x, top_k, experts)
    s.run(fn)  # warm-up pass
    torch.cuda.synchronize()
    b0 = s.stats()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    passes = 3
    start.record()
    for _ in range(passes):
        s.run(fn)
    end.record()
    torch.cuda.synchronize()
    wall = start.elapsed_time(end) / passes
    b1 = s.stats()
    copy_ms = (b1["copy_ms"] - b0["copy_ms"]) / passes
    nbytes = (b1["bytes"] - b0["bytes"]) / passes
    start.record()
    for _ in range(passes * n_layers):
        rb.apply_moe(d, x, top_k, experts)
    end.record()
    torch.cuda.synchronize()
    compute = start.elapsed_time(end) / passes
    s.close()
    packed.close()
    out = {"layers_per_pass": n_layers, "prefetch_buffer_size": depth, "layer_bytes": packed.nbytes,
           "tokens_per_layer": x.shape[0],
           "ms_per_pass": round(wall, 3), "h2d_gbs": round(nbytes / (copy_ms / 1000.0) / 1e9, 2),
           "h2d_gbs_wall": round(nbytes / (wall / 1000.0) / 1e9, 2),
           "compute_ms_per_pass": round(compute, 3),
           "exposed_copy_ms_per_pass": round(max(wall - compute, 0.0), 3),
           "tokens_per_s": round(x.shape[0] / (wall / 1000.0), 1),
           "note": "pinned host -> HBM over PCIe on a copy stream; copies of layers i+1 overlap layer i's block"}
    if label:
        out = {"layer": label, **out}
    return out


def stream_measure_8x22b(rb, torch, device, n_layers=2, tokens=16, seed=5):
    """The streaming measurement on a Mixtral-8x22B-shaped layer (hidden
    6144, intermediate 16384, 8 experts, top-2; N(0, 0.02) weights seed 5
    quantized to NF4, 1.57 GB per layer) with a 16-token decode batch."""
    h, inter = 6144, 16384
    d = make_layer(rb, torch, device, seed=seed, hidden=h, inter=inter, experts=E)
    gen = torch.Generator(device=device).manual_seed(seed + 1)
    x = torch.empty(tokens, h, device=device).normal_(0, 1, generator=gen).to(torch.bfloat16)
    out = stream_measure(rb, torch, d, x, n_layers=n_layers,
                         label="mixtral-8x22b block (H 6144, I 16384, E 8, top-2, NF4)")
    del d
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


def stream_model_measure(rb, torch, device, layers=4, batch=16, prompt_len=1024, new_tokens=64, seed=5, depth=2):
    """Mixtral-8x22B decoding at reduced depth (hidden 6144, 48/8 heads,
    intermediate 16384, 8 experts, top-2, V 32768; `layers` of the model's 56
    layers; synthetic weights as in decode_measure, experts NF4) run twice:
    with the MoE tensors resident in HBM (decode steps replayed from a graph)
    and streamed from pinned host memory through `depth` device slots
    (ModelOptions.prefetch_layers, eager steps). A batch of `batch` prompts
    of `prompt_len` ids, then `new_tokens` teacher-forced decode steps.
    exposed_copy_ms_per_layer = (streamed - resident) / layers: the part of
    each layer's copy that the compute does not hide."""
    from riallm_b200 import decoder as D
    from riallm_b200.streaming import LayerStreamer, PackedLayer
    cfg = D.DecoderConfig(layers=layers, hidden=6144, heads=48, kv_heads=8, head_dim=128, eps=1e-5, theta=1e6,
                          vocab=32768, experts=8, top_k=2, intermediate=16384)
    qw = D.synthetic_model(cfg, seed=seed, device=str(device))
    names = ("mlp.gate.weight", "mlp.experts.gate_up_proj", "mlp.experts.down_proj")
    ctx = rb.Context.get(device.index or 0)
    packed = [PackedLayer({n: qw[f"model.layers.{l}.{n}"] for n in names}, ctx=ctx) for l in range(layers)]
    streamer = LayerStreamer(packed, depth=depth, device=device.index or 0)
    max_seq = prompt_len + new_tokens + 3
    resident = D.Decoder(cfg, qw, max_batch=batch, max_seq=max_seq, device=device.index or 0)
    resident_w = {k: v for k, v in qw.items() if ".mlp." not in k}
    streamed = D.Decoder(cfg, resident_w, max_batch=batch, max_seq=max_seq, device=device.index or 0,
                         streamer=streamer)
    del qw
    g = torch.Generator().manual_seed(seed)
    prompt = torch.randint(0, cfg.vocab, (batch, prompt_len), generator=g).to(device)
    cont = torch.randint(0, cfg.vocab, (new_tokens, batch, 1), generator=g).to(device)

    def ev():
        return torch.cuda.Event(enable_timing=True)

    def run(model):
        model.generate(prompt, 2)  # warm-up: prefill shapes, scratch arenas, the decode graph
        model.reset()
        p0, p1, d1 = ev(), ev(), ev()
        torch.cuda.synchronize()
        p0.record()
        model.forward(prompt)
        p1.record()
        model.decode_forced(cont)
        d1.record()
        torch.cuda.synchronize()
        pms, dms = p0.elapsed_time(p1), p1.elapsed_time(d1)
        return {"prefill_ms": round(pms, 2), "prefill_tok_s": round(batch * prompt_len / (pms / 1000.0), 1),
                "ms_per_decode_step": round(dms / new_tokens, 3),
                "decode_tok_s": round(batch * new_tokens / (dms / 1000.0), 1)}
    r = run(resident)
    b0 = streamer.stats()
    s = run(streamed)
    b1 = streamer.stats()
    nbytes, copy_ms = b1["bytes"] - b0["bytes"], b1["copy_ms"] - b0["copy_ms"]
    h2d = nbytes / (copy_ms / 1000.0) / 1e9 if copy_ms > 0 else 0.0
    s["h2d_gbs"] = round(h2d, 2)
    layer_bytes = packed[0].nbytes
    streamed.close()
    streamer.close()
    # Routed: each decode step routes with resident routers and copies only
    # the experts its batch routes to (prefills still copy whole layers).
    routed_st = LayerStreamer(packed, depth=depth, device=device.index or 0, routed=True)
    routed = D.Decoder(cfg, {k: v for k, v in resident_w.items()}, max_batch=batch, max_seq=max_seq,
                       device=device.index or 0, streamer=routed_st)
    rr = run(routed)
    rb_stats = routed_st.stats()
    prefill_bytes = 2 * layers * layer_bytes  # warm-up and timed prefills copy whole layers
    rr["bytes_per_decode_step"] = int((rb_stats["bytes"] - prefill_bytes) / (new_tokens + 1))
    rr["layer_fraction_copied_per_decode_step"] = round(rr["bytes_per_decode_step"] / (layers * layer_bytes), 3)
    routed.close()
    routed_st.close()
    out = {"model": f"mixtral-8x22b shapes, {layers} of 56 layers, synthetic weights (seed {seed}), experts NF4, "
                    "attention/embedding bf16",
           "batch": batch, "prompt_tokens": prompt_len, "new_tokens": new_tokens, "prefetch_buffer_size": depth,
           "layer_bytes": layer_bytes, "resident": r, "streamed": s, "streamed_routed": rr,
           "copy_ms_per_layer": round(layer_bytes / h2d / 1e6, 3) if h2d else None,
           "exposed_copy_ms_per_layer_decode": round((s["ms_per_decode_step"] - r["ms_per_decode_step"]) / layers, 3),
           "exposed_copy_ms_per_layer_prefill": round((s["prefill_ms"] - r["prefill_ms"]) / layers, 3),
           "note": "streamed: every forward copies each layer's router + experts from pinned host memory while the "
                   "previous layer computes; resident decode steps are graph replays, streamed ones eager"}
    resident.close()
    for p in packed:
        p.close()
    del resident, streamed, routed
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


def decode_batches(args):
    return tuple(int(v) for v in args.decode_batches.split(",") if v)


def fine_model_config():
    """The fine-grained model's shapes: 48 layers, hidden 2048, 32/4 heads
    (head_dim 64), 128 experts, top-8, intermediate 768, V 32000."""
    from riallm_b200 import decoder as D
    return D.DecoderConfig(layers=48, hidden=2048, heads=32, kv_heads=4, head_dim=64, eps=1e-5, theta=1e6,
                           vocab=32000, experts=128, top_k=8, intermediate=768)


FINE_BYTES_PER_EXPERT = int(3 * 2048 * 768 * NF4_BYTES_PER_WEIGHT)  # 2,949,120


def decode_measure(rb, torch, device, batches=(1, 32), prompt_len=512, new_tokens=128, seed=3, cfg=None,
                   bytes_per_expert=BYTES_PER_EXPERT, name="mixtral-8x7b"):
    """Mixtral-8x7B (32 layers, 32/8 heads, V=32000; or `cfg`) NF4 decoding,
    weights resident in HBM: prefill a prompt of `prompt_len` ids, then
    `new_tokens` decode steps replayed from one CUDA graph per batch size
    (all layers, LM head and argmax on the device), fed a seeded random
    continuation. Timed with CUDA events on the decoding stream."""
    from riallm_b200 import decoder as D
    cfg = cfg or D.DecoderConfig.mixtral_8x7b()
    hbm_peak = load_peaks()[0]
    t0 = time.perf_counter()
    qw = D.synthetic_model(cfg, seed=seed, device=str(device))
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    model = D.Decoder(cfg, qw, max_batch=max(batches), max_seq=prompt_len + new_tokens + 1, device=device.index or 0)
    del qw
    attn_bytes = ((cfg.heads + 2 * cfg.kv_heads) * cfg.head_dim * cfg.hidden + cfg.hidden * cfg.heads * cfg.head_dim) * 2
    lm_bytes = cfg.vocab * cfg.hidden * 2
    out = {"model": f"{name}: {cfg.layers} layers, synthetic weights (seed {seed}), experts NF4, "
                    "attention/embedding bf16",
           "prompt_tokens": prompt_len, "new_tokens": new_tokens, "build_s": round(build_s, 2), "runs": []}
    g = torch.Generator().manual_seed(seed)

    def ev():
        return torch.cuda.Event(enable_timing=True)
    for B in batches:
        prompt = torch.randint(0, cfg.vocab, (B, prompt_len), generator=g).to(device)
        model.generate(prompt, 2)  # warm-up: prefill shapes (cuBLAS, scratch arena), the decode graph for B
        # Each decode step is fed the next ids of a seeded random continuation
        # (teacher forcing): greedy decoding of random weights collapses every
        # sequence onto one token, which would route all of them to the same
        # experts. The step itself (all layers, LM head, argmax) is unchanged.
        cont = torch.randint(0, cfg.vocab, (new_tokens + 1, B, 1), generator=g).to(device)
        model.reset()
        p0, p1, d0, d1 = ev(), ev(), ev(), ev()
        torch.cuda.synchronize()
        p0.record()
        model.forward(prompt)
        p1.record()
        d0.record()
        model.decode_forced(cont[:new_tokens])
        d1.record()
        torch.cuda.synchronize()
        dec_ms = d0.elapsed_time(d1)
        ms_tok = dec_ms / new_tokens
        # Experts each layer's block actually routed to, from one more decode
        # step run eagerly (after the timed region) with a router probe.
        used = model.experts_per_layer(cont[new_tokens])
        U = sum(used) / len(used)
        kv_read = B * cfg.kv_heads * (prompt_len + new_tokens // 2) * cfg.head_dim * 2 * 2
        step_bytes = sum(u * bytes_per_expert for u in used) + cfg.layers * (attn_bytes + kv_read) + lm_bytes
        gbs = step_bytes / (ms_tok / 1000.0) / 1e9
        pms = p0.elapsed_time(p1)
        out["runs"].append({
            "batch": B, "decode_tok_s": round(B * new_tokens / (dec_ms / 1000.0), 1),
            "ms_per_decode_step": round(ms_tok, 3), "prefill_ms": round(pms, 2),
            "prefill_tok_s": round(B * prompt_len / (pms / 1000.0), 1),
            "step_bytes": int(step_bytes), "achieved_gbs": round(gbs, 1), "frac_hbm": round(gbs / hbm_peak, 4),
            "experts_per_layer": round(U, 2),
            "bytes_note": "per decode step: the NF4 experts each layer routed to (counted on one more step) + "
                          f"{cfg.layers} x (bf16 attention weights + mean KV-cache read) + LM head"})
    model.close()
    del model
    torch.cuda.empty_cache()
    return out


def zipf_bias(torch, n, s=1.1, seed=4):
    """Expert-popularity bias of the fine-grained configuration:
    bias_e = ln(r_e^-s / sum_r r^-s), the ranks r_e = 1..n given to the
    experts by a seeded permutation (torch CPU generator)."""
    g = torch.Generator().manual_seed(seed)
    ranks = torch.randperm(n, generator=g).double() + 1.0
    w = ranks ** -s
    return torch.log(w / w.sum()).float()


def quant_measure(rb, torch, device, d, hbm_peak, peak_src, reps=5, experts=None):
    """The standalone block dequantizer and quantizer (src/quantization.rs:
    45-245) on the Mixtral-8x7B layer's gate_up_proj (8 x 28672 x 4096 =
    939,524,096 weights): HBM GB/s = algorithmic bytes (codes + float32
    scales and zero points read, values written; or float32 read and codes,
    scales, zero points written) / CUDA-event time on the launching stream,
    best of `reps` launches after one warm-up, against the measured copy
    peak. Inputs and outputs are larger than L2. experts=K takes the first K
    experts' slice only (K = 1: 117 M weights, still above L2 with its
    output), the size a profiler capture is run on."""
    gu = d["mlp.experts.gate_up_proj"]
    label = "mixtral8x7b gate_up_proj [8, 28672, 4096]"
    if experts:
        gu = gu.expert_slice(0, experts)
        label = f"mixtral8x7b gate_up_proj, experts 0..{experts - 1} [{experts}, 28672, 4096]"
    n = gu.numel
    out = {"tensor": label, "elements": n,
           "peak": hbm_peak, "peak_source": peak_src, "runs": []}

    def best(fn):
        fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        return min(ts)

    def entry(name, nbytes, ms):
        gbs = nbytes / (ms / 1000.0) / 1e9
        out["runs"].append({"op": name, "bytes": int(nbytes), "ms": round(ms, 4), "gbs": round(gbs, 1),
                            "frac": round(gbs / hbm_peak, 4)})

    code_b = gu.data.numel() + 8 * gu.scales.numel()
    for dt, esz in ((torch.bfloat16, 2), (torch.float32, 4)):
        ms = best(lambda: gu.dequantize(dt))
        entry(f"dequantize NF4 -> {str(dt).split('.')[-1]}", code_b + esz * n, ms)
    src = gu.dequantize(torch.float32)  # any float32 values of this size
    for c, name in ((rb.CompressionType.EightBit, "8-bit"), (rb.CompressionType.FourBit, "NF4")):
        ms = best(lambda: rb.quantize_tensor(src, c))
        q = rb.quantize_tensor(src, c)
        entry(f"quantize float32 -> {name}", 4 * n + q.data.numel() + 8 * q.scales.numel(), ms)
        if c == rb.CompressionType.EightBit:
            ms = best(lambda: q.dequantize(torch.bfloat16))
            entry("dequantize 8-bit -> bfloat16", q.data.numel() + 8 * q.scales.numel() + 2 * n, ms)
        del q
    del src
    return out


def fine_grained_measure(rb, torch, device, steps=20):
    """The fine-grained MoE configuration (hidden 2048, 128 experts, top-8,
    intermediate 768; N(0, 0.02) weights, seed 4): a 64-token decode batch
    with NF4 and with 8-bit experts, an 8192-token prefill with NF4, and a
    64-token NF4 decode batch whose router logits carry a Zipf(1.1)
    expert-popularity bias. The router has no bias input, so the bias rides
    on the last hidden feature: it is set to 1 in every token and the
    router's last column holds the bias; that router stays float32 (a
    quantized one would lose the bias to the block's absmax). Expert-GEMM
    time from the library's phase events; one block call per step."""
    Hf, If, Ef, kf = 2048, 768, 128, 8
    ctx = rb.Context.get(device.index or 0)
    hbm_peak, bf16_peak, _, _ = load_peaks()
    out = {"config": "fine-grained: hidden 2048, 128 experts, top-8, intermediate 768", "runs": []}
    for qt, T, zipf in ((rb.CompressionType.FourBit, 64, False), (rb.CompressionType.EightBit, 64, False),
                        (rb.CompressionType.FourBit, 8192, False), (rb.CompressionType.FourBit, 64, True)):
        g = torch.Generator(device=device).manual_seed(4)
        wg = torch.randn(Ef, Hf, device=device, generator=g) * 0.02
        if zipf:
            wg[:, Hf - 1] = zipf_bias(torch, Ef).to(device)
        d = {"mlp.gate.weight": wg if zipf else rb.quantize_tensor(wg, qt),
             "mlp.experts.gate_up_proj": rb.quantize_tensor(
                 torch.randn(Ef, 2 * If, Hf, device=device, generator=g) * 0.02, qt),
             "mlp.experts.down_proj": rb.quantize_tensor(torch.randn(Ef, Hf, If, device=device, generator=g) * 0.02, qt)}
        x = torch.randn(T, Hf, device=device, generator=g)
        if zipf:
            x[:, Hf - 1] = 1.0
        x = x.to(torch.bfloat16)
        counts = rb.route(d["mlp.gate.weight"], x, kf, Ef)[2]
        U = int((counts > 0).sum().item())
        for _ in range(3):
            rb.apply_moe(d, x, kf, Ef)
        ms = timed(torch, lambda: rb.apply_moe(d, x, kf, Ef), steps, 3, None, 1)
        ph, _ = phase_profile(torch, _Call(rb, d, x, kf, Ef, ctx), max(steps, 10))
        kern_ms = ph["gate_up"] + ph["down"]
        bpw = 0.625 if qt == rb.CompressionType.FourBit else 1.0 + 8.0 / 128.0
        run = {"qtype": qt.name, "tokens": T, "tokens_per_s": round(T * steps / (ms / 1000.0), 1),
               "ms_per_step": round(ms / steps, 4), "distinct_experts": U,
               "max_pairs_per_expert": int(counts.max().item()), "kernel_ms": round(kern_ms, 4),
               "phase_ms": {k: round(v, 4) for k, v in ph.items()}}
        if zipf:
            run["router"] = "float32 with a Zipf(1.1) expert-popularity bias"
        if T <= 512:
            bytes_step = U * 3 * Hf * If * bpw
            gbs = bytes_step / (kern_ms / 1000.0) / 1e9
            run.update({"bound": "hbm", "achieved_gbs": round(gbs, 1), "frac": round(gbs / hbm_peak, 4)})
        else:
            tf = 2.0 * T * kf * 3 * Hf * If / (kern_ms / 1000.0) / 1e12
            run.update({"bound": "tensor", "achieved_tflops": round(tf, 1), "frac_of_burst_peak": round(tf / bf16_peak, 4)})
        out["runs"].append(run)
        del d
        torch.cuda.empty_cache()
    return out


class _Call:
    """A block call in the shape phase_profile expects."""

    def __init__(self, rb, d, x, k, E, ctx):
        self.rb, self.d, self.x, self.k, self.E, self.ctx = rb, d, x, k, E, ctx

    def __call__(self, stream_ptr=None):
        self.rb.apply_moe(self.d, self.x, self.k, self.E)


def cpu_baseline(rb, torch, d, blk):
    """The oracle's fp32 CPU port on the same weights, timed on this host's
    cores on a bounded sample (one full decode batch, repeated)."""
    import numpy as np
    from oracle import oracle as O
    O.build()

    def host_q(q):
        return O.QTensor(int(q.qtype), q.data.cpu().numpy(), q.scales.cpu().numpy(),
                         q.zero_points.cpu().numpy(), q.numel, q.block_size)
    w = O.MoeWeights(host_q(d["mlp.gate.weight"]), host_q(d["mlp.experts.gate_up_proj"]),
                     host_q(d["mlp.experts.down_proj"]))
    x = blk.x.view(torch.int16).cpu().numpy().view(np.uint16)
    threads = os.cpu_count() or 1
    T = x.shape[0]
    t0 = time.perf_counter()
    reps = 0
    while True:
        O.moe_forward(w, x, T, H, I, E, TOP_K, n_threads=threads)
        reps += 1
        el = time.perf_counter() - t0
        if el > 8.0 or reps >= 3:
            break
    return {"value": round(T * reps / el, 2), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{reps} x full {T}-token decode batch through the fp32 oracle port "
                      f"(oracle/riallm_oracle.c, OpenMP), same NF4 weights"}


def parse_args(argv=None):
    """Command-line options; fewer than 3 warm-up steps are raised to 3."""
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--ep-path", choices=("replicated", "all_to_all", "all_to_all_peer"), default="replicated",
                    help="expert-parallel design the multi-GPU line reports (the other is timed beside it)")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--skip-cpu-baseline", action="store_true")
    ap.add_argument("--no-stream", action="store_true", help="skip the layer-streaming measurement")
    ap.add_argument("--no-decode", action="store_true", help="skip the Mixtral-8x7B decode measurement")
    ap.add_argument("--quant-only", action="store_true",
                    help="only the standalone quantize / dequantize measurement (prints {\"quant\": ...})")
    ap.add_argument("--quant-experts", type=int, default=0,
                    help="with --quant-only: the first K experts' slice of gate_up_proj instead of all 8")
    ap.add_argument("--fine-grained-only", action="store_true",
                    help="only the 128-expert top-8 measurement (prints {\"fine_grained\": ...})")
    ap.add_argument("--fine-model-only", action="store_true",
                    help="only the 48-layer fine-grained model decode (prints {\"fine_model_decode\": ...})")
    ap.add_argument("--stream-model-only", action="store_true",
                    help="only the reduced-depth streamed Mixtral-8x22B decode (prints {\"streaming_model\": ...})")
    ap.add_argument("--decode-only", action="store_true",
                    help="run only the Mixtral-8x7B decode measurement and print its JSON")
    ap.add_argument("--decode-batches", default="1,32", help="batch sizes of the decode measurement")
    ap.add_argument("--decode-new", type=int, default=128, help="decode steps per batch size")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    return args


def main():
    args = parse_args()
    rank, world, local = dist_setup()
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.decode_only:
        import torch
        import riallm_b200 as rb
        torch.cuda.set_device(local)
        r = decode_measure(rb, torch, torch.device("cuda", local), decode_batches(args), new_tokens=args.decode_new)
        print(json.dumps({"decode": r}), flush=True)
        return 0
    if args.fine_model_only:
        import torch
        import riallm_b200 as rb
        torch.cuda.set_device(local)
        r = decode_measure(rb, torch, torch.device("cuda", local), (1, 64), prompt_len=128, new_tokens=32, seed=4,
                           cfg=fine_model_config(), bytes_per_expert=FINE_BYTES_PER_EXPERT, name="fine-grained")
        print(json.dumps({"fine_model_decode": r}), flush=True)
        return 0
    if args.stream_model_only:
        import torch
        import riallm_b200 as rb
        torch.cuda.set_device(local)
        r = stream_model_measure(rb, torch, torch.device("cuda", local))
        print(json.dumps({"streaming_model": r}), flush=True)
        return 0
    if args.quant_only or args.fine_grained_only:
        import torch
        import riallm_b200 as rb
        torch.cuda.set_device(local)
        device = torch.device("cuda", local)
        hbm_peak, _, _, peak_src = load_peaks()
        if args.quant_only:
            r = quant_measure(rb, torch, device, make_layer(rb, torch, device), hbm_peak, peak_src,
                              experts=args.quant_experts or None)
            print(json.dumps({"quant": r}), flush=True)
        else:
            print(json.dumps({"fine_grained": fine_grained_measure(rb, torch, device)}), flush=True)
        return 0
    return run_ours(args, rank, world, local)


if __name__ == "__main__":
    sys.exit(main())

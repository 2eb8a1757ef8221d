"""Benchmark of the poly-attention hot path on B200.

Workload (the headline metric's configuration): order-2 causal poly
attention forward + backward, bf16, batch 8 x 16 heads x seq 4096 x
dim_head 64 (the attention core of PolyAttention(dim=1024, heads=16,
dim_head=64, causal=True)). One step = pass 1 + pass 2 forward, then pass 2 +
pass 1 backward, over synthetic N(0, 1) inputs resident in HBM (4 inputs + dO,
67 MB each, together larger than the 126 MB L2).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU (torchrun, one rank per GPU): every rank runs the full per-GPU
workload on its own batch (batch x head sharding, no collective), so total
work grows with N ("weak"); time is the max over ranks.

The reference arm (--impl reference) times the CPU restatement of the
reference algorithm (oracle/poly_oracle.py, numpy, all host threads) on a
bounded sample: one (batch, head) unit of the same workload per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "poly-attention_b200"))

METRIC = "order-2 poly-attn fwd+bwd tokens/s/GPU @4K ctx (% bf16 peak); decode tok/s"
B, H, N, D = 8, 16, 4096, 64


def pass_fwd_flop(b):
    """Algorithmic FLOPs of one causal pass forward: 2 GEMMs of 2*n*n*d/2 per (b, h)."""
    return 2 * 2 * (N * N / 2) * D * b * H


# DRAM bytes per launch per batch element, from the ncu captures summarised in
# profiles/ (batch-1 case; traffic scales with batch: every (b, h) reads its own
# q/k/v once). pass_fwd_tc2: read 25.2 MB; pass_bwd_tc: read 50.9 MB.
TRAFFIC_PER_BATCH = {"pass1_fwd": 25.23e6, "pass2_fwd": 25.49e6, "pass2_bwd": 50.9e6, "pass1_bwd": 50.9e6}


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            pk = json.load(f)
        return pk["bf16_tflops_sustained"], pk["bf16_tflops"], pk["hbm_gbs"], "measured"
    return 1400.0, 1590.0, 6650.0, "fallback"


class ClockSampler:
    """SM clocks and throttle reasons sampled during the timed region: NVML
    queries every 10 ms from a background thread (read-only; the GPU is found
    by the CUDA device's UUID), or nvidia-smi every 200 ms where NVML is not
    usable. A timed region of tens of milliseconds gets several samples."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []
        self.samples = []          # (sm_mhz, max_mhz, reasons) from NVML
        self.source = None
        self._stop = None
        self._thread = None

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        uuid = "GPU-" + str(torch.cuda.get_device_properties(self.index).uuid)
        return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid)

    def _nvml_loop(self, pynvml, hdl):
        bits = [getattr(pynvml, "nvmlClocksEventReason" + n, None) for n in
                ("HwSlowdown", "HwThermalSlowdown", "SwThermalSlowdown", "SwPowerCap")]
        mx = pynvml.nvmlDeviceGetMaxClockInfo(hdl, pynvml.NVML_CLOCK_SM)
        while not self._stop.is_set():
            try:
                sm = pynvml.nvmlDeviceGetClockInfo(hdl, pynvml.NVML_CLOCK_SM)
                r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(hdl)
                self.samples.append((sm, mx, [n for n, bt in zip(self.NAMES, bits) if bt is not None and r & bt]))
            except Exception:  # noqa: BLE001 - a failed query only loses a sample
                pass
            self._stop.wait(0.01)

    def __enter__(self):
        import threading
        try:
            pynvml, hdl = self._nvml_handle()
            self._stop = threading.Event()
            self._thread = threading.Thread(target=self._nvml_loop, args=(pynvml, hdl), daemon=True)
            self._thread.start()
            self.source = "nvml 10 ms"
            return self
        except Exception:  # noqa: BLE001 - NVML absent or unusable: nvidia-smi instead
            self._thread = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.source = "nvidia-smi 200 ms"
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
            try:
                import pynvml
                pynvml.nvmlShutdown()
            except Exception:  # noqa: BLE001 - shutdown failure changes nothing measured
                pass
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        for s_mhz, m_mhz, rs in self.samples:
            sm.append(float(s_mhz))
            mx = float(m_mhz)
            reasons.update(rs)
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(self.NAMES, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": self.source}


def make_inputs(device, seed, b):
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    return [torch.randn(b, H, N, D, device=device, dtype=torch.bfloat16, generator=g) for _ in range(5)]


def step_device(P, q1, q2, q3, v3, do, ev=None):
    """One forward + backward of both passes through the library's pass API."""
    if ev is not None:
        ev[0].record()
    msg, lse23 = P.pass_fwd(q2, q3, v3, causal=True)
    if ev is not None:
        ev[1].record()
    out, lse12 = P.pass_fwd(q1, q2, msg, causal=True, bias=lse23)
    if ev is not None:
        ev[2].record()
    _, dq2, dmsg, dlse23 = P.pass_bwd(q1, q2, msg, out, lse12, do, causal=True, bias=lse23, want_dbias=True)
    if ev is not None:
        ev[3].record()
    P.pass_bwd(q2, q3, v3, msg, lse23, dmsg, causal=True, dlse=dlse23, dq=dq2, dq_accumulate=True)
    if ev is not None:
        ev[4].record()


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import poly_attention_b200 as P
    from poly_attention_b200 import _lib

    b = args.batch
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    q1, q2, q3, v3, do = make_inputs(dev, 1234 + rank, b)
    for _ in range(args.warmup):
        step_device(P, q1, q2, q3, v3, do)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    # device-resident timed region: K steps between two events
    n0 = _lib.launch_count()
    per = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        torch.cuda.synchronize()
        start.record()
        for i in range(args.steps):
            step_device(P, q1, q2, q3, v3, do, per[i])
        end.record()
        torch.cuda.synchronize()
    launches = _lib.launch_count() - n0
    phases = [statistics.median(e[k].elapsed_time(e[k + 1]) for e in per) for k in range(4)]
    t = torch.tensor([start.elapsed_time(end)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())

    # end to end through the public API: host (pinned) inputs in, gradients out.
    # Headline: HostStreamedOrder2 (batch chunks streamed, PCIe both ways
    # overlapped with the kernels); also the plain autograd call
    # (flash_poly_attention + backward, copies before and after).
    e2e = None
    if not args.no_e2e:
        hosts = [x.cpu().pin_memory() for x in (q1, q2, q3, v3, do)]
        grads_h = [torch.empty_like(hosts[0]).pin_memory() for _ in range(4)]
        streamer = P.HostStreamedOrder2(batch=b, heads=H, kv_heads=H, seq_len=N, dim_head=D, device=dev,
                                        chunk=args.e2e_chunk)

        def e2e_streamed():
            # consecutive steps overlap (the next step's inputs stream in while
            # this one finishes); the timed region ends after join()
            streamer.step(*hosts, grads=grads_h, sync=False)

        def e2e_autograd():
            d_in = [h.to(dev, non_blocking=True) for h in hosts]
            ts = [x.requires_grad_(True) for x in d_in[:4]]
            out = P.flash_poly_attention(*ts, is_causal=True)
            out.backward(d_in[4])
            for gh, tt in zip(grads_h, ts):
                gh.copy_(tt.grad, non_blocking=True)

        def timed(fn, finish=None):
            fn()
            if finish:
                finish()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            k2 = max(3, min(args.steps, 10))
            s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s2.record()
            for _ in range(k2):
                fn()
            if finish:
                finish()
            e2.record()
            torch.cuda.synchronize()
            te = torch.tensor([s2.elapsed_time(e2) / k2], device=dev)
            if world > 1:
                dist.all_reduce(te, op=dist.ReduceOp.MAX)
            return b * N * world / (float(te.item()) * 1e-3)

        h2d, d2h = streamer.bytes_per_step()
        e2e = {"value": timed(e2e_streamed, streamer.join), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "api": f"HostStreamedOrder2.step (chunk {args.e2e_chunk})",
               "autograd_serial": {"value": timed(e2e_autograd), "unit": "tokens/s",
                                   "api": "flash_poly_attention + backward, copies before / after"}}
    decode = None if args.no_decode else run_decode(args, dev)
    if world > 1:
        dist.barrier()
    if rank != 0:
        return None

    sustained, burst, hbm, kind = peaks()
    ms_step = ms_max / args.steps
    pf = pass_fwd_flop(b)
    step_flop = 6 * pf
    names = ["pass1_fwd", "pass2_fwd", "pass2_bwd", "pass1_bwd"]
    flops = [pf, pf, 2 * pf, 2 * pf]
    dom = max(range(4), key=lambda k: phases[k])
    achieved = flops[dom] / (phases[dom] * 1e-3) / 1e12
    return {
        "metric": METRIC,
        "value": b * N * world / (ms_step * 1e-3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic N(0,1), seeded; inputs resident in HBM",
        "config": {"workload": "order-2 causal poly-attention core fwd+bwd (config 2)", "global_batch": b * world,
                   "heads": H, "seq_len": N, "dim_head": D, "parallelism": f"dp{world} (batch x head sharding)",
                   "l2": "inputs (5 x 67 MB per GPU at batch 8) larger than L2; no flush"},
        "tflops": step_flop / (ms_step * 1e-3) / 1e12,
        "frac_of_peak": step_flop / (ms_step * 1e-3) / 1e12 / sustained,
        "phases_ms": dict(zip(names, phases)),
        "roofline": {"bound": "tensor", "kernel": names[dom], "achieved": achieved, "peak": sustained,
                     "unit": "TFLOP/s", "frac": achieved / sustained,
                     "traffic": TRAFFIC_PER_BATCH[names[dom]] * b,
                     "traffic_note": "ncu DRAM read+write bytes of a batch-1 capture x batch",
                     "peak_kind": f"{kind} bf16 sustained"},
        "e2e": e2e,
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
        "cpu_baseline": cpu_baseline() if (world == 1 and not args.no_cpu) else None,
        "decode": decode,
    }


def run_decode(args, dev):
    """Config 4 decode: NPolyAttention order 3 core, batch 32, 16 query / 4 kv
    heads, d 128, bf16; caches of 2048 positions (synthetic N(0,1) contents
    stand in for the prefill), then 256 single-token steps through
    ChainDecoder (in-place cache appends + one decode launch per level).
    --decode-batch / --decode-cache change batch and prefilled length (e.g.
    one sequence with a 131072-position cache, the global-split mode)."""
    import torch

    from poly_attention_b200 import _lib
    from poly_attention_b200.decode import ChainDecoder
    b, h, g, d, order, L0 = args.decode_batch, 16, 4, 128, 3, args.decode_cache
    steps = 256 if args.workload != "decode" else max(1, args.steps)
    dec = ChainDecoder(batch=b, order=order, heads=h, kv_heads=g, dim_head=d, capacity=L0 + steps + 8,
                       dtype=torch.bfloat16, device=dev)
    gen = torch.Generator(device=dev).manual_seed(77)
    for buf in dec.qs + dec.vs + dec.msgs:
        buf[:, :, :L0].normal_(generator=gen)
    for buf in dec.lses:
        buf[:, :, :L0].normal_(generator=gen)
    dec.length = L0
    q1 = torch.randn(b, h, 1, d, device=dev, dtype=torch.bfloat16, generator=gen)
    qn = [torch.randn(b, g, 1, d, device=dev, dtype=torch.bfloat16, generator=gen) for _ in range(order)]
    vn = [torch.randn(b, g, 1, d, device=dev, dtype=torch.bfloat16, generator=gen) for _ in range(order - 1)]
    out = torch.empty(b, h, 1, d, device=dev, dtype=torch.bfloat16)
    for _ in range(3):  # warm-up steps, then rewind
        dec.append_kv(qn, vn)
        dec.step(q1, out)
    dec.length = L0
    torch.cuda.synchronize()
    total_bytes = 0
    n0 = _lib.launch_count()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        dec.append_kv(qn, vn)
        dec.step(q1, out)
        total_bytes += dec.bytes_per_step()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e)
    _, _, hbm, kind = peaks()
    gbs = total_bytes / (ms * 1e-3) / 1e9
    return {"metric": "decode tok/s", "value": b * steps / (ms * 1e-3), "unit": "tokens/s", "steps": steps,
            "ms_per_step": ms / steps, "config": {"workload": "NPolyAttention order 3 core decode (config 4)"
                                                  if (b, L0) == (32, 2048) else "NPolyAttention order 3 core decode",
                                                  "batch": b, "heads": h, "kv_heads": g, "dim_head": d,
                                                  "cache_len": f"{L0 + 1}..{L0 + steps}"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                         "traffic": None, "peak_kind": f"{kind} copy bandwidth",
                         "bytes_note": "7 bf16 cache tensors + 2 fp32 lse caches at kv-head width per position"},
            "gpu_launches": int(_lib.launch_count() - n0)}


def run_longctx(args, rank, world, local_rank):
    """Config 5: order-2 causal forward, b1 h16 n32768 d64 bf16, keys split
    across the ranks (zig-zag shards, one max all-reduce + one reduce-scatter of
    fp32 partials); total work fixed ("strong" scaling)."""
    import torch
    import torch.distributed as dist

    from poly_attention_b200 import _lib
    from poly_attention_b200.distributed import context_parallel_order2_fwd, zigzag_shard
    b, h, n, d = 1, 16, 32768, 64
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(5)
    full = [torch.randn(b, h, n, d, device=dev, dtype=torch.bfloat16, generator=g) for _ in range(4)]
    loc = [zigzag_shard(t, rank, world).contiguous() for t in full]
    del full
    for _ in range(args.warmup):
        context_parallel_order2_fwd(*loc)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    n0 = _lib.launch_count()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        context_parallel_order2_fwd(*loc)
    e.record()
    torch.cuda.synchronize()
    t = torch.tensor([s.elapsed_time(e) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank != 0:
        return None
    ms = float(t.item())
    flop = 2 * 2 * 2 * (n * n / 2) * d * h * b            # two causal passes
    sustained, _, _, kind = peaks()
    return {"metric": "long-context order-2 fwd ms (config 5)", "value": ms, "unit": "ms", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1), seeded",
            "config": {"workload": "order-2 causal fwd, keys split across GPUs", "batch": b, "heads": h,
                       "seq_len": n, "dim_head": d, "parallelism": f"cp{world} (zig-zag key split)"},
            "tflops": flop / (ms * 1e-3) / 1e12, "frac_of_peak": flop / (ms * 1e-3) / 1e12 / (sustained * world),
            "peak_kind": f"{kind} bf16 sustained x {world}", "gpu_launches_rank0": int(_lib.launch_count() - n0)}


def _time_module(fn, args, dev):
    import torch
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / args.steps


def run_module_configs(args, dev):
    """Configs 1, 3 and the config-4 prefill through the drop-in modules
    (projections / norms / MLPs in PyTorch, attention cores in libpolyattn)."""
    import torch

    import poly_attention_b200 as P
    torch.manual_seed(0)
    out = {}
    if args.workload == "config1":
        m = P.PolyAttention(dim=512, heads=8, dim_head=64, causal=False).to(dev)
        x = torch.randn(1, 1024, 512, device=dev)
        with torch.no_grad():
            ms = _time_module(lambda: m(x), args, dev)
        out = {"metric": "config 1 PolyAttention fp32 forward tokens/s", "value": 1024 / (ms * 1e-3),
               "unit": "tokens/s", "ms_per_step": ms, "dtype": "f32",
               "config": {"workload": "PolyAttention(dim=512, heads=8, dim_head=64) fwd, x [1, 1024, 512]"}}
    elif args.workload == "vit":
        m = P.PolyViT(image_size=256, patch_size=32, num_classes=1000, dim=1024, depth=6, heads=16, dim_head=64,
                      mlp_dim=2048, order=2).to(dev, torch.bfloat16)
        img = torch.randn(256, 3, 256, 256, device=dev, dtype=torch.bfloat16)
        with torch.no_grad():
            ms = _time_module(lambda: m(img), args, dev)
        flop = 2.01e12
        sustained, _, _, kind = peaks()
        out = {"metric": "config 3 PolyViT bf16 forward images/s", "value": 256 / (ms * 1e-3), "unit": "images/s",
               "ms_per_step": ms, "dtype": "bf16", "tflops": flop / (ms * 1e-3) / 1e12,
               "frac_of_peak": flop / (ms * 1e-3) / 1e12 / sustained,
               "config": {"workload": "PolyViT(256/32, dim 1024, depth 6, heads 16, mlp 2048) fwd, batch 256",
                          "tokens": "64 patches (the reference has no cls token)"}}
    elif args.workload == "prefill4":
        m = P.NPolyAttention(dim=2048, order=3, heads=16, kv_heads=4, dim_head=128, causal=True).to(
            dev, torch.bfloat16)
        x = torch.randn(32, 2048, 2048, device=dev, dtype=torch.bfloat16)
        with torch.no_grad():
            ms = _time_module(lambda: m(x), args, dev)
        out = {"metric": "config 4 NPolyAttention order-3 GQA prefill tokens/s", "value": 32 * 2048 / (ms * 1e-3),
               "unit": "tokens/s", "ms_per_step": ms, "dtype": "bf16",
               "config": {"workload": "NPolyAttention(dim=2048 assumed, order 3, h16, g4, d128, causal) fwd, "
                                      "x [32, 2048, 2048]"}}
    out.update({"n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "data": "synthetic N(0,1), seeded",
                "higher_is_better": True, "vs_baseline": None})
    return out


def cpu_unit_seconds():
    """Oracle (numpy, fp32) forward + backward of one (batch, head) unit of the workload."""
    import numpy as np

    from oracle import poly_oracle as O
    r = np.random.default_rng(0)
    a = [r.standard_normal((1, 1, N, D)).astype(np.float32) for _ in range(5)]
    t0 = time.perf_counter()
    O.order2_fwd(a[0], a[1], a[1], a[2], a[3], causal=True)
    O.order2_bwd(a[0], a[1], a[1], a[2], a[3], a[4], causal=True)
    return time.perf_counter() - t0


def cpu_baseline():
    sec = cpu_unit_seconds()
    # one unit = one head of one sequence; a token needs all H heads
    return {"value": N / (sec * H), "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"one (batch, head) unit: seq {N}, dim_head {D}, fp32 numpy fwd+bwd, {sec:.2f} s"}


def run_reference(args, rank):
    if rank != 0:
        return None
    for _ in range(args.warmup):
        cpu_unit_seconds()
    sec = statistics.median(cpu_unit_seconds() for _ in range(args.steps))
    v = N / (sec * H)
    return {
        "metric": METRIC, "impl": "reference", "value": v, "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1), seeded",
        "config": {"workload": "order-2 causal poly-attention core fwd+bwd (config 2)", "global_batch": B,
                   "heads": H, "seq_len": N, "dim_head": D, "parallelism": "cpu"},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": "one (batch, head) unit per step, fp32 numpy restatement of the reference"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=B, help="per-GPU batch (smaller for profiling captures)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--e2e-chunk", type=int, default=1, help="batch elements per streamed chunk (e2e leg)")
    ap.add_argument("--no-decode", action="store_true", help="skip the KV-cache decode leg")
    ap.add_argument("--decode-batch", type=int, default=32, help="decode leg batch (config 4: 32)")
    ap.add_argument("--decode-cache", type=int, default=2048, help="decode leg prefilled cache length (config 4: 2048)")
    ap.add_argument("--workload", choices=["train", "longctx", "config1", "vit", "prefill4", "decode"], default="train",
                    help="train: config 2 fwd+bwd (the headline); longctx: config 5 key-split forward")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        res = run_reference(args, rank)
    else:
        if world > 1:
            import torch
            import torch.distributed as dist
            torch.cuda.set_device(local_rank)
            dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
        if args.workload == "longctx":
            res = run_longctx(args, rank, world, local_rank)
        elif args.workload == "decode":
            import torch
            res = run_decode(args, torch.device("cuda", local_rank)) if rank == 0 else None
        elif args.workload in ("config1", "vit", "prefill4"):
            import torch
            res = run_module_configs(args, torch.device("cuda", local_rank)) if rank == 0 else None
        else:
            res = run_ours(args, rank, world, local_rank)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()

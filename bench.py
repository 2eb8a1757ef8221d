"""Benchmark of the poly-attention hot path on B200.

Workload (the headline metric's configuration): order-2 causal poly
attention forward + backward, bf16, batch 8 x 16 heads x seq 4096 x
dim_head 64 (the attention core of PolyAttention(dim=1024, heads=16,
dim_head=64, causal=True)). One step = pass 1 + pass 2 forward, then pass 2 +
pass 1 backward, over synthetic N(0, 1) inputs resident in HBM (4 inputs + dO,
67 MB each, together larger than the 126 MB L2).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

The default line also carries, as sub-objects, the other BASELINE configs
measured on the same GPU (config 1 module fp32 forward, config 3 PolyViT,
config 4 prefill and decode, config 5 long-context forward), each with its
own clock record and roofline fraction, the reference's own Triton kernel
timed on the same inputs (``triton_reference``, run in a child process), and
``cpu_baseline``: the reference's torch CPU path on one sequence of the
bench's own inputs, whose results also check the GPU's for that sequence.

Multi-GPU (torchrun, one rank per GPU): every rank runs the full per-GPU
config-2 workload on its own batch (batch x head sharding, no collective), so
total work grows with N ("weak"); time is the max over ranks and ``value`` is
the aggregate over all ranks. The line then also carries the config-5 leg:
the n = 32768 forward with its keys split across the N ranks (one NCCL
exchange), total work fixed ("strong").

The reference arm (--impl reference) times the reference's own CPU torch
path (``reference_poly_attention`` from the unmodified package copied to
baseline/_ref, run with the test-only shims for its three absent
dependencies) on all host threads, fp32, forward + backward on a bounded
sample of the config-2 workload per step (one sequence, as many of its 16
heads as keep the run within a few minutes).
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
# `value` is the aggregate over all GPUs of the job; `value_per_gpu` divides by N.
UNIT = "tokens/s (all GPUs)"
B, H, N, D = 8, 16, 4096, 64


def pass_fwd_flop(b):
    """Algorithmic FLOPs of one causal pass forward: 2 GEMMs of 2*n*n*d/2 per (b, h)."""
    return 2 * 2 * (N * N / 2) * D * b * H


# DRAM bytes per launch per batch element, from the ncu captures summarised in
# profiles/ (batch-1 case; traffic scales with batch: every (b, h) reads its own
# q/k/v once). pass_fwd_tc2: read 25.2 MB; pass_bwd_tc: read 51.1-51.3 MB, write 0.4-0.5 MB.
TRAFFIC_PER_BATCH = {"pass1_fwd": 25.23e6, "pass2_fwd": 25.50e6, "pass2_bwd": 51.88e6, "pass1_bwd": 51.47e6}


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

    def _uuid(self):
        import torch
        return "GPU-" + str(torch.cuda.get_device_properties(self.index).uuid)

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(self._uuid())
        except Exception:
            pynvml.nvmlShutdown()   # init succeeded: release it before falling back
            raise

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
            # nvidia-smi numbers GPUs in PCI order, ignoring CUDA_VISIBLE_DEVICES: select by UUID
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self._uuid()}", f"--query-gpu={self.Q}",
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
    """One forward + backward of both passes through the library's pass API.
    Returns (out, dq1, dq2, dq3, dv3)."""
    if ev is not None:
        ev[0].record()
    msg, lse23 = P.pass_fwd(q2, q3, v3, causal=True)
    if ev is not None:
        ev[1].record()
    out, lse12 = P.pass_fwd(q1, q2, msg, causal=True, bias=lse23)
    if ev is not None:
        ev[2].record()
    dq1, dq2, dmsg, dlse23 = P.pass_bwd(q1, q2, msg, out, lse12, do, causal=True, bias=lse23, want_dbias=True)
    if ev is not None:
        ev[3].record()
    _, dq3, dv3, _ = P.pass_bwd(q2, q3, v3, msg, lse23, dmsg, causal=True, dlse=dlse23, dq=dq2, dq_accumulate=True)
    if ev is not None:
        ev[4].record()
    return out, dq1, dq2, dq3, dv3


def timed_region(fn, steps, dev, world, local_rank):
    """K calls of fn between two CUDA events on the current stream, barrier and
    synchronize on both sides, clocks sampled during; returns (ms per call,
    max over ranks; clock summary)."""
    import torch
    import torch.distributed as dist
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        torch.cuda.synchronize()
        s.record()
        for _ in range(steps):
            fn()
        e.record()
        torch.cuda.synchronize()
    t = torch.tensor([s.elapsed_time(e) / steps], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()), clk.summary()


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

    # results of one more (untimed) step, sequence 0: checked against the
    # reference's CPU path in the cpu_baseline leg
    sample = None
    if world == 1 and not args.no_cpu:
        res = step_device(P, q1, q2, q3, v3, do)
        sample = {"inputs": [x[:1].float().cpu() for x in (q1, q2, q3, v3, do)],
                  "gpu": [x[:1].float().cpu() for x in res]}
        del res

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
        e2e = {"value": timed(e2e_streamed, streamer.join), "unit": UNIT, "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "api": f"HostStreamedOrder2.step (chunk {args.e2e_chunk})",
               "autograd_serial": {"value": timed(e2e_autograd), "unit": UNIT,
                                   "api": "flash_poly_attention + backward, copies before / after"}}
        del hosts, grads_h, streamer
    del q1, q2, q3, v3, do
    torch.cuda.empty_cache()

    decode = None if args.no_decode or rank != 0 else run_decode(args, dev)
    configs = {}
    if not args.no_configs:
        if world == 1:
            for name in ("config1", "vit", "prefill4", "chain_train_d128"):
                configs[name] = run_module_config(name, args, dev, local_rank)
                torch.cuda.empty_cache()
        # config 5: one GPU alone, or keys split across all ranks (one NCCL exchange)
        configs["longctx"] = run_longctx(args, rank, world, local_rank)
        torch.cuda.empty_cache()
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
    value = b * N * world / (ms_step * 1e-3)
    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "value_per_gpu": value / world,
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
        "frac_of_peak": step_flop / (ms_step * 1e-3) / 1e12 / burst,
        "phases_ms": dict(zip(names, phases)),
        "roofline": {"bound": "tensor", "kernel": names[dom], "achieved": achieved, "peak": burst,
                     "unit": "TFLOP/s", "frac": achieved / burst,
                     "traffic": TRAFFIC_PER_BATCH[names[dom]] * b,
                     "traffic_note": "ncu DRAM read+write bytes of a batch-1 capture x batch",
                     "peak_kind": f"{kind} bf16 burst (timed region well under a second)"},
        "e2e": e2e,
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
        "decode": decode,
        "configs": configs or None,
    }
    if world == 1 and not args.no_triton:
        line["triton_reference"] = triton_reference(args)
    if world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(sample)
    return line


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
    with ClockSampler(dev.index or 0) as clk:
        torch.cuda.synchronize()
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
    module_step = run_module_decode(args, dev, b, L0, steps) if (b, L0) == (32, 2048) else None
    return {"metric": "decode tok/s", "value": b * steps / (ms * 1e-3), "unit": "tokens/s", "steps": steps,
            "ms_per_step": ms / steps, "config": {"workload": "NPolyAttention order 3 core decode (config 4)"
                                                  if (b, L0) == (32, 2048) else "NPolyAttention order 3 core decode",
                                                  "batch": b, "heads": h, "kv_heads": g, "dim_head": d,
                                                  "cache_len": f"{L0 + 1}..{L0 + steps}"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                         "traffic": None, "peak_kind": f"{kind} copy bandwidth",
                         "bytes_note": "7 bf16 cache tensors + 2 fp32 lse caches at kv-head width per position"},
            "clocks": clk.summary(), "gpu_launches": int(_lib.launch_count() - n0), "module_step": module_step}


def run_module_decode(args, dev, b, L0, steps):
    """The same decode through the drop-in module: NPolyAttention(dim=2048,
    order=3, heads=16, kv_heads=4, dim_head=128, causal=True) prefilled with
    L0 tokens (return_cache=True), then `steps` single-token calls each
    passing back the returned cache tuple (appended in place). Includes the
    projections, q-norms and output projection of every step."""
    import torch

    import poly_attention_b200 as P
    torch.manual_seed(0)
    m = P.NPolyAttention(dim=2048, order=3, heads=16, kv_heads=4, dim_head=128, causal=True).to(dev, torch.bfloat16)
    g = torch.Generator(device=dev).manual_seed(78)
    x = torch.randn(b, L0 + steps + 3, 2048, device=dev, dtype=torch.bfloat16, generator=g)
    with torch.no_grad():
        _, cache0 = m(x[:, :L0], return_cache=True)
        c = cache0
        for i in range(3):                         # warm-up steps on a branch of the cache
            _, c = m(x[:, L0 + i:L0 + i + 1], cache=c, return_cache=True)
        _, c = m(x[:, :L0], return_cache=True)     # fresh prefill, then the timed steps
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for i in range(steps):
            _, c = m(x[:, L0 + i:L0 + i + 1], cache=c, return_cache=True)
        e.record()
        torch.cuda.synchronize()
    ms = s.elapsed_time(e) / steps
    del m, x, c, cache0
    return {"api": "NPolyAttention.forward(x_t, cache=..., return_cache=True)", "ms_per_step": ms,
            "value": b / (ms * 1e-3), "unit": "tokens/s",
            "note": "whole module step: projections, q-norms, in-place cache append, decode kernels, to_out"}


LONGCTX = (1, 16, 32768, 64)


def run_longctx(args, rank, world, local_rank):
    """Config 5: order-2 causal forward, b1 h16 n32768 d64 bf16, keys split
    across the ranks (zig-zag shards, see poly_attention_b200.distributed);
    total work fixed ("strong" scaling). At one GPU the same code runs without
    any collective."""
    import torch

    from poly_attention_b200 import _lib
    from poly_attention_b200.distributed import context_parallel_order2_fwd, zigzag_shard
    b, h, n, d = LONGCTX
    dev = torch.device("cuda", local_rank)
    g = torch.Generator(device=dev).manual_seed(5)
    full = [torch.randn(b, h, n, d, device=dev, dtype=torch.bfloat16, generator=g) for _ in range(4)]
    loc = [zigzag_shard(t, rank, world).contiguous() for t in full]
    del full
    for _ in range(args.warmup):
        context_parallel_order2_fwd(*loc)
    n0 = _lib.launch_count()
    ms, clk = timed_region(lambda: context_parallel_order2_fwd(*loc), args.steps, dev, world, local_rank)
    launches = _lib.launch_count() - n0
    del loc
    flop = 2 * 2 * 2 * (n * n / 2) * d * h * b            # two causal passes
    _, burst, _, kind = peaks()
    tf = flop / (ms * 1e-3) / 1e12
    return {"metric": "long-context order-2 fwd ms (config 5)", "value": ms, "unit": "ms", "n_gpus": world,
            "higher_is_better": False, "scaling": "strong", "dtype": "bf16", "data": "synthetic N(0,1), seeded",
            "config": {"workload": "order-2 causal fwd, keys split across GPUs", "batch": b, "heads": h,
                       "seq_len": n, "dim_head": d, "parallelism": f"cp{world} (zig-zag key split)"},
            "tflops": tf,
            "roofline": {"bound": "tensor", "achieved": tf / world, "peak": burst, "unit": "TFLOP/s per GPU",
                         "frac": tf / world / burst, "peak_kind": f"{kind} bf16 burst",
                         "flop_note": "2 causal passes x 2 GEMMs x 2 n^2 d / 2 x heads"},
            "clocks": clk, "gpu_launches_per_rank": int(launches / max(args.steps, 1))}


def run_chain_train(args, dev, local_rank):
    """Order-3 chain forward + backward at config 4's head shape (16 query /
    4 kv heads, d 128, causal, bf16), batch 8 x 2048 tokens: the training
    path of NPolyAttention at that size (not a BASELINE metric; config 4 is
    inference). Runs on the tcgen05 forward and the head_dim-128 backward."""
    import torch

    import poly_attention_b200 as P
    from poly_attention_b200 import _lib
    b, h, g, n, d = args.chain_batch, 16, 4, 2048, 128
    gen = torch.Generator(device=dev).manual_seed(9)
    mk = lambda heads: torch.randn(b, heads, n, d, device=dev, dtype=torch.bfloat16,  # noqa: E731
                                   generator=gen).requires_grad_(True)
    q1, q2, q3, k1, k2, k3, v1, v2 = mk(h), mk(g), mk(g), mk(g), mk(g), mk(g), mk(g), mk(g)
    do = torch.randn(b, h, n, d, device=dev, dtype=torch.bfloat16, generator=gen)
    leaves = (q1, q2, q3, k1, k2, k3, v1, v2)

    def step():
        for t in leaves:
            t.grad = None
        out, _, _ = P.poly_attention_chain([q1, q2, q3], [k1, k2, k3], [v1, v2], causal=True)
        out.backward(do)

    for _ in range(args.warmup):
        step()
    n0 = _lib.launch_count()
    ms, clk = timed_region(step, args.steps, dev, 1, local_rank)
    launches = _lib.launch_count() - n0
    # causal pass: 2 GEMMs x 2 n^2 d / 2; two levels at kv-head width, the last at h
    # heads; backward counts 2x the forward
    fwd = 2 * 2 * (n * n / 2) * d * b * (g + g + h)
    flop = 3 * fwd
    _, burst, _, kind = peaks()
    tf = flop / (ms * 1e-3) / 1e12
    return {"metric": "order-3 chain fwd+bwd tokens/s at config 4's head shape", "value": b * n / (ms * 1e-3),
            "unit": "tokens/s", "ms_per_step": ms, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "dtype": "bf16", "data": "synthetic N(0,1), seeded", "higher_is_better": True, "vs_baseline": None,
            "config": {"workload": "poly_attention_chain order 3, causal, fwd + bwd (training path, not a BASELINE "
                                   "config)", "batch": b, "heads": h, "kv_heads": g, "seq_len": n, "dim_head": d},
            "roofline": {"bound": "tensor", "achieved": tf, "peak": burst, "unit": "TFLOP/s", "frac": tf / burst,
                         "peak_kind": f"{kind} bf16 burst",
                         "flop_note": "3 causal passes (2 at 4 kv heads, 1 at 16) fwd, bwd counted 2x"},
            "clocks": clk, "gpu_launches_per_step": int(launches / max(args.steps, 1))}


def run_module_config(name, args, dev, local_rank):
    """Configs 1, 3 and the config-4 prefill through the drop-in modules
    (projections / norms / MLPs in PyTorch, attention cores in libpolyattn)."""
    import torch

    import poly_attention_b200 as P
    from poly_attention_b200 import _lib
    if name == "chain_train_d128":
        return run_chain_train(args, dev, local_rank)
    torch.manual_seed(0)
    sustained, burst, _, kind = peaks()
    if name == "config1":
        m = P.PolyAttention(dim=512, heads=8, dim_head=64, causal=False).to(dev)
        x = torch.randn(1, 1024, 512, device=dev)
        fn, tokens, unit = (lambda: m(x)), 1024, "tokens/s"
        flop, fl_note = 6.98e9, "core 4.295 GFLOP + projections 2.68 GFLOP"
        out = {"metric": "config 1 PolyAttention fp32 forward tokens/s", "dtype": "f32",
               "config": {"workload": "PolyAttention(dim=512, heads=8, dim_head=64) fwd, x [1, 1024, 512]"}}
        bound = "latency (one small fp32 forward; attention on 3xTF32 tensor-core passes)"
    elif name == "vit":
        m = P.PolyViT(image_size=256, patch_size=32, num_classes=1000, dim=1024, depth=6, heads=16, dim_head=64,
                      mlp_dim=2048, order=2).to(dev, torch.bfloat16)
        x = torch.randn(256, 3, 256, 256, device=dev, dtype=torch.bfloat16)
        fn, tokens, unit = (lambda: m(x)), 256, "images/s"
        flop, fl_note = 2.01e12, "whole model forward (linears 1.96e12 + attention core 5.15e10 + head)"
        out = {"metric": "config 3 PolyViT bf16 forward images/s", "dtype": "bf16",
               "config": {"workload": "PolyViT(256/32, dim 1024, depth 6, heads 16, mlp 2048) fwd, batch 256",
                          "tokens": "64 patches (the reference has no cls token)"}}
        bound = "tensor"
    else:
        m = P.NPolyAttention(dim=2048, order=3, heads=16, kv_heads=4, dim_head=128, causal=True).to(
            dev, torch.bfloat16)
        pb = args.prefill_batch
        x = torch.randn(pb, 2048, 2048, device=dev, dtype=torch.bfloat16)
        fn, tokens, unit = (lambda: m(x)), pb * 2048, "tokens/s"
        flop, fl_note = 8.25e11, "attention core only (order 3, kv-side passes at 4 kv heads); projections excluded"
        out = {"metric": "config 4 NPolyAttention order-3 GQA prefill tokens/s", "dtype": "bf16",
               "config": {"workload": "NPolyAttention(dim=2048 assumed, order 3, h16, g4, d128, causal) fwd, "
                                      "x [32, 2048, 2048]"}}
        bound = "tensor"
    with torch.no_grad():
        for _ in range(args.warmup):
            fn()
        n0 = _lib.launch_count()
        ms, clk = timed_region(fn, args.steps, dev, 1, local_rank)
        launches = _lib.launch_count() - n0
    tf = flop / (ms * 1e-3) / 1e12
    out.update({"value": tokens / (ms * 1e-3), "unit": unit, "ms_per_step": ms, "n_gpus": 1, "steps": args.steps,
                "warmup": args.warmup, "data": "synthetic N(0,1), seeded; random-init weights",
                "higher_is_better": True, "vs_baseline": None,
                "roofline": {"bound": bound, "achieved": tf, "peak": burst, "unit": "TFLOP/s", "frac": tf / burst,
                             "peak_kind": f"{kind} bf16 burst", "flop_note": fl_note},
                "clocks": clk, "gpu_launches_per_step": int(launches / max(args.steps, 1))})
    del m, x
    return out


# ---------------------------------------------------------------- references

def _reference_package():
    """The reference's own modules: the unmodified package copied to
    baseline/_ref (its pip build needs hatchling, absent offline), imported
    with the test-only shims for einx / torch-einops-utils /
    rotary-embedding-torch (tests/golden/shims: call-site patterns only)."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isfile(os.path.join(ref, "poly_attention", "poly_attention.py")):
        raise RuntimeError("baseline/_ref/poly_attention is missing (copy the reference package there)")
    for p in (os.path.join(ROOT, "tests", "golden", "shims"), ref):
        if p not in sys.path:
            sys.path.insert(0, p)
    import poly_attention.poly_attention as refmod
    return refmod


def reference_cpu_step(refmod, ins):
    """reference_poly_attention (poly_attention/poly_attention.py:48-116)
    forward + autograd backward on CPU, fp32. ins = (q1, q2, q3, v3, dout)
    [1, hs, N, D]. Returns (out, dq1, dq2, dq3, dv3)."""
    import torch
    q1, q2, q3, v3 = [x.detach().clone().requires_grad_(True) for x in ins[:4]]
    out, _, _ = refmod.reference_poly_attention(q1, q2, q2, q3, v3, causal=True)
    out.backward(ins[4])
    with torch.no_grad():
        return out.detach(), q1.grad, q2.grad, q3.grad, v3.grad


def cpu_baseline(sample):
    """The reference's torch CPU path on sequence 0 of the bench's own inputs
    (all 16 heads, fp32 upcast: bf16 matmuls on CPU are not representative),
    timed once on all host threads, and the GPU's results for that sequence
    checked against it (bf16 vs fp32: max-abs 2e-2 + rel 1e-2)."""
    import torch
    torch.set_num_threads(os.cpu_count())
    try:
        refmod = _reference_package()
    except Exception as exc:  # noqa: BLE001 - the port below stands in, labelled
        return cpu_baseline_port(f"reference package unavailable: {exc}")
    ins = sample["inputs"]
    reference_cpu_step(refmod, [x[:, :1, :256] for x in ins])      # warm-up (allocator, threads)
    t0 = time.perf_counter()
    ref = reference_cpu_step(refmod, ins)
    sec = time.perf_counter() - t0
    names = ["out", "dq1", "dq2", "dq3", "dv3"]
    parity = {}
    ok = True
    for nm, g, r in zip(names, sample["gpu"], ref):
        err = (g - r).abs()
        tol = 2e-2 + 1e-2 * r.abs()
        ok &= bool((err <= tol).all())
        parity[nm] = {"max_abs_err": float(err.max()), "max_excess_over_tol": float((err - tol).max())}
    parity["pass"] = ok
    parity["tolerance"] = "|gpu - ref| <= 2e-2 + 1e-2 |ref| elementwise, GPU bf16 vs reference fp32"
    return {"value": N / sec, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "reference",
            "sample": f"one sequence (16 heads) of the bench's inputs, seq {N}, fp32 torch CPU fwd+bwd of "
                      f"reference_poly_attention, {sec:.2f} s",
            "parity_vs_gpu": parity}


def cpu_baseline_port(why):
    """Fallback when the reference package is absent: the numpy restatement
    (oracle/poly_oracle.py, BLAS matmuls) on one (batch, head) unit."""
    import numpy as np

    from oracle import poly_oracle as O
    r = np.random.default_rng(0)
    a = [r.standard_normal((1, 1, N, D)).astype(np.float32) for _ in range(5)]
    t0 = time.perf_counter()
    O.order2_fwd(a[0], a[1], a[1], a[2], a[3], causal=True)
    O.order2_bwd(a[0], a[1], a[1], a[2], a[3], a[4], causal=True)
    sec = time.perf_counter() - t0
    return {"value": N / (sec * H), "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"one (batch, head) unit, numpy port, {sec:.2f} s ({why})"}


def triton_reference(args):
    """The reference's own Triton kernel (flash_poly_attention,
    poly_attention/flash_poly_attention.py:448-456) on the config-2 workload,
    forward + backward, timed on this GPU. Run in a child process so that any
    failure of the reference's JIT path cannot affect this process."""
    cmd = [sys.executable, os.path.abspath(__file__), "--workload", "triton_ref", "--steps", str(args.steps),
           "--warmup", str(args.warmup)]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
    except subprocess.TimeoutExpired:
        return {"unavailable": "the Triton reference did not finish within 900 s"}
    for ln in reversed(r.stdout.splitlines()):
        if ln.startswith("{"):
            return json.loads(ln)
    tail = (r.stderr or r.stdout).strip().splitlines()[-1:] or ["no output"]
    return {"unavailable": f"child exited {r.returncode}: {tail[0][:300]}"}


def run_triton_ref(args):
    import torch
    try:
        _reference_package()
        from poly_attention.flash_poly_attention import flash_poly_attention
    except Exception as exc:  # noqa: BLE001
        return {"unavailable": f"import failed: {type(exc).__name__}: {exc}"}
    dev = torch.device("cuda", 0)
    q1, q2, q3, v3, do = make_inputs(dev, 1234, B)
    ts = [x.requires_grad_(True) for x in (q1, q2, q3, v3)]

    def step():
        for t in ts:
            t.grad = None
        out = flash_poly_attention(*ts, is_causal=True)
        out.backward(do)

    t0 = time.perf_counter()
    step()                      # autotune + JIT
    torch.cuda.synchronize()
    jit_s = time.perf_counter() - t0
    for _ in range(args.warmup):
        step()
    ms, clk = timed_region(step, args.steps, dev, 1, 0)
    _, burst, _, kind = peaks()
    tf = 6 * pass_fwd_flop(B) / (ms * 1e-3) / 1e12
    return {"impl": "reference Triton kernel (flash_poly_attention) on this GPU", "value": B * N / (ms * 1e-3),
            "unit": "tokens/s", "ms_per_step": ms, "tflops": tf, "frac": tf / burst,
            "peak_kind": f"{kind} bf16 burst", "first_call_s": jit_s, "clocks": clk,
            "config": {"workload": "order-2 causal poly-attention core fwd+bwd (config 2)", "batch": B,
                       "heads": H, "seq_len": N, "dim_head": D}}


def run_reference(args, rank):
    """--impl reference: the reference's torch CPU path, all host threads,
    fp32, forward + backward of one sequence x hs heads per step (hs chosen
    from a one-head calibration so the whole run stays within a few minutes)."""
    if rank != 0:
        return None
    import torch
    torch.set_num_threads(os.cpu_count())
    common = {"metric": METRIC, "impl": "reference", "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
              "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
              "dtype": "f32", "data": "synthetic N(0,1), seeded",
              "config": {"workload": "order-2 causal poly-attention core fwd+bwd (config 2)", "global_batch": B,
                         "heads": H, "seq_len": N, "dim_head": D, "parallelism": "cpu"}}
    try:
        refmod = _reference_package()
    except Exception as exc:  # noqa: BLE001
        port = cpu_baseline_port(str(exc))
        v = port["value"]
        return {**common, "value": v, "cpu_baseline": port,
                "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    g = torch.Generator().manual_seed(1234)

    def inputs(hs):
        return [torch.randn(1, hs, N, D, generator=g) for _ in range(5)]

    reference_cpu_step(refmod, inputs(1))          # first call: allocator and thread-pool start-up
    t0 = time.perf_counter()
    reference_cpu_step(refmod, inputs(2))
    per_head = (time.perf_counter() - t0) / 2
    hs = int(max(1, min(H, 200.0 / (max(per_head, 1e-3) * (args.steps + args.warmup)))))
    ins = inputs(hs)
    for _ in range(args.warmup):
        reference_cpu_step(refmod, ins)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        reference_cpu_step(refmod, ins)
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    v = N / (sec * H / hs)          # a token needs all 16 heads
    sample = (f"one sequence x {hs} of 16 heads per step, seq {N}, fp32 torch CPU fwd+bwd of "
              f"reference_poly_attention (unmodified package in baseline/_ref)")
    return {**common, "value": v, "ms_per_step": sec * 1e3,
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "reference",
                             "sample": sample},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=B, help="per-GPU batch (smaller for profiling captures)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--no-triton", action="store_true", help="skip the reference Triton kernel leg")
    ap.add_argument("--no-configs", action="store_true", help="skip the config 1 / 3 / 4-prefill / 5 legs")
    ap.add_argument("--chain-batch", type=int, default=8, help="batch of the chain_train_d128 leg")
    ap.add_argument("--prefill-batch", type=int, default=32, help="config-4 prefill batch (32; smaller for captures)")
    ap.add_argument("--e2e-chunk", type=int, default=1, help="batch elements per streamed chunk (e2e leg)")
    ap.add_argument("--no-decode", action="store_true", help="skip the KV-cache decode leg")
    ap.add_argument("--decode-batch", type=int, default=32, help="decode leg batch (config 4: 32)")
    ap.add_argument("--decode-cache", type=int, default=2048, help="decode leg prefilled cache length (config 4: 2048)")
    ap.add_argument("--workload", choices=["train", "longctx", "config1", "vit", "prefill4", "chain_train_d128", "decode",
                                           "triton_ref"],
                    default="train", help="train: everything (the default line); the others run one leg alone")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        res = run_reference(args, rank)
    elif args.workload == "triton_ref":
        res = run_triton_ref(args) if rank == 0 else None
    else:
        import torch
        if world > 1:
            import torch.distributed as dist
            torch.cuda.set_device(local_rank)
            dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
        dev = torch.device("cuda", local_rank)
        torch.cuda.set_device(dev)
        if args.workload == "longctx":
            res = run_longctx(args, rank, world, local_rank)
            res = res if rank == 0 else None
        elif args.workload == "decode":
            res = run_decode(args, dev) if rank == 0 else None
        elif args.workload in ("config1", "vit", "prefill4", "chain_train_d128"):
            res = run_module_config(args.workload, args, dev, local_rank) if rank == 0 else None
        else:
            res = run_ours(args, rank, world, local_rank)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()

"""Benchmark: packed GEMV HBM GB/s (M=1) and packed GEMM TFLOP/s (M=4096) on B200.

Default workload (one "step"): headline config c2 at M=1 -- y[1, 8192] = x[1, 8192] @ W^T with
W an FP4 E2M1 (8192, 8192) packed matrix with per-32 E8M0 scales, bf16 x and y. Each step
reads a different one of C resident weight copies (C * 35.7 MB > 4 x 126 MB L2), so every
step streams its weights from HBM. The timed region replays a CUDA graph of exactly K
packed-GEMV launches. A secondary measurement (key "gemm") times headline config c3
(FP6 E3M2, M=4096, K=4096, N=14336, per-row fp16 scales) in TFLOP/s.

Multi-GPU (torchrun, one process per GPU): every rank runs the same per-GPU workload on its
own weights (independent matrices, no collective in the data path) -> "scaling": "weak";
value = total bytes of all ranks / max-over-ranks time.

``--impl reference`` times the CPU restatement of the reference's path (the reference
itself is tinygrad-on-DX12 Python and cannot run here) on the host cores, rank 0 only.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

L2_BYTES = 126 * 2**20
GEMV_CFG = dict(fmt="fp4_e2m1", n=8192, k=8192, block=32, scale="e8m0", xdt="bfloat16", m=1)
GEMM_CFG = dict(fmt="fp6_e3m2", n=14336, k=4096, block=4096, scale="f16row", xdt="float16", m=4096)
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of each timed kernel,
# from one ncu capture of `bench.py --profile-case gemv|gemm` (profiles/gemv_stream_c2_m1.md,
# profiles/gemm_c3_fp6.md). Refreshed whenever the kernel changes.
NCU_TRAFFIC = {"gemv": 35_714_304 + 0, "gemm": 81_690_000 + 89_330_000}


def algo_bytes(cfg) -> int:
    """Algorithmic bytes per call: packed W + scales + x read once, y written once."""
    n, k, m = cfg["n"], cfg["k"], cfg["m"]
    bits = 6 if cfg["fmt"].startswith("fp6") else 4
    w = n * k * bits // 8
    nblk = -(-k // cfg["block"])
    sbytes = n * nblk * (1 if cfg["scale"] == "e8m0" else 2)
    xb = m * k * 2
    yb = m * n * 2
    return w + sbytes + xb + yb


def algo_flops(cfg) -> int:
    return 2 * cfg["m"] * cfg["n"] * cfg["k"]


# ------------------------------------------------------------------------------------
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.file = None

    def __enter__(self):
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            self.proc.wait(timeout=10)

    def summary(self) -> dict:
        rows = []
        try:
            for line in pathlib.Path(self.file.name).read_text().splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        finally:
            os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for nm, val in zip(names, r[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ------------------------------------------------------------------------------------
def make_weights(cfg, device, copies: int, seed: int):
    """Random packed weights resident on the device (codes uniform over the format's payloads)."""
    import torch
    import tinygrad_dx12_b200 as tg

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    n, k = cfg["n"], cfg["k"]
    bits = 6 if cfg["fmt"].startswith("fp6") else 4
    nbytes = n * k * bits // 8
    ws = []
    for _ in range(copies):
        data = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device=device, generator=g)
        if cfg["scale"] == "e8m0":
            e = torch.randint(-8, -1, (n, k // cfg["block"]), device=device, generator=g)
            scales = (e + 127).to(torch.uint8).view(torch.float8_e8m0fnu)
            ws.append(tg.PackedTensor(data, cfg["fmt"], (n, k), scales, cfg["block"]))
        elif cfg["scale"] == "f16u":  # per-block fp16 ~U(0.005, 0.02)
            s = torch.rand((n, k // cfg["block"]), device=device, generator=g) * 0.015 + 0.005
            ws.append(tg.PackedTensor(data, cfg["fmt"], (n, k), s.to(torch.float16), cfg["block"]))
        else:  # per-row fp16 ~U(0.01, 0.05)
            s = torch.rand((n, 1), device=device, generator=g) * 0.04 + 0.01
            ws.append(tg.PackedTensor(data, cfg["fmt"], (n, k), s.to(torch.float16), k))
    return ws


def run_gpu_arm(args, world, rank, local):
    import torch
    import torch.distributed as dist
    import tinygrad_dx12_b200 as tg
    from tinygrad_dx12_b200 import _lib
    from tinygrad_dx12_b200.linalg import _packed_linear, linear_plan

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
            os.environ["NCCL_DEBUG"] = "WARN"  # stdout carries exactly one JSON line
        dist.init_process_group("nccl", device_id=device, timeout=__import__("datetime").timedelta(seconds=120))
    cfg = dict(GEMV_CFG)
    xdt = getattr(torch, cfg["xdt"])
    per_copy = cfg["n"] * cfg["k"] // 2
    copies = max(4, -(-4 * L2_BYTES // per_copy))
    ws = make_weights(cfg, device, copies, seed=1234 + rank)
    x = torch.randn((cfg["m"], cfg["k"]), device=device).to(xdt)
    y = torch.empty((cfg["m"], cfg["n"]), device=device, dtype=xdt)
    plan = linear_plan(ws[0], xdt, cfg["m"], xdt)
    descs = [w.desc() for w in ws]
    sflags = [w.scale_flags() for w in ws]  # B200_FLAG_SCALES_ORDINARY, as tg.matmul passes it
    fn = _lib.lib().b200_packed_linear
    xdt_code, ydt_code = _lib.DT[cfg["xdt"]], _lib.DT[cfg["xdt"]]

    # B200_FLAG_PDL: each step's kernel may start streaming its (parameter) weights while the
    # previous step finishes; it still waits for the previous kernel before reading x / writing y
    pdl = 0x100

    def launch(i, stream):
        rc = fn(ctypes.byref(descs[i % copies]), x.data_ptr(), xdt_code, cfg["m"], cfg["k"], 1, y.data_ptr(),
                ydt_code, cfg["n"], 1, pdl | sflags[i % copies], stream)
        if rc:
            raise RuntimeError(_lib.last_error())

    # warm-up (untimed) through plain launches, then capture exactly K launches in a graph
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            launch(i, stream.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(args.steps):
            launch(args.warmup + i, stream.cuda_stream)
    with torch.cuda.stream(stream):
        graph.replay()  # one untimed replay (graph upload)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        with torch.cuda.stream(stream):  # replay() launches on the current stream
            # untimed replays for ~0.3 s right before the timed one, so the timed K launches do
            # not start from the idle power state the sampler's start-up pause leaves behind;
            # the last ones are queued directly ahead of it (no idle gap)
            warm_until = time.time() + 0.3
            while time.time() < warm_until:
                for _ in range(8):
                    graph.replay()
                stream.synchronize()
            for _ in range(4):
                graph.replay()
            ev0.record(stream)
            graph.replay()
            ev1.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    bytes_step = algo_bytes(cfg)
    per_launch_s = ms / 1e3 / args.steps
    value = bytes_step * args.steps * world / (ms_max / 1e3) / 1e9

    # e2e through the public API, every step: x from pinned host memory to the device (the
    # library's staging kernel reads it over the host link), the matmul, y into pinned host memory
    # (the decode kernel stores it there itself): tg.matmul(W, x_host.T, dtype, out=y_host.T)
    xh = torch.randn((cfg["m"], cfg["k"])).to(xdt).pin_memory()
    yh = torch.empty((cfg["m"], cfg["n"]), dtype=xdt).pin_memory()
    for i in range(max(3, copies)):  # warm-up touches every weight copy once (per-weight plan cache)
        tg.matmul(ws[i % copies], xh.t(), dtype=xdt, out=yh.t())
    torch.cuda.synchronize()
    e_steps = max(10, min(args.steps, 200))
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(e_steps):
        tg.matmul(ws[i % copies], xh.t(), dtype=xdt, out=yh.t())
    e1.record()
    torch.cuda.synchronize()
    ems = torch.tensor([e0.elapsed_time(e1)], device=device)
    if world > 1:
        dist.all_reduce(ems, op=dist.ReduceOp.MAX)
    e2e_value = bytes_step * e_steps * world / (float(ems.item()) / 1e3) / 1e9

    # the same step as a decode loop runs it: recorded once per weight with tg.GraphStep (the
    # counterpart of tinygrad's TinyJit graph runner) and called every step with a new pinned host
    # token; each call copies it into the step's pinned input and replays the recorded staging
    # kernel and decode kernel, which stores y into pinned host memory
    gsteps = [tg.GraphStep(lambda x, w=w: tg.matmul(w, x.t(), dtype=xdt, out=yh.t()), xh) for w in ws]
    tokens = [torch.randn((cfg["m"], cfg["k"])).to(xdt).pin_memory() for _ in range(2)]
    g_steps = max(10, min(args.steps, 200))
    for i in range(max(3, copies)):
        gsteps[i % copies](tokens[i % 2])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record()
    for i in range(g_steps):
        gsteps[i % copies](tokens[i % 2])
    g1.record()
    torch.cuda.synchronize()
    del gsteps
    gms = torch.tensor([g0.elapsed_time(g1)], device=device)
    if world > 1:
        dist.all_reduce(gms, op=dist.ReduceOp.MAX)
    e2e_graph_value = bytes_step * g_steps * world / (float(gms.item()) / 1e3) / 1e9

    gemm = None
    if not args.no_gemm:
        gemm = run_gemm(args, device, world, rank)
    stack = None
    if not args.no_stack:
        stack = run_stack(args, device, world, rank)
    configs = None
    if not args.no_configs:
        configs = run_configs(args, device, world, rank)
    strong = None
    if not args.no_configs:
        strong = run_strong(args, device, world, rank)
    peaks = measured_peaks()
    result = None
    if rank == 0:
        achieved = bytes_step / per_launch_s / 1e9
        result = {
            "metric": "packed GEMV HBM GB/s (M=1)",
            "value": round(value, 1),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_max / args.steps, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "fp4_e2m1 x bf16 -> fp32 acc",
            "data": "synthetic (seeded random codes / E8M0 scales / N(0,1) bf16 x), random-init weights",
            "config": {"workload": "c2 FP4 E2M1 packed GEMV M=1, N=K=8192, per-32 E8M0 scales, bf16 x/y",
                       "m": cfg["m"], "n": cfg["n"], "k": cfg["k"], "kernel": plan,
                       "weight_copies": copies, "l2": "inputs larger than L2: rotating %d weight copies (%.0f MB)" % (
                           copies, copies * bytes_step / 1e6),
                       "timing": "CUDA graph of K launches, CUDA events on the launch stream; ~0.3 s of untimed replays of the same graph queued right before it (power-state ramp, no idle gap)",
                       "launch": "programmatic dependent launch (B200_FLAG_PDL): weights prefetched while the "
                                 "previous step drains; x read / y written only after it completes",
                       "parallelism": f"independent weights per GPU x{world}"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": NCU_TRAFFIC["gemv"],
                         "peak_source": peaks["source"] + " (MEASURED_PEAKS.json hbm_gbs)",
                         "algorithmic_bytes_per_launch": bytes_step},
            "e2e": {"value": round(e2e_graph_value, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": cfg["m"] * cfg["k"] * 2, "d2h_bytes_per_step": cfg["m"] * cfg["n"] * 2,
                    "path": "tinygrad_dx12_b200.GraphStep (the TinyJit counterpart) of "
                            "tg.matmul(W, x_host.T, dtype=bf16, out=y_host.T), one per weight copy, called every "
                            "step with a new pinned host token: the call copies it into the step's pinned input and "
                            "replays the library's staging kernel (x over the host link) and the decode kernel, "
                            "which stores y into pinned host memory",
                    "eager_value": round(e2e_value, 2),
                    "eager_path": "the same tg.matmul call from Python every step (two library calls)"},
            "gpu_launches": args.steps,
            "clocks": clk.summary(),
        }
        if gemm is not None:
            result["gemm"] = gemm
        if stack is not None:
            result["stack"] = stack
        if configs is not None:
            result["configs"] = configs
        if strong is not None:
            result["strong_scaling"] = strong
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


def _graph_time_ms(launch, steps: int, device) -> float:
    """Average ms per launch of a CUDA graph of `steps` launches (warm-up launches first)."""
    import torch

    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        for i in range(3):
            launch(i, stream.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(steps):
            launch(i, stream.cuda_stream)
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    del graph
    return e0.elapsed_time(e1) / steps


def run_configs(args, device, world, rank):
    """The other headline configurations, one GPU each (every rank measures its own; rank 0's
    line reports the max time over ranks): c1 INT4 M=1, c2 FP4 M=8 / 32, one c5 layer's
    projections at M=2048 and the c4 INT4 stack at M=1 (one token through 32 layers)."""
    import torch
    import torch.distributed as dist
    from tinygrad_dx12_b200 import _lib
    from tinygrad_dx12_b200 import stack as S
    from tinygrad_dx12_b200.linalg import linear_plan

    peaks = measured_peaks()
    fn = _lib.lib().b200_packed_linear
    out = {}

    def max_ms(ms):
        t = torch.tensor([ms], device=device)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def gemv_case(name, cfg, copies, steps):
        ws = make_weights(cfg, device, copies, seed=7 + rank)
        xdt = getattr(torch, cfg["xdt"])
        x = torch.randn((cfg["m"], cfg["k"]), device=device).to(xdt)
        y = torch.empty((cfg["m"], cfg["n"]), device=device, dtype=xdt)
        descs = [w.desc() for w in ws]
        sflags = [w.scale_flags() for w in ws]
        code = _lib.DT[cfg["xdt"]]
        flags = 0x100  # B200_FLAG_PDL (the decode kernels at these token counts honour it)

        def launch(i, stream):
            rc = fn(ctypes.byref(descs[i % copies]), x.data_ptr(), code, cfg["m"], cfg["k"], 1, y.data_ptr(), code,
                    cfg["n"], 1, flags | sflags[i % copies], stream)
            if rc:
                raise RuntimeError(_lib.last_error())

        ms = max_ms(_graph_time_ms(launch, steps, device))
        gbs = algo_bytes(cfg) / (ms / 1e3) / 1e9
        out[name] = {"us_per_call": round(ms * 1e3, 2), "GB/s": round(gbs, 1), "frac_of_hbm": round(gbs / peaks["hbm_gbs"], 4),
                     "kernel": linear_plan(ws[0], xdt, cfg["m"], xdt), "algorithmic_bytes": algo_bytes(cfg),
                     "l2": f"{copies} rotating weight copies (> 4 x L2)"}
        del ws

    c1 = dict(fmt="int4", n=4096, k=4096, block=32, scale="f16u", xdt="float16", m=1)
    gemv_case("c1_int4_m1", c1, copies=64, steps=max(20, min(args.steps, 200)))
    for m in (8, 32):
        gemv_case(f"c2_fp4_m{m}", dict(GEMV_CFG, m=m), copies=16, steps=max(20, min(args.steps, 100)))

    # one c5 layer's four projections (fused qkv, o, fused gate|up, down) at M=2048, bf16
    cfg5 = S.C5
    layer = {p: S.make_matrix(cfg5, 0, p, device, seed=3 + rank) for p in cfg5.proj_shapes()}
    sh = S.shard_layer(layer, cfg5, 0, 1)
    m5 = 2048
    xs = {k: torch.randn((m5, w.shape[1]), device=device).to(torch.bfloat16) for k, w in
          (("qkv", sh.qkv), ("o", sh.o), ("gu", sh.gu), ("down", sh.down))}
    ys = {k: torch.empty((m5, w.shape[0]), device=device, dtype=torch.bfloat16) for k, w in
          (("qkv", sh.qkv), ("o", sh.o), ("gu", sh.gu), ("down", sh.down))}
    ws5 = {"qkv": sh.qkv, "o": sh.o, "gu": sh.gu, "down": sh.down}
    d5 = {k: w.desc() for k, w in ws5.items()}
    bf = _lib.DT["bfloat16"]

    def launch5(i, stream):
        for k, w in ws5.items():
            rc = fn(ctypes.byref(d5[k]), xs[k].data_ptr(), bf, m5, w.shape[1], 1, ys[k].data_ptr(), bf, w.shape[0], 1,
                    w.scale_flags(), stream)
            if rc:
                raise RuntimeError(_lib.last_error())

    ms = max_ms(_graph_time_ms(launch5, 5, device))
    flops = sum(2 * m5 * w.shape[0] * w.shape[1] for w in ws5.values())
    tf = flops / (ms / 1e3) / 1e12
    out["c5_layer_m2048"] = {"ms_per_layer": round(ms, 3), "TFLOP/s": round(tf, 1),
                             "frac_of_tensor_peak": round(tf / peaks["bf16_tflops_sustained"], 4),
                             "peak": "bf16_tflops_sustained (long loop)", "kernel": linear_plan(sh.gu, torch.bfloat16, m5,
                                                                                              torch.bfloat16),
                             "flops_per_layer": flops,
                             "note": "one layer's packed weights (454 MB) are larger than the 126 MB L2, so every "
                                     "launch reads them from HBM; at 2048 tokens the layer is tensor-bound"}
    del layer, sh, ws5, xs, ys

    # c4 INT4 stack, one token through 32 layers on this GPU (no tensor parallelism)
    st = S.TPStack(S.C4, 0, 1, device=device, seed=5 + rank)
    total = S.C4.layer_weight_bytes() * S.C4.layers
    for m4 in (1, 16, 64):
        h0 = torch.randn((m4, S.C4.hidden), device=device).to(S.C4.act)
        h = h0.clone()

        def launch4(i, stream):
            h.copy_(h0)
            st.forward(h)

        ms = max_ms(_graph_time_ms(launch4, 5, device))
        out[f"c4_stack_m{m4}"] = {"ms_per_step": round(ms, 3), "tokens_per_s": round(m4 * 1e3 / ms, 1),
                                  "weight_gbs": round(total / (ms / 1e3) / 1e9, 1),
                                  "frac_of_hbm": round(total / (ms / 1e3) / 1e9 / peaks["hbm_gbs"], 4),
                                  "weight_bytes_per_step": total, "layers": S.C4.layers,
                                  "kernel": linear_plan(st.layers[0].gu, S.C4.act, m4, S.C4.act),
                                  "note": "INT4 group-128 fp16 scales; one GPU, whole stack as one CUDA graph"}
    del st
    return out


def run_strong(args, device, world, rank):
    """Strong scaling of the single-matrix configs (c1, c2 at M=1, c3 at M=4096): the one matrix
    is split column-parallel over the ranks (each rank owns N / world output rows of the same
    weights, x replicated; no collective: each rank's rows are independent outputs). Time = max
    over ranks; value = the whole matrix's algorithmic bytes (or flops) / that time."""
    import torch
    import torch.distributed as dist
    from tinygrad_dx12_b200 import _lib
    from tinygrad_dx12_b200.linalg import linear_plan

    fn = _lib.lib().b200_packed_linear
    peaks = measured_peaks()
    out = {}

    def max_ms(ms):
        t = torch.tensor([ms], device=device)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for name, base in (("c1_int4_m1", dict(fmt="int4", n=4096, k=4096, block=32, scale="f16u", xdt="float16", m=1)),
                       ("c2_fp4_m1", dict(GEMV_CFG))):
        cfg = dict(base, n=base["n"] // world)
        per_copy = cfg["n"] * cfg["k"] // 2
        copies = max(4, -(-4 * L2_BYTES // per_copy))
        ws = make_weights(cfg, device, copies, seed=21 + rank)
        xdt = getattr(torch, cfg["xdt"])
        x = torch.randn((1, cfg["k"]), device=device).to(xdt)
        y = torch.empty((1, cfg["n"]), device=device, dtype=xdt)
        descs = [w.desc() for w in ws]
        sflags = [w.scale_flags() for w in ws]
        code = _lib.DT[cfg["xdt"]]

        def launch(i, stream):
            rc = fn(ctypes.byref(descs[i % copies]), x.data_ptr(), code, 1, cfg["k"], 1, y.data_ptr(), code, cfg["n"], 1,
                    0x100 | sflags[i % copies], stream)
            if rc:
                raise RuntimeError(_lib.last_error())

        ms = max_ms(_graph_time_ms(launch, max(20, min(args.steps, 100)), device))
        total = algo_bytes(base)
        gbs = total / (ms / 1e3) / 1e9
        out[name] = {"rows_per_rank": cfg["n"], "us_per_call": round(ms * 1e3, 2), "GB/s": round(gbs, 1),
                     "per_gpu_frac_of_hbm": round(gbs / world / peaks["hbm_gbs"], 4),
                     "kernel": linear_plan(ws[0], xdt, 1, xdt), "l2": f"{copies} rotating weight copies per rank"}
        del ws
    cfg = dict(GEMM_CFG, n=GEMM_CFG["n"] // world)
    w = make_weights(cfg, device, 1, seed=31 + rank)[0]
    x = (torch.randn((cfg["m"], cfg["k"]), device=device) / 8).to(torch.float16)
    y = torch.empty((cfg["m"], cfg["n"]), device=device, dtype=torch.float16)
    d = w.desc()
    f16 = _lib.DT["float16"]

    def launch_g(i, stream):
        rc = fn(ctypes.byref(d), x.data_ptr(), f16, cfg["m"], cfg["k"], 1, y.data_ptr(), f16, cfg["n"], 1, 0, stream)
        if rc:
            raise RuntimeError(_lib.last_error())

    ms = max_ms(_graph_time_ms(launch_g, 5, device))
    tf = algo_flops(GEMM_CFG) / (ms / 1e3) / 1e12
    out["c3_fp6_gemm"] = {"rows_per_rank": cfg["n"], "ms_per_call": round(ms, 4), "TFLOP/s": round(tf, 1),
                          "per_gpu_frac_of_tensor_peak": round(tf / world / peaks["bf16_tflops_sustained"], 4),
                          "kernel": linear_plan(w, torch.float16, cfg["m"], torch.float16),
                          "l2": "weights larger than L2 at every split (44 MB / world + 34 MB of x)"}
    out["parallelism"] = f"column-parallel N/{world} of one matrix, x replicated, no collective"
    return out


def run_gemm(args, device, world, rank):
    import torch
    import torch.distributed as dist
    from tinygrad_dx12_b200 import _lib
    from tinygrad_dx12_b200.linalg import linear_plan

    cfg = dict(GEMM_CFG)
    xdt = torch.float16
    w = make_weights(cfg, device, 1, seed=99 + rank)[0]
    x = (torch.randn((cfg["m"], cfg["k"]), device=device) / 8).to(xdt)
    y = torch.empty((cfg["m"], cfg["n"]), device=device, dtype=xdt)
    plan = linear_plan(w, xdt, cfg["m"], xdt)
    d = w.desc()
    fn = _lib.lib().b200_packed_linear
    stream = torch.cuda.Stream(device)

    def launch():
        rc = fn(ctypes.byref(d), x.data_ptr(), _lib.DT["float16"], cfg["m"], cfg["k"], 1, y.data_ptr(),
                _lib.DT["float16"], cfg["n"], 1, 0, stream.cuda_stream)
        if rc:
            raise RuntimeError(_lib.last_error())

    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=device)
    steps = max(3, min(args.steps, 20))
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            launch()
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        with torch.cuda.stream(stream):
            flush.fill_(1)  # L2 flush between timed launches
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        launch()
        e1.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    ms = statistics.median(times)
    t = torch.tensor([ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    flops = algo_flops(cfg)
    tflops = flops / (ms / 1e3) / 1e12
    peaks = measured_peaks()
    return {
        "metric": "packed GEMM TFLOP/s (M=4096)",
        "value": round(tflops * world, 2),
        "unit": "TFLOP/s",
        "ms_per_call": round(ms, 4),
        "config": {"workload": "c3 FP6 E3M2 packed GEMM M=4096 K=4096 N=14336, per-row fp16 scales, fp16 x/y",
                   "kernel": plan, "l2": "flushed (256 MB write) before each timed launch", "timed_launches": steps},
        "roofline": {"bound": "tensor", "achieved": round(tflops, 2), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": round(tflops / peaks["bf16_tflops"], 4), "traffic": NCU_TRAFFIC["gemm"],
                     "peak_source": peaks["source"] + " (MEASURED_PEAKS.json bf16_tflops, dense fp16/bf16 kind)",
                     "algorithmic_flops_per_launch": flops},
    }


def run_stack(args, device, world, rank):
    """c5 70B-shaped FP4 projection stack at M=1: one token through all layers per step,
    tensor-parallel over the world (column-parallel q/k/v/gate/up, row-parallel o/down, two
    fp32 NCCL all-reduces per layer). The whole forward is one CUDA graph."""
    import torch
    import torch.distributed as dist
    from tinygrad_dx12_b200 import stack as S

    cfg = S.C5
    layers = cfg.layers if args.stack_layers is None else args.stack_layers
    ops = S.PeerOps(rows_max=8, hidden=cfg.hidden) if world > 1 else None  # fused peer-memory reduction
    st = S.TPStack(cfg, rank, world, device=device, layers=layers, seed=11, ops=ops)
    g = torch.Generator(device=device)
    g.manual_seed(5)
    h0 = torch.randn((1, cfg.hidden), device=device, generator=g).to(cfg.act)  # identical on every rank
    h = h0.clone()
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        for _ in range(2):  # eager warm-up (communicator set-up)
            h.copy_(h0)
            st.forward(h)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        h.copy_(h0)
        st.forward(h)
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup // 4)):
            graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    steps = max(3, min(args.steps, 20))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1) / steps], device=device)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    finite = bool(torch.isfinite(h.float()).all().item())
    del graph  # released before the process group
    torch.cuda.synchronize()
    if ops is not None:
        if world > 1:
            dist.barrier()  # no rank unmaps a buffer a peer may still read
        ops.close()
    total = cfg.layer_weight_bytes() * layers
    peaks = measured_peaks()
    per_gpu = st.weight_bytes() / (ms / 1e3) / 1e9
    return {
        "workload": f"c5 70B-shaped FP4 E2M1 stack (per-32 E8M0), M=1 bf16, {layers} layers, tensor-parallel x{world}",
        "ms_per_token": round(ms, 4), "tokens_per_s": round(1e3 / ms, 2),
        "weight_bytes_per_token": total, "weight_gbs": round(total / (ms / 1e3) / 1e9, 1),
        "per_gpu_weight_gbs": round(per_gpu, 1), "per_gpu_frac_of_hbm": round(per_gpu / peaks["hbm_gbs"], 4),
        "allreduces_per_token": 2 * layers if world > 1 else 0, "kernels_per_token": layers * 6 + 1,
        "allreduce": "fused one-shot peer-memory reduction + residual + RMS norm (b200_peer_allreduce_add_rmsnorm)"
                     if world > 1 else "none",
        "timing": "CUDA graph of one forward (all layers), CUDA events, max over ranks",
        "output_finite": finite,
    }


# ------------------------------------------------------------------------------------
def cpu_port_run(cfg, nthreads: int, budget_s: float, seed: int = 0):
    """Time the oracle's C restatement of the reference path on this host's cores."""
    from oracle import build as obuild
    from oracle import packed_ref as ref

    clib = obuild.load()
    rng = np.random.default_rng(seed)
    spec = ref.make_packed(rng, cfg["fmt"], cfg["n"], cfg["k"], cfg["block"], cfg["scale"])
    sc = ref.e8m0_bytes(spec.scales) if cfg["scale"] == "e8m0" else spec.scales
    sdt = 16 if cfg["scale"] == "e8m0" else 12
    x = rng.standard_normal((cfg["m"], cfg["k"])).astype(np.float32)
    xs = x.astype(ref.BF16) if cfg["xdt"] == "bfloat16" else x.astype(np.float16)
    xdt = 13 if cfg["xdt"] == "bfloat16" else 12
    y = np.empty((cfg["m"], cfg["n"]), np.float32)
    P = ctypes.c_void_p

    def once():
        rc = clib.oref_linear(spec.data.ctypes.data_as(P), spec.data.size, {"int4": 0, "uint4": 1, "fp4_e2m1": 2,
                              "fp6_e2m3": 3, "fp6_e3m2": 4}[cfg["fmt"]], cfg["n"], cfg["k"], sc.ctypes.data_as(P), sdt,
                              spec.block_size, np.ascontiguousarray(xs).ctypes.data_as(P), xdt, cfg["m"],
                              y.ctypes.data_as(P), nthreads)
        assert rc == 0

    once()  # warm-up
    times = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        once()
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start >= budget_s and len(times) >= 3:
            break
    return statistics.median(times), len(times)


def cpu_baseline(nthreads: int, budget_s: float) -> dict:
    cfg = dict(GEMV_CFG)
    sec, reps = cpu_port_run(cfg, nthreads, budget_s)
    return {"value": round(algo_bytes(cfg) / sec / 1e9, 3), "unit": "GB/s", "cores": nthreads, "kind": "port",
            "sample": f"{reps} full c2 M=1 calls (8192x8192 FP4, E8M0 scales, bf16 x), median "
                      f"{sec * 1e3:.1f} ms/call; oracle/cpu_ref.c decode-to-fp32 row + fp32 dot, OpenMP"}


def cpu_configs(nthreads: int, budget_s: float) -> dict:
    """The reference's CPU path timed for every benchmark config on this host's cores, two ways:

    * "port": oracle/cpu_ref.c (the C restatement: decode each weight row to fp32, fp32 dot
      products; OpenMP over rows, `nthreads` threads);
    * "numpy": the reference's CPU branch as written (codegen/linalg.py:169-174): decode the
      packed matrix to a materialised fp32 tensor (the `.contiguous()` at :172) with the numpy
      restatement, then x @ W^T through numpy's BLAS sgemm. Timed on the first 1024 weight rows
      and scaled by rows / 1024 (decode and sgemm are both linear in the rows).

    Samples are bounded so the whole leg takes a minute or two: c3 at M = 64 of its 4096 tokens,
    one layer of the c4 / c5 stacks at M=1 (per-layer figures times the layer count). Values are
    in each config's own metric (GB/s of algorithmic bytes for the decode shapes, TFLOP/s for c3).
    """
    from oracle import build as obuild
    from oracle import packed_ref as ref

    clib = obuild.load()
    P = ctypes.c_void_p
    fmt_code = {"int4": 0, "uint4": 1, "fp4_e2m1": 2, "fp6_e2m3": 3, "fp6_e3m2": 4}
    out = {}
    t_leg = time.perf_counter()

    def timed(fn, reps_budget):
        fn()  # warm-up
        times, t0 = [], time.perf_counter()
        while True:
            a = time.perf_counter()
            fn()
            times.append(time.perf_counter() - a)
            if time.perf_counter() - t0 >= reps_budget and len(times) >= 2:
                break
        return statistics.median(times), len(times)

    def both(name, spec, m, xdt, per):
        rng = np.random.default_rng(1)
        x = rng.standard_normal((m, spec.shape[1])).astype(np.float32)
        xs = x.astype(ref.BF16) if xdt == "bfloat16" else x.astype(np.float16)
        sdt = 16 if spec.scale_dtype == "float32" else 12
        sc = ref.e8m0_bytes(spec.scales) if sdt == 16 else spec.scales
        y = np.empty((m, spec.shape[0]), np.float32)

        def port():
            rc = clib.oref_linear(spec.data.ctypes.data_as(P), spec.data.size, fmt_code[spec.format], spec.shape[0],
                                  spec.shape[1], sc.ctypes.data_as(P), sdt, spec.block_size,
                                  np.ascontiguousarray(xs).ctypes.data_as(P), 13 if xdt == "bfloat16" else 12, m,
                                  y.ctypes.data_as(P), nthreads)
            assert rc == 0

        rows = min(1024, spec.shape[0])
        rb = spec.shape[1] * ref.FORMATS[spec.format][0] // 8
        part = ref.PackedSpec(spec.data[:rows * rb], spec.format, (rows, spec.shape[1]), spec.scales[:rows],
                              spec.block_size, spec.scale_dtype)

        def numpy_path():
            ref.packed_linear_ref(part, xs.astype(np.float32))

        tp, np_ = timed(port, budget_s / 24)
        tn, nn = timed(numpy_path, budget_s / 48)
        tn *= spec.shape[0] / rows
        out[name] = {"port": per(tp), "numpy": per(tn), "port_s_per_call": round(tp, 4),
                     "numpy_s_per_call": round(tn, 4), "calls": [np_, nn]}

    gb = lambda nbytes: (lambda sec: round(nbytes / sec / 1e9, 3))  # noqa: E731
    c1 = ref.make_packed(np.random.default_rng(0), "int4", 4096, 4096, 32, "f16u")
    both("c1_int4_m1", c1, 1, "float16", gb(algo_bytes(dict(fmt="int4", n=4096, k=4096, block=32, scale="f16u", m=1))))
    c2 = ref.make_packed(np.random.default_rng(0), "fp4_e2m1", 8192, 8192, 32, "e8m0")
    for m in (1, 8, 32):
        both(f"c2_fp4_m{m}", c2, m, "bfloat16", gb(algo_bytes(dict(GEMV_CFG, m=m))))
    del c2
    c3 = ref.make_packed(np.random.default_rng(0), "fp6_e3m2", 14336, 4096, 4096, "f16row")
    m3 = 64
    both("c3_fp6_gemm", c3, m3, "float16", lambda sec: round(2 * m3 * 14336 * 4096 / sec / 1e12, 5))
    out["c3_fp6_gemm"]["sample"] = f"M={m3} of 4096 tokens (TFLOP/s of the sample; time is linear in M here)"
    del c3
    for name, cfg in (("c4_stack_m1", "C4"), ("c5_stack_m1", "C5")):
        from tinygrad_dx12_b200 import stack as S
        sc_ = getattr(S, cfg)
        sh = sc_.proj_shapes()
        layer_bytes = sc_.layer_weight_bytes()
        tp = tn = 0.0
        for proj, (n, k) in sh.items():
            kind = "e8m0" if sc_.scale == "e8m0" else "f16u"
            spec = ref.make_packed(np.random.default_rng(hash(proj) & 0xFFFF), sc_.fmt, n, k, sc_.block, kind)
            both(f"_{name}_{proj}", spec, 1, "bfloat16" if sc_.scale == "e8m0" else "float16", lambda sec: sec)
            tp += out[f"_{name}_{proj}"]["port_s_per_call"]
            tn += out[f"_{name}_{proj}"]["numpy_s_per_call"]
            del out[f"_{name}_{proj}"], spec
        out[name] = {"port": round(layer_bytes / tp / 1e9, 3), "numpy": round(layer_bytes / tn / 1e9, 3),
                     "port_ms_per_token": round(tp * sc_.layers * 1e3, 1),
                     "numpy_ms_per_token": round(tn * sc_.layers * 1e3, 1),
                     "sample": f"one layer's seven projections at M=1, times {sc_.layers} layers"}
    out["unit"] = "GB/s of algorithmic bytes (c3: TFLOP/s)"
    out["cores"] = nthreads
    out["leg_s"] = round(time.perf_counter() - t_leg, 1)
    return out


def profile_case(case: str, launches: int):
    """Small untimed workload for ncu captures: `launches` plain b200_packed_linear calls.

    gemv: c2 M=1 over 4 resident weight copies (143 MB > L2); skinny: the same at M=8;
    gemm: c3 M=4096 (one weight); mx: the c5 gate|up projection at TP=1 (57344 x 8192 FP4,
    E8M0, M=1; the automatic path takes the block-scaled tcgen05 kernel there), 2 copies.
    Nothing is timed; the process only has to exit 0 so the same command line can be profiled.
    """
    import torch
    from tinygrad_dx12_b200 import _lib

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    cfg = dict(GEMV_CFG if case in ("gemv", "skinny", "mx") else GEMM_CFG)
    if case == "skinny":
        cfg["m"] = 8
    if case == "mx":
        cfg["n"] = 57344
    xdt = getattr(torch, cfg["xdt"])
    ws = make_weights(cfg, device, 1 if case == "gemm" else 2 if case == "mx" else 4, seed=0)
    x = (torch.randn((cfg["m"], cfg["k"]), device=device) / 8).to(xdt)
    y = torch.empty((cfg["m"], cfg["n"]), device=device, dtype=xdt)
    code = _lib.DT[cfg["xdt"]]
    fn = _lib.lib().b200_packed_linear
    for i in range(launches):
        d = ws[i % len(ws)].desc()
        rc = fn(ctypes.byref(d), x.data_ptr(), code, cfg["m"], cfg["k"], 1, y.data_ptr(), code, cfg["n"], 1,
                ws[i % len(ws)].scale_flags(), None)
        if rc:
            raise RuntimeError(_lib.last_error())
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": case, "launches": launches, "ok": True}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-gemm", action="store_true")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline leg")
    ap.add_argument("--no-stack", action="store_true", help="skip the c5 layer-stack leg")
    ap.add_argument("--no-configs", action="store_true", help="skip the c1 / c2 M=8,32 / c5 M=2048 / c4 legs")
    ap.add_argument("--stack-layers", type=int, default=None, help="layers of the c5 stack leg (default: all 80)")
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    ap.add_argument("--profile-case", choices=["gemv", "skinny", "gemm", "mx"], default=None,
                    help="run a small untimed workload for ncu and exit")
    ap.add_argument("--launches", type=int, default=6, help="launches of --profile-case")
    args = ap.parse_args()
    if args.profile_case:
        profile_case(args.profile_case, args.launches)
        return
    args.warmup = max(3, args.warmup)
    world, rank, local = dist_env()
    nthreads = os.cpu_count() or 1

    if args.impl == "reference":
        if rank != 0:
            return
        cfg = dict(GEMV_CFG)
        per_step = []
        for _ in range(args.warmup):
            cpu_port_run(cfg, nthreads, 0.0)
        for _ in range(args.steps):
            sec, _ = cpu_port_run(cfg, nthreads, 0.0)
            per_step.append(sec)
        tot = sum(per_step)
        value = algo_bytes(cfg) * args.steps / tot / 1e9
        print(json.dumps({
            "impl": "reference", "metric": "packed GEMV HBM GB/s (M=1)", "value": round(value, 3), "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(tot / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp4_e2m1 x bf16 -> fp32 acc", "data": "synthetic",
            "config": {"workload": "c2 FP4 E2M1 packed GEMV M=1, N=K=8192, per-32 E8M0 scales, bf16 x/y",
                       "note": "the reference runs this path through tinygrad's CPU device; tinygrad is not "
                               "installable here (no network, Python 3.14 syntax), so the timed code is the CPU "
                               "restatement oracle/cpu_ref.c of the same arithmetic"},
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": nthreads, "kind": "port",
                             "sample": f"{args.steps} full c2 M=1 calls"},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }))
        return

    res = run_gpu_arm(args, world, rank, local)
    if rank == 0 and res is not None:
        if not args.no_cpu and world == 1:
            res["cpu_baseline"] = cpu_baseline(nthreads, args.cpu_budget)
            res["cpu_configs"] = cpu_configs(nthreads, args.cpu_budget)
        print(json.dumps(res))


if __name__ == "__main__":
    main()

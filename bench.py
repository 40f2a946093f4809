"""Benchmark of the Lngram v2 memory lookup on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload sb_prefill]
    python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...   (N > 1)

Workload ``sb_prefill`` (the metric's configuration): one SB memory layer
forward over h [32, 2048, 1024] bf16 per GPU, R = 184 routes, 4-bit codes, order 3, table
[753,664 x 136] bf16, fp32 router [736, 1024], folded readout in bf16.  A step is one
``LngramMemory.forward`` over the whole batch (router -> codes -> gather + sink attention ->
output projection -> conv).  Synthetic seeded inputs; inputs (table 205 MB, h + h_norm 268 MB,
two alternating input sets) are larger than the 126 MB L2.  N GPUs run independent replicas
(weak scaling, no collective on the data path); the job time is the max over ranks.

``--impl reference`` times the reference algorithm's CPU restatement (the numpy oracle, all host
threads) on a bounded sample of the same workload and prints the same metric.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "memory-lookup positions/sec + HBM GB/s % of peak at 1/2/4/8 B200; draft tokens/sec"
SB = dict(B=32, T=2048, d=1024, routes=184, bits=4, ngrams=(3,), mem_dim=136, q_heads=16, kv_heads=4, head_dim=64)
# kernels of this library launched by one lng_memory_forward: router, rms(h), qa GEMM, gather+attention,
# output GEMM, rms(mixed), conv finish
LAUNCHES_PER_FORWARD = 7
L2_BYTES = 126 * 1024 * 1024


def peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock / throttle-reason sampling (every 200 ms) during the timed region, through NVML in a
    background thread (the fields of ``nvidia-smi --query-gpu=clocks.sm,clocks.max.sm,
    clocks_event_reasons.*``).  A separate nvidia-smi process was measured to stall this process's
    CUDA launches, so it is only the fallback when NVML cannot be loaded."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, index: int, period_s: float = 0.2):
        self.index, self.period = index, period_s
        self.rows: list = []
        self.stop = threading.Event()
        self.t = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            uuid = torch.cuda.get_device_properties(self.index).uuid
            handle = None
            for i in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(i)
                u = pynvml.nvmlDeviceGetUUID(h)
                u = u.decode() if isinstance(u, bytes) else u
                if str(uuid) in u:
                    handle = h
            if handle is None:
                handle = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.nvml, self.handle = pynvml, handle
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        except Exception as exc:  # NVML unavailable: leave the record empty and say why
            self.error = f"{type(exc).__name__}: {exc}"
        return self

    def _run(self):
        nv = self.nvml
        while not self.stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.rows.append((sm, rs))
            except Exception:
                pass
            self.stop.wait(self.period)

    def __exit__(self, *exc):
        self.stop.set()
        if self.t is not None:
            self.t.join(timeout=5)

    def summary(self) -> dict:
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"],
                    "error": getattr(self, "error", None)}
        nv = self.nvml
        reasons = sorted({name for _, rs in self.rows for name, const in self.REASONS if rs & getattr(nv, const)})
        return {"sm_mhz": statistics.median(float(s) for s, _ in self.rows), "sm_max_mhz": float(self.max_mhz),
                "reasons": reasons, "samples": len(self.rows), "source": "nvml"}


# --------------------------------------------------------------------------- distributed plumbing
def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world <= 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# --------------------------------------------------------------------------- synthetic SB layer
def build_sb(pkg, dev, seed: int = 0):
    c = SB
    mem = pkg.LngramMemory(c["d"], {"routes": c["routes"], "mem_dim": c["mem_dim"], "kv_heads": c["kv_heads"],
                                    "q_heads": c["q_heads"], "head_dim": c["head_dim"], "ngrams": list(c["ngrams"]),
                                    "bits_per_route": c["bits"]}, norm_eps=1e-5, device=dev,
                           dtype=torch.bfloat16).eval()
    g = torch.Generator(device=dev).manual_seed(seed + 2)
    with torch.no_grad():
        m = mem.module
        for t in m.tables.values():
            t.weight.copy_((torch.randn(t.weight.shape, device=dev, generator=g) * 0.02).to(torch.bfloat16))
        for name, std in (("readout_q_proj", 0.02), ("readout_kv_proj", 0.02), ("readout_o_proj", 0.006)):
            w = getattr(m, name).weight
            w.copy_((torch.randn(w.shape, device=dev, generator=g) * std).to(w.dtype))
        m.short_conv.conv.weight.copy_((torch.randn(m.short_conv.conv.weight.shape, device=dev, generator=g) * 0.2)
                                       .to(torch.bfloat16))
        mem.router.weight.copy_(torch.randn(mem.router.weight.shape, device=dev, generator=g) * 0.02)
    return mem


def sb_inputs(dev, seed: int):
    g = torch.Generator(device=dev).manual_seed(seed)
    h = torch.randn(SB["B"], SB["T"], SB["d"], device=dev, generator=g).to(torch.bfloat16)
    hf = h.float()
    hn = (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-5)).to(torch.bfloat16)
    return h, hn


def attend_bytes_per_position() -> int:
    """Algorithmic bytes of the gather + sink-attention kernel per position: the R rows of every
    order (bf16), the folded query and the output (QH x Dt bf16 each), the R codes (u8)."""
    c = SB
    dt = len(c["ngrams"]) * c["mem_dim"]
    return c["routes"] * dt * 2 + 2 * c["q_heads"] * dt * 2 + c["routes"]


def run_ours(args, rank, world, local) -> dict:
    from __graft_entry__ import load_package

    pkg = load_package()
    lib = pkg._lib
    dev = torch.device("cuda", local)
    mem = build_sb(pkg, dev, seed=0)
    inputs = [sb_inputs(dev, 100 + rank * 10 + i) for i in range(2)]
    M = SB["B"] * SB["T"]
    out = torch.empty(SB["B"], SB["T"], SB["d"], device=dev, dtype=torch.bfloat16)
    codes = torch.empty(SB["B"], SB["T"], SB["routes"], device=dev, dtype=torch.uint8)
    desc_t = mem.module.tables_desc()
    desc_r = mem.module.readout_desc(mem.router.weight)
    ws = torch.empty(lib.library().lng_memory_workspace_bytes(desc_t, desc_r, M), device=dev, dtype=torch.uint8)

    def step(i):
        h, hn = inputs[i % 2]
        mem(h, hn, codes_out=codes, out=out, workspace=ws)

    with torch.no_grad(), ClockSampler(local) as clk:
        time.sleep(0.5)  # let the sampler start before anything is timed
        for i in range(args.warmup):
            step(i)
        torch.cuda.synchronize()
        lib.device_error(clear=True)
        barrier(world)
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for i in range(args.steps):
            step(i)
        ev1.record()
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1)
        barrier(world)
        ms_max = max_over_ranks(ms, world)
        # roofline: the dominant kernel (fused gather + sink attention) timed alone, same stream
        h, hn = inputs[0]
        att = time_attend(mem, lib, h, codes, ws, args.steps)
        stages = time_stages(mem, lib, h, hn)
        # e2e through the public API with pinned host buffers
        e2e = time_e2e(mem, inputs, args, world)
        dev_err = lib.device_error(clear=True)
    if dev_err:
        raise RuntimeError(f"device error word {dev_err} after the timed region")
    pk = peaks()
    units = M * world * args.steps
    value = units / (ms_max / 1e3)
    bpp = attend_bytes_per_position()
    achieved = bpp * M / (att["ms"] / 1e3) / 1e9
    traffic = profiled_traffic("attend_mma", M)
    line = {
        "metric": METRIC, "value": value, "unit": "positions/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) hidden states, N(0,0.02) tables)",
        "config": {"workload": "sb_prefill", "batch": SB["B"], "seq_len": SB["T"], "d_model": SB["d"],
                   "routes": SB["routes"], "bits": SB["bits"], "ngrams": list(SB["ngrams"]), "mem_dim": SB["mem_dim"],
                   "readout": "q16/kv4/hd64 folded", "parallelism": f"replicas{world}",
                   "l2": "inputs larger than L2 (205 MB table, 2 x 268 MB alternating h/h_norm sets)"},
        "roofline": {"bound": "hbm", "kernel": "attend_mma_kernel (fused gather + sink attention)",
                     "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                     "peak_source": pk["source"], "traffic": traffic, "bytes_per_position": bpp,
                     "ms_per_launch": att["ms"], "launches": att["launches"]},
        "e2e": e2e,
        "stages_ms": stages,
        "gpu_launches": LAUNCHES_PER_FORWARD * args.steps,
        "clocks": clk.summary(),
    }
    return line


def time_attend(mem, lib, h, codes, ws, steps) -> dict:
    """CUDA-event time of lng_route_attend alone over the SB batch (qa from one forward)."""
    m = mem.module
    M = SB["B"] * SB["T"]
    dt = m.route_token_dim
    qd = m.readout_num_heads * dt
    qa = torch.empty(M, qd, device=h.device, dtype=torch.bfloat16)
    u = torch.empty_like(qa)
    rs = torch.empty(M, device=h.device, dtype=torch.float32)
    f = m.folded()
    s = lib.stream_ptr()
    L = lib.library()
    lib.check(L.lng_rms_rows(h.data_ptr(), lib.BF16, M, SB["d"], m.eps, rs.data_ptr(), s))
    lib.check(L.lng_gemm(h.data_ptr(), lib.BF16, SB["d"], f["w_qk"].data_ptr(), lib.BF16, SB["d"], qa.data_ptr(),
                         lib.BF16, qd, M, qd, SB["d"], None, 0, s))
    desc = m.tables_desc()

    def launch():
        lib.check(L.lng_route_attend(desc, codes.data_ptr(), lib.U8, SB["B"], SB["T"], 0, None, None, None, 0, 0,
                                     SB["routes"], m.readout_num_heads, m.eps, m.readout_sink_logit, qa.data_ptr(),
                                     rs.data_ptr(), u.data_ptr(), lib.BF16, 0, None, None, s))

    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    n = max(3, steps)
    for _ in range(n):
        launch()
    e1.record()
    torch.cuda.synchronize()
    return {"ms": e0.elapsed_time(e1) / n, "launches": n}


def time_stages(mem, lib, h, hn, reps: int = 5) -> dict:
    """CUDA-event time of each stage of one forward, called one C entry point at a time."""
    m = mem.module
    M = SB["B"] * SB["T"]
    dt = m.route_token_dim
    qd = m.readout_num_heads * dt
    dev = h.device
    L = lib.library()
    s = lib.stream_ptr()
    f = m.folded()
    split = mem.router_split()
    codes = torch.empty(M, SB["routes"], device=dev, dtype=torch.uint8)
    rs = torch.empty(M, device=dev, dtype=torch.float32)
    qa = torch.empty(M, qd, device=dev, dtype=torch.bfloat16)
    u = torch.empty_like(qa)
    mixed = torch.empty(M, SB["d"], device=dev, dtype=torch.bfloat16)
    out = torch.empty_like(mixed)
    desc_t, desc_r = m.tables_desc(), m.readout_desc()
    stages = {
        "router_tc": lambda: lib.check(L.lng_route_codes_split(hn.data_ptr(), M, SB["d"], SB["d"], split.data_ptr(),
                                                               SB["routes"], SB["bits"], codes.data_ptr(), s)),
        "rms_h": lambda: lib.check(L.lng_rms_rows(h.data_ptr(), lib.BF16, M, SB["d"], m.eps, rs.data_ptr(), s)),
        "qa_gemm_tc": lambda: lib.check(L.lng_gemm(h.data_ptr(), lib.BF16, SB["d"], f["w_qk"].data_ptr(), lib.BF16,
                                                   SB["d"], qa.data_ptr(), lib.BF16, qd, M, qd, SB["d"], None, 0, s)),
        "gather_attend": lambda: lib.check(L.lng_route_attend(desc_t, codes.data_ptr(), lib.U8, SB["B"], SB["T"], 0,
                                                              None, None, None, 0, 0, SB["routes"],
                                                              m.readout_num_heads,
                                                              m.eps, m.readout_sink_logit, qa.data_ptr(),
                                                              rs.data_ptr(), u.data_ptr(), lib.BF16, 0, None, None,
                                                              s)),
        "out_gemm_tc": lambda: lib.check(L.lng_gemm(u.data_ptr(), lib.BF16, qd, f["w_vo"].data_ptr(), lib.BF16, qd,
                                                    mixed.data_ptr(), lib.BF16, SB["d"], M, SB["d"], qd, None, 0, s)),
        "conv_finish": lambda: lib.check(L.lng_conv_finish(desc_r, mixed.data_ptr(), SB["B"], SB["T"], None, None,
                                                           out.data_ptr(), None, s)),
    }
    res = {}
    for name, fn in stages.items():
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        res[name] = round(e0.elapsed_time(e1) / reps, 4)
    return res


def time_e2e(mem, inputs, args, world) -> dict:
    """Same metric through LngramMemory.forward with pinned HOST inputs/outputs: H2D of h and
    h_norm, the forward, D2H of the output, every step."""
    dev = inputs[0][0].device
    hosts = [(h.cpu().pin_memory(), hn.cpu().pin_memory()) for h, hn in inputs]
    out_host = torch.empty(SB["B"], SB["T"], SB["d"], dtype=torch.bfloat16).pin_memory()
    hd = torch.empty_like(inputs[0][0])
    hnd = torch.empty_like(inputs[0][1])

    def step(i):
        h, hn = hosts[i % 2]
        hd.copy_(h, non_blocking=True)
        hnd.copy_(hn, non_blocking=True)
        out = mem(hd, hnd)
        out_host.copy_(out, non_blocking=True)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        step(i)
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    M = SB["B"] * SB["T"]
    return {"value": M * world * args.steps / (ms / 1e3), "unit": "positions/s",
            "h2d_bytes_per_step": 2 * hd.numel() * 2, "d2h_bytes_per_step": out_host.numel() * 2,
            "ms_per_step": ms / args.steps}


def profiled_traffic(kernel: str, units: int):
    """DRAM bytes per launch of ``kernel`` from the committed ncu summary, scaled to ``units``."""
    p = REPO / "profiles" / "traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text()).get(kernel)
    if not d:
        return None
    return d["dram_bytes"] * units / d["units"]


# --------------------------------------------------------------------------- CPU baseline / reference arm
def cpu_sb_sample(budget_s: float = 12.0) -> dict:
    """The numpy restatement of the reference forward (oracle/memory.py) on whole SB sequences
    (B = 1 x T = 2048) until ``budget_s`` seconds have passed (at least one sequence)."""
    from oracle import memory as om
    from tests.golden import cases

    c = SB
    p = cases.oracle_params("sb_slice")
    rng = np.random.default_rng(0)
    router_w = cases.memory_params("sb_slice")["router.weight"]
    n_pos = 0
    t0 = time.perf_counter()
    seqs = 0
    while True:
        h = cases.bf16_round(rng.standard_normal((1, c["T"], c["d"]), dtype=np.float32))
        x = cases.bf16_round(om.rms_norm(h, None, 1e-5))
        om.lngram_memory_forward(h, x, router_w, p)
        n_pos += c["T"]
        seqs += 1
        if time.perf_counter() - t0 >= budget_s or seqs >= 4:
            break
    dt = time.perf_counter() - t0
    threads = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    return {"value": n_pos / dt, "unit": "positions/s", "cores": threads, "kind": "port",
            "sample": f"{seqs} x (1 x 2048) SB positions through the numpy oracle forward (fp32, bf16-valued data)"}


def run_reference(args, rank, world) -> dict | None:
    if rank != 0:
        return None
    per_step = []
    base = None
    for i in range(args.warmup + args.steps):
        r = cpu_sb_sample(budget_s=0.0)  # one sequence per step
        if i >= args.warmup:
            per_step.append(r["value"])
        base = r
    value = statistics.mean(per_step)
    return {"impl": "reference", "metric": METRIC, "value": value, "unit": "positions/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": SB["T"] / value * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded)", "config": {"workload": "sb_prefill", "batch": SB["B"], "seq_len": SB["T"],
                                                     "routes": SB["routes"], "sample": "1 x 2048 positions per step"},
            "cpu_baseline": dict(base, value=value),
            "e2e": {"value": value, "unit": "positions/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("sb_prefill",), default="sb_prefill")
    ap.add_argument("--batch", type=int, default=SB["B"], help="sequences per GPU (32 = BASELINE; smaller for ncu)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args(argv)
    SB["B"] = int(args.batch)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank, world, local = dist_setup(args.gpus) if args.impl == "ours" else (
        int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), 0)
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return 0
    line = run_ours(args, rank, world, local)
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_sb_sample()
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

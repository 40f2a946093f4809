"""Benchmark of the Lngram v2 memory lookup on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload W]
    python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...   (N > 1)

Workloads (synthetic seeded inputs of the shapes the configurations name):

* ``sb_prefill`` (default; the metric's configuration): one SB memory layer forward over
  h [32, 2048, 1024] bf16 per GPU, R = 184 routes, 4-bit codes, order 3, table [753,664 x 136]
  bf16, fp32 router [736, 1024], folded readout in bf16.  A step is one ``LngramMemory.forward``
  over the whole batch (router -> codes -> gather + sink attention -> output projection -> conv).
  Inputs (table 205 MB, h + h_norm 268 MB, two alternating input sets) are larger than the 126 MB
  L2.  N GPUs run independent replicas (weak scaling, no collective on the data path).  ``e2e`` is
  the same forward through ``LngramMemory.forward_host``: pinned host h in, h_norm = attn_norm(h)
  on the device, output out, the copies overlapped with the forward by sequence groups.
  Unless ``--no-extras``, the default line also carries ``workloads``: the three other workloads
  below, each measured on its own configuration (at most 10 steps) in the same run.
* ``sdb_draft``: the SD-B drafter (182 routes, embed2 token router, vocab 32000); a step drafts
  4 greedy tokens for each of 64 sequences with 1024-token prefixes (``GpuDrafter.draft_batch``).
* ``tree_verify``: 64 sequences x a 16-node draft tree after a 1024-position context on the SB
  layer; a step is the nodes' router codes + ``tree_memory_block``.
* ``scaled`` (``route_sharded`` in ``workloads``): the 52 GB scaled table (184 routes x 2**20 rows x
  136, 5-bit codes, order 4) over h [64, 4096, 1024]; at N > 1 the routes are sharded across the
  GPUs (strong scaling), with per-phase times and the NCCL bytes of a rank.

The job time is the max over ranks of CUDA-event time.  ``--impl reference`` times the reference's
CPU implementation of the same workload on a bounded sample, on all host threads: the reference's
own C++ drafter (built from its sources) for ``sdb_draft``; for ``sb_prefill`` / ``tree_verify``
a torch-CPU restatement of the reference forward (``oracle/torch_port.py``: the reference's own
operator sequence, measured at the reference's speed with identical outputs), because the
reference's Python does not travel to the GPU box.
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
        # the block's attn_norm weight (bf16 model): h_norm = attn_norm(h) is the router input
        mem.attn_norm_weight = (1.0 + 0.1 * torch.randn(c["d"], device=dev, generator=g)).to(torch.bfloat16)
    return mem


def sb_inputs(pkg, mem, dev, seed: int):
    """h [B, T, d] bf16 N(0, 1) and h_norm = attn_norm(h) (the block norm, ``ffnmem/model.py:114``)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    h = torch.randn(SB["B"], SB["T"], SB["d"], device=dev, generator=g).to(torch.bfloat16)
    return h, pkg.rms_norm(h, mem.attn_norm_weight, 1e-5)


def layer_bytes_per_position() -> int:
    """Algorithmic bytes of the memory lookup per position: the R rows of every order (bf16) a position
    must read + its hidden state in + its output out (d bf16 each) = 54,144 B at SB."""
    c = SB
    dt = len(c["ngrams"]) * c["mem_dim"]
    return c["routes"] * dt * 2 + 2 * c["d"] * 2


def attend_bytes_per_position() -> int:
    """Bytes the gather + sink-attention kernel itself moves per position: the R rows of every order
    (bf16), the folded query and the output (QH x Dt bf16 each), the R codes (u8) = 58,936 B at SB."""
    c = SB
    dt = len(c["ngrams"]) * c["mem_dim"]
    return c["routes"] * dt * 2 + 2 * c["q_heads"] * dt * 2 + c["routes"]


def sb_config(world: int) -> dict:
    return {"workload": "sb_prefill", "batch": SB["B"], "seq_len": SB["T"], "d_model": SB["d"],
            "routes": SB["routes"], "bits": SB["bits"], "ngrams": list(SB["ngrams"]), "mem_dim": SB["mem_dim"],
            "readout": "q16/kv4/hd64", "parallelism": f"replicas{world}",
            "l2": "inputs larger than L2 (205 MB table, 2 x 268 MB alternating h/h_norm sets)"}


def sdb_config(config: dict, world: int) -> dict:
    return {"workload": "sdb_draft", "sequences": SDB["nseq"], "prefix": SDB["plen"], "gamma": SDB["gamma"],
            "vocab": int(config["vocab"]), "d_model": int(config["d_model"]), "routes": int(config["routes"]),
            "bits": int(config["bits"]), "ngrams": list(config["ngrams"]), "router": "embed2 (token only)",
            "sampling": "argmax", "parallelism": f"replicas{world}",
            "l2": "flushed between timed steps (outside the step events): a 252 MB buffer rewritten, then another 252 MB read so L2 holds clean lines"}


def tree_config(world: int) -> dict:
    from tests.golden import cases

    return {"workload": "tree_verify", "sequences": TREE["nseq"], "context": TREE["ctx"],
            "nodes": len(cases.TREE_PARENT), "parent": list(cases.TREE_PARENT), "routes": SB["routes"],
            "bits": SB["bits"], "ngrams": list(SB["ngrams"]), "mem_dim": SB["mem_dim"],
            "step": "router codes of the nodes + tree_memory_block (n-gram and conv windows along ancestors)",
            "parallelism": f"replicas{world}",
            "l2": "flushed between timed steps (outside the step events): a 252 MB buffer rewritten, then another 252 MB read so L2 holds clean lines"}


def run_ours(args, rank, world, local) -> dict:
    from __graft_entry__ import load_package

    pkg = load_package()
    lib = pkg._lib
    dev = torch.device("cuda", local)
    mem = build_sb(pkg, dev, seed=0)
    inputs = [sb_inputs(pkg, mem, dev, 100 + rank * 10 + i) for i in range(2)]
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
        launches = count_launches(lambda: step(0), fallback=LAUNCHES_PER_FORWARD)
        dev_err = lib.device_error(clear=True)
    if dev_err:
        raise RuntimeError(f"device error word {dev_err} after the timed region")
    pk = peaks()
    units = M * world * args.steps
    value = units / (ms_max / 1e3)
    bpp = layer_bytes_per_position()
    achieved = bpp * M / (att["ms"] / 1e3) / 1e9
    kio = attend_bytes_per_position()
    traffic = profiled_traffic("attend_mma", M)
    line = {
        "metric": METRIC, "value": value, "unit": "positions/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) hidden states, N(0,0.02) tables)",
        "config": sb_config(world),
        "roofline": {"bound": "hbm", "kernel": "attend_mma_kernel (fused gather + sink attention)",
                     "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                     "peak_source": pk["source"], "traffic": traffic, "bytes_per_position": bpp,
                     "bytes_rule": "R x Dt x 2 (rows) + 2 x d x 2 (hidden in, output out)",
                     "kernel_io_bytes_per_position": kio,
                     "achieved_kernel_io": kio * M / (att["ms"] / 1e3) / 1e9,
                     "ms_per_launch": att["ms"], "launches": att["launches"]},
        "e2e": e2e,
        "stages_ms": stages,
        "gpu_launches": launches["per_step"] * args.steps, "launch_count": launches,
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


E2E_GROUPS = 8


def time_e2e(mem, inputs, args, world) -> dict:
    """Same metric through the public host-memory call ``LngramMemory.forward_host``: every step copies
    that step's pinned host h in, makes h_norm = attn_norm(h) on the device, runs the forward and copies
    the output back to pinned host memory, in E2E_GROUPS groups of sequences pipelined over three streams
    (copy in / forward / copy out overlap)."""
    hosts = [h.cpu().pin_memory() for h, _ in inputs]
    out_host = torch.empty(SB["B"], SB["T"], SB["d"], dtype=torch.bfloat16).pin_memory()

    groups = int(getattr(args, "e2e_groups", E2E_GROUPS))

    def step(i):
        mem.forward_host(hosts[i % 2], norm_weight=mem.attn_norm_weight, norm_eps=1e-5, out=out_host,
                         groups=groups, synchronize=False)

    for i in range(args.warmup):
        step(i)
    mem.wait_host()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        step(i)
    mem.wait_host()                                  # the last step's copies out end the timed region
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    M = SB["B"] * SB["T"]
    return {"value": M * world * args.steps / (ms / 1e3), "unit": "positions/s",
            "h2d_bytes_per_step": hosts[0].numel() * 2, "d2h_bytes_per_step": out_host.numel() * 2,
            "ms_per_step": ms / args.steps,
            "call": f"LngramMemory.forward_host(h, norm_weight=attn_norm.weight, groups={groups}): h in, "
                    "h_norm on the device, output out; copies overlapped with the forward"}


def count_launches(fn, fallback: int) -> dict:
    """Kernels of this library (namespace ``lng::``) launched by one untimed call of ``fn``, counted from
    the CUDA activity record of ``torch.profiler``; nothing timed comes from this pass."""
    try:
        from torch.profiler import ProfilerActivity, profile

        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize()
        names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
        ours = [n for n in names if "lng::" in n]
        return {"per_step": len(ours), "other_kernels_per_step": len([n for n in names if "lng::" not in n
                                                                     and "emcpy" not in n and "emset" not in n]),
                "source": "torch.profiler kernel record of one untimed step"}
    except Exception as exc:  # profiler unavailable: the static count of the launch sites
        return {"per_step": fallback, "source": f"static count ({type(exc).__name__})"}


_CLEAN: dict = {}


def flush_l2(flush: torch.Tensor) -> None:
    """Evict L2 between timed steps: rewrite ``flush`` (larger than L2), then read a second buffer of
    the same size, so L2 holds clean lines of that buffer and the next timed step neither finds its
    own data there nor pays the write-back of the flush's dirty lines."""
    clean = _CLEAN.get(flush.device)
    if clean is None:
        clean = _CLEAN[flush.device] = (torch.zeros_like(flush), torch.empty(1, device=flush.device))
    flush.add_(1)
    torch.sum(clean[0], dim=0, keepdim=True, out=clean[1])


def timed_steps(step, steps: int, flush: torch.Tensor | None) -> float:
    """Sum of per-step CUDA-event times (ms); with ``flush``, L2 is flushed between steps
    (``flush_l2``), outside the timed events."""
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i, (a, b) in enumerate(evs):
        if flush is not None:
            flush_l2(flush)
        a.record()
        step(i)
        b.record()
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in evs)


def kernel_ms(launch, reps: int, flush: torch.Tensor | None = None) -> float:
    """Average CUDA-event duration of one call of ``launch`` (after 3 warm-up calls)."""
    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    return timed_steps(lambda i: launch(), reps, flush) / reps


def profiled_traffic(kernel: str, units: int):
    """DRAM bytes per launch of ``kernel`` from the committed ncu summary, scaled to ``units``."""
    p = REPO / "profiles" / "traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text()).get(kernel)
    if not d:
        return None
    return d["dram_bytes"] * units / d["units"]


# --------------------------------------------------------------------------- SD-B drafting
SDB = dict(nseq=64, plen=1024, gamma=4)


def sdb_bundle():
    """The SD-B drafter bundle: 182 routes, embed2 token router, order 3, 136 dims, vocab 32000,
    d = 1024, weights N(0, 0.02) (seeded; tables fp32 in the bundle, bf16 on the GPU)."""
    from tests.golden import cases

    return cases.draft_bundle("sdb")


def run_sdb(args, rank, world, local) -> dict:
    from __graft_entry__ import load_package

    pkg = load_package()
    lib = pkg._lib
    dev = torch.device("cuda", local)
    config, arrays = sdb_bundle()
    drafter = pkg.GpuDrafter(pkg.Bundle(config, arrays, {}), act_dtype=torch.bfloat16, device=dev)
    nseq, plen, gamma = SDB["nseq"], SDB["plen"], SDB["gamma"]
    V, d = int(config["vocab"]), int(config["d_model"])
    g = torch.Generator(device=dev).manual_seed(300 + rank)
    prefixes = [torch.randint(0, V, (nseq, plen), device=dev, generator=g) for _ in range(2)]
    toks = torch.empty(nseq, gamma, device=dev, dtype=torch.int64)
    flush = torch.zeros(2 * L2_BYTES // 4, device=dev, dtype=torch.float32)

    def step(i):
        drafter.draft_batch(prefixes[i % 2], gamma, out=toks)

    with torch.no_grad(), ClockSampler(local) as clk:
        time.sleep(0.5)
        for i in range(args.warmup):
            step(i)
        torch.cuda.synchronize()
        lib.device_error(clear=True)
        barrier(world)
        torch.cuda.synchronize()
        ms = timed_steps(step, args.steps, flush)
        barrier(world)
        ms_max = max_over_ranks(ms, world)
        # roofline: the draft-head logits + top-1 over the vocabulary (bf16 embedding), timed alone as
        # back-to-back lng_logits_topk calls (row split, logits_tc_topk_kernel, merge) that cycle
        # through three copies of the embedding (196 MB together, more than L2), so every call streams
        # its vocabulary from HBM with no flush in between; the three calls are replayed as a CUDA graph
        # (as the draft step runs them), so the host's per-call set-up is not in the device time
        E1 = torch.from_numpy(np.ascontiguousarray(arrays["embedding"])).to(dev).to(torch.bfloat16)
        Es = [E1] + [E1.clone() for _ in range(2)]
        hq = torch.randn(nseq, d, device=dev, generator=g)
        ids = torch.empty(nseq, 1, device=dev, dtype=torch.int64)
        vals = torch.empty(nseq, 1, device=dev, dtype=torch.float32)
        L = lib.library()
        sb = L.lng_logits_topk_scratch_bytes(nseq, d, V, 1)
        scratch = torch.empty(sb, device=dev, dtype=torch.uint8)
        s = lib.stream_ptr()
        lk_reps = 3 * max(4, args.steps)
        lk_i = [0]

        def lk_call():
            E = Es[lk_i[0] % 3]
            lk_i[0] += 1
            lib.check(L.lng_logits_topk(hq.data_ptr(), nseq, d, E.data_ptr(), lib.BF16, V, 1, ids.data_ptr(),
                                        vals.data_ptr(), None, scratch.data_ptr(), sb, s))

        for _ in range(3):
            lk_call()
        torch.cuda.synchronize()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            s = lib.stream_ptr()
            with torch.cuda.graph(graph, stream=side):
                for _ in range(3):
                    lk_call()
        torch.cuda.current_stream(dev).wait_stream(side)
        graph.replay()
        torch.cuda.synchronize()
        ev_a, ev_b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev_a.record()
        for _ in range(lk_reps // 3):
            graph.replay()
        ev_b.record()
        torch.cuda.synchronize()
        lk_ms = ev_a.elapsed_time(ev_b) / (3 * (lk_reps // 3))
        del graph, Es
        # e2e: pinned host prefix in, drafted tokens out, every step
        hosts = [p.cpu().pin_memory() for p in prefixes]
        dpre = torch.empty_like(prefixes[0])
        out_host = torch.empty(nseq, gamma, dtype=torch.int64).pin_memory()

        def e2e_step(i):
            dpre.copy_(hosts[i % 2], non_blocking=True)
            drafter.draft_batch(dpre, gamma, out=toks)
            out_host.copy_(toks, non_blocking=True)

        for i in range(args.warmup):
            e2e_step(i)
        torch.cuda.synchronize()
        barrier(world)
        e2e_ms = max_over_ranks(timed_steps(e2e_step, args.steps, flush), world)
        launches = count_launches(lambda: step(0), fallback=0)
        dev_err = lib.device_error(clear=True)
    if dev_err:
        raise RuntimeError(f"device error word {dev_err} after the timed region")
    pk = peaks()
    units = nseq * gamma * world * args.steps
    lk_bytes = V * d * 2 + nseq * d * 4 + nseq * 12
    achieved = lk_bytes / (lk_ms / 1e3) / 1e9
    return {
        "metric": METRIC, "value": units / (ms_max / 1e3), "unit": "draft tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded uniform token prefixes, N(0,0.02) weights)",
        "config": sdb_config(config, world),
        "roofline": {"bound": "hbm", "kernel": "logits_tc_topk_kernel (draft-head logits + top-1 on tcgen05, bf16 vocab; "
                               "timed as whole lng_logits_topk calls: row split + logits + merge)",
                     "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                     "peak_source": pk["source"], "traffic": profiled_traffic("logits_tc", nseq),
                     "bytes_per_launch": lk_bytes,
                     "ms_per_launch": lk_ms, "launches_per_step": gamma},
        "e2e": {"value": units / (e2e_ms / 1e3), "unit": "draft tokens/s", "h2d_bytes_per_step": nseq * plen * 8,
                "d2h_bytes_per_step": nseq * gamma * 8, "ms_per_step": e2e_ms / args.steps},
        "gpu_launches": launches["per_step"] * args.steps, "launch_count": launches,
        "clocks": clk.summary(),
    }


def cpu_sdb_sample(budget_s: float = 12.0, reps: int | None = None) -> dict:
    """The reference's C++ drafter (``drafting/cpu/drafter.cpp``, built from the reference sources into
    ``oracle/_ref``) -- or the oracle restatement when that build is absent -- on SD-B sequences: one
    drafter per host thread, each holding one committed 1024-token prefix (commit untimed), then
    ``draft(4)`` + ``truncate`` repeated in parallel on all threads for about ``budget_s`` seconds."""
    import concurrent.futures as cf

    config, arrays = sdb_bundle()
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    threads = max(1, min(threads, SDB["nseq"]))
    rng = np.random.default_rng(5)
    V, plen, gamma = int(config["vocab"]), SDB["plen"], SDB["gamma"]
    prefixes = rng.integers(0, V, size=(threads, plen))
    from oracle.build import load_reference_drafter

    ext = load_reference_drafter()
    if ext is not None:
        tensors = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in arrays.items()}
        num = {k: float(config[k]) for k in ("d_model", "vocab", "routes", "bits", "mem_dim", "kv_heads", "head_dim",
                                             "q_heads", "ssm_dim", "sketch_k", "norm_eps", "ssm_eps", "router_eps",
                                             "draft_eps", "mem_eps", "softmax_scale", "sink_logit")}
        num.update(shortlist_cap=float(config["shortlist_cap"]), router_ssm=float(config["router_kind"] == "embed2_ssm"),
                   query_ssm=float(bool(config["query_ssm"])))
        cores = [ext.Drafter(tensors, num, [int(n) for n in config["ngrams"]], 1) for _ in range(threads)]
        kind = "reference"
        draft = lambda c: c.draft(gamma, [], 1, False)  # noqa: E731
    else:
        from oracle.drafter import OracleDrafter

        cores = [OracleDrafter(config, arrays) for _ in range(threads)]
        kind = "port"
        draft = lambda c: c.draft(gamma, (), 1)  # noqa: E731
    with cf.ThreadPoolExecutor(threads) as ex:
        list(ex.map(lambda i: cores[i].commit([int(t) for t in prefixes[i]]), range(threads)))
        t0 = time.perf_counter()
        draft(cores[0])
        cores[0].truncate(plen)
        one = time.perf_counter() - t0
        n = reps if reps is not None else max(1, int(budget_s / max(one, 1e-3) / 2))

        def work(i):
            for _ in range(n):
                draft(cores[i])
                cores[i].truncate(plen)

        t0 = time.perf_counter()
        list(ex.map(work, range(threads)))
        dt = time.perf_counter() - t0
    tokens = threads * n * gamma
    return dict({"value": tokens / dt, "unit": "draft tokens/s", "cores": threads, "kind": kind,
                 "sample": f"{threads} sequences (1024-token prefixes, one drafter per thread) x {n} drafts of "
                           f"{gamma} tokens, full-vocabulary argmax"}, **host_cpu())


# --------------------------------------------------------------------------- tree verification
TREE = dict(nseq=64, ctx=1024)


def run_tree(args, rank, world, local) -> dict:
    from __graft_entry__ import load_package
    from tests.golden import cases

    pkg = load_package()
    lib = pkg._lib
    dev = torch.device("cuda", local)
    mem = build_sb(pkg, dev, seed=0)
    m = mem.module
    parent = cases.TREE_PARENT
    nseq, ctx, n = TREE["nseq"], TREE["ctx"], len(parent)
    d = SB["d"]
    cache = pkg.MemoryCache(m, nseq, ctx + n, device=dev)
    g = torch.Generator(device=dev).manual_seed(400 + rank)

    def hidden(T):
        h = torch.randn(nseq, T, d, device=dev, generator=g).to(torch.bfloat16)
        hf = h.float()
        return h, (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-5)).to(torch.bfloat16)

    with torch.no_grad():
        hc, hnc = hidden(ctx)                                   # the context, through the prefill seam
        pkg.memory_step(m, cache, hc, mem.route_codes(hnc))
        cache.length = ctx
        del hc, hnc
        nodes = [hidden(n) for _ in range(2)]
    flush = torch.zeros(2 * L2_BYTES // 4, device=dev, dtype=torch.float32)

    def step(i):
        h, hn = nodes[i % 2]
        pkg.tree_memory_block(m, cache, h, mem.route_codes(hn), parent)

    with torch.no_grad(), ClockSampler(local) as clk:
        time.sleep(0.5)
        for i in range(args.warmup):
            step(i)
        torch.cuda.synchronize()
        lib.device_error(clear=True)
        barrier(world)
        torch.cuda.synchronize()
        ms = timed_steps(step, args.steps, flush)
        barrier(world)
        ms_max = max_over_ranks(ms, world)
        # roofline: the fused gather + sink attention over the nodes' tree windows, timed alone
        att_ms, att_bytes = time_tree_attend(pkg, mem, cache, nodes[0], parent, args.steps, flush)
        hosts = [(h.cpu().pin_memory(), hn.cpu().pin_memory()) for h, hn in nodes]
        hd, hnd = torch.empty_like(nodes[0][0]), torch.empty_like(nodes[0][1])
        out_host = torch.empty(nseq, n, d, dtype=torch.bfloat16).pin_memory()

        def e2e_step(i):
            h, hn = hosts[i % 2]
            hd.copy_(h, non_blocking=True)
            hnd.copy_(hn, non_blocking=True)
            out_host.copy_(pkg.tree_memory_block(m, cache, hd, mem.route_codes(hnd), parent), non_blocking=True)

        for i in range(args.warmup):
            e2e_step(i)
        torch.cuda.synchronize()
        barrier(world)
        e2e_ms = max_over_ranks(timed_steps(e2e_step, args.steps, flush), world)
        launches = count_launches(lambda: step(0), fallback=0)
        dev_err = lib.device_error(clear=True)
    if dev_err:
        raise RuntimeError(f"device error word {dev_err} after the timed region")
    pk = peaks()
    units = nseq * n * world * args.steps
    achieved = att_bytes / (att_ms / 1e3) / 1e9
    return {
        "metric": METRIC, "value": units / (ms_max / 1e3), "unit": "tree nodes/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) hidden states, N(0,0.02) tables)",
        "config": tree_config(world),
        "roofline": {"bound": "hbm", "kernel": "attend_mma_kernel (tree windows)", "achieved": achieved,
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                     "peak_source": pk["source"], "traffic": None, "bytes_per_launch": att_bytes,
                     "ms_per_launch": att_ms},
        "e2e": {"value": units / (e2e_ms / 1e3), "unit": "tree nodes/s", "h2d_bytes_per_step": 2 * nseq * n * d * 2,
                "d2h_bytes_per_step": nseq * n * d * 2, "ms_per_step": e2e_ms / args.steps},
        "gpu_launches": launches["per_step"] * args.steps, "launch_count": launches,
        "clocks": clk.summary(),
    }


def time_tree_attend(pkg, mem, cache, node_inputs, parent, steps, flush):
    """CUDA-event time and algorithmic bytes of lng_route_attend on the tree windows of one step."""
    m = mem.module
    lib = pkg._lib
    L = lib.library()
    h, hn = node_inputs
    B, n, d = h.shape
    hist = m.route_history_length
    W = hist + 1
    plan = pkg.seams._tree_plan(parent, cache.length, B, cache.max_len, hist, m.short_conv.kernel_size,
                                m.short_conv.dilation, h.device)
    Lc = cache.length
    codes = mem.route_codes(hn)
    allc = torch.cat((cache.codes[:, Lc - plan["h0"]:Lc], codes), 1)
    ctx = (allc[:, plan["gidx"]] * plan["gok"]).reshape(B * n, W, -1).contiguous()
    f = m.folded()
    M = B * n
    qd = m.readout_num_heads * m.route_token_dim
    rs = torch.empty(M, device=h.device, dtype=torch.float32)
    s = lib.stream_ptr()
    lib.check(L.lng_rms_rows(h.data_ptr(), lib.BF16, M, d, m.eps, rs.data_ptr(), s))
    qa = m._linear(h.reshape(M, d), f["w_qk"])
    u = torch.empty(M, qd, device=h.device, dtype=torch.bfloat16)
    desc = m.tables_desc()
    seg = plan["seg"]
    ms = kernel_ms(lambda: lib.check(L.lng_route_attend(desc, ctx.data_ptr(), lib.U8, M, 0, W, None, None,
                                                        seg.data_ptr(), 0, 0, m.num_routes, m.readout_num_heads,
                                                        m.eps, m.readout_sink_logit, qa.data_ptr(), rs.data_ptr(),
                                                        u.data_ptr(), lib.BF16, 0, None, None, s)),
                   max(3, steps), flush)
    R, Dt = m.num_routes, m.route_token_dim
    nbytes = M * (R * Dt * 2 + 2 * qd * 2 + W * R + W * 4 + 4)
    return ms, nbytes


# --------------------------------------------------------------------------- scaled route-sharded
SCALED = dict(B=64, T=4096, d=1024, routes=184, bits=5, ngrams=(4,), mem_dim=136, q_heads=16, kv_heads=4, head_dim=64)
# sequence groups of the route-sharded forward: each group's reduce-scatter overlaps the next group's gather
SCALED_CHUNKS = 4
# route shards of the scaled table at N > 1: every GPU (0, the configuration: 23 routes per GPU at 8);
# the ``route_data_grid`` sub-object uses GRID_ROUTE_SHARDS (the other GPUs split the sequences)
SCALED_ROUTE_SHARDS = 0
GRID_ROUTE_SHARDS = 2


def build_scaled_shard(pkg, dev, rank: int, world: int, seed: int = 0, group=None, group_m=None):
    """This rank's block of routes of the scaled layer (tables N(0, 0.02) bf16, filled route chunk by
    route chunk from a seed per global route, so every world size holds the same table), with the
    readout weights and router rows seeded identically on every rank."""
    c = SCALED
    r0, r1 = pkg.sharded.route_bounds(c["routes"], world)[rank]
    # the table is created zeroed (no whole-table fp32 init temporary) and filled route by route below
    mem = pkg.LngramMemory(c["d"], {"routes": r1 - r0, "mem_dim": c["mem_dim"], "kv_heads": c["kv_heads"],
                                    "q_heads": c["q_heads"], "head_dim": c["head_dim"], "ngrams": list(c["ngrams"]),
                                    "bits_per_route": c["bits"], "table_init_std_scale": 0.0}, norm_eps=1e-5,
                           device=dev, dtype=torch.bfloat16).eval()
    m = mem.module
    span = (1 << c["bits"]) ** c["ngrams"][0]
    with torch.no_grad():
        w = m.tables[f"ngram_{c['ngrams'][0]}"].weight
        for r in range(r0, r1):
            g = torch.Generator(device=dev).manual_seed(seed * 100003 + 7919 + r)
            w[(r - r0) * span:(r - r0 + 1) * span].copy_(
                (torch.randn(span, c["mem_dim"], device=dev, generator=g) * 0.02).to(torch.bfloat16))
        g = torch.Generator(device=dev).manual_seed(seed + 2)
        for name, std in (("readout_q_proj", 0.02), ("readout_kv_proj", 0.02), ("readout_o_proj", 0.006)):
            p = getattr(m, name).weight
            p.copy_((torch.randn(p.shape, device=dev, generator=g) * std).to(p.dtype))
        m.short_conv.conv.weight.copy_((torch.randn(m.short_conv.conv.weight.shape, device=dev, generator=g) * 0.2)
                                       .to(torch.bfloat16))
        router = torch.randn(c["routes"] * c["bits"], c["d"], device=dev, generator=g) * 0.02
        mem.router.weight.copy_(router[r0 * c["bits"]:r1 * c["bits"]])
    return mem, pkg.RouteShardedMemory(mem, rank, world, group=group, routes_total=c["routes"], group_m=group_m)


def run_scaled(args, rank, world, local) -> dict:
    from __graft_entry__ import load_package

    pkg = load_package()
    lib = pkg._lib
    dev = torch.device("cuda", local)
    c = SCALED
    B, T, d = c["B"], c["T"], c["d"]
    # route x data grid: route_shards ranks split the routes of one layer copy and share a block of
    # sequences; the world / route_shards such groups split the batch (no exchange between groups)
    chunks = int(getattr(args, "scaled_chunks", SCALED_CHUNKS))
    rs = int(getattr(args, "route_shards", SCALED_ROUTE_SHARDS)) or world
    rs = min(rs, world)
    if world % rs:
        raise ValueError(f"--route-shards {rs} must divide the {world} GPUs")
    place = pkg.sharded.route_data_grid(world, rs, rank) if world > 1 else pkg.sharded.GridPlace(0, 1, 1)
    mem, shard = build_scaled_shard(pkg, dev, place.route_index, rs, group=place.group, group_m=place.group_m)
    g = torch.Generator(device=dev).manual_seed(500)        # the same hidden states on every rank
    h = torch.randn(B, T, d, device=dev, generator=g).to(torch.bfloat16)
    hf = h.float()
    hn = (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-5)).to(torch.bfloat16)
    del hf
    M = B * T
    Bl = B // place.data_shards                             # this rank's route group's sequences
    h, hn = h[place.data_index * Bl:(place.data_index + 1) * Bl], hn[place.data_index * Bl:(place.data_index + 1) * Bl]
    Ml = Bl * T
    if rs == 1:   # the whole table on every GPU of the group: the fused single-GPU forward
        out = torch.empty(Bl, T, d, device=dev, dtype=torch.bfloat16)
        ws = torch.empty(lib.library().lng_memory_workspace_bytes(mem.module.tables_desc(),
                                                                  mem.module.readout_desc(mem.router.weight), Ml),
                         device=dev, dtype=torch.uint8)

        def step(i):
            mem(h, hn, out=out, workspace=ws)
    else:
        def step(i):
            shard.forward(h, hn, chunks=chunks)

    with torch.no_grad(), ClockSampler(local) as clk:
        time.sleep(0.5)
        for i in range(args.warmup):
            step(i)
        torch.cuda.synchronize()
        lib.device_error(clear=True)
        barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(args.steps):
            step(i)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        barrier(world)
        ms_max = max_over_ranks(ms, world)
        # roofline: the rank's fused gather + sink attention over its routes (partial mode), alone
        m = mem.module
        Rl = shard.r1 - shard.r0
        codes = mem.route_codes(hn)
        f = m.folded()
        qd = m.readout_num_heads * m.route_token_dim
        rsq = torch.empty(Ml, device=dev, dtype=torch.float32)
        L = lib.library()
        s = lib.stream_ptr()
        lib.check(L.lng_rms_rows(h.data_ptr(), lib.BF16, Ml, d, m.eps, rsq.data_ptr(), s))
        qa = m._linear(h.reshape(Ml, d), f["w_qk"])
        u = torch.empty(Ml, m.readout_num_heads, m.route_token_dim, device=dev, dtype=torch.float32)
        ml = torch.empty(Ml, m.readout_num_heads, device=dev, dtype=torch.float32)
        ll = torch.empty_like(ml)
        desc = shard._tables_desc()
        att_ms = kernel_ms(lambda: lib.check(L.lng_route_attend(desc, codes.data_ptr(), lib.U8, Bl, T, 0, None, None,
                                                                None, 0, 0, Rl, m.readout_num_heads, m.eps,
                                                                shard.sink_logit, qa.data_ptr(), rsq.data_ptr(),
                                                                u.data_ptr(), lib.F32, 1, ml.data_ptr(),
                                                                ll.data_ptr(), s)), 3)
        del u, qa
        phases = time_scaled_phases(pkg, shard, h, hn, world) if rs > 1 else None
        launches = count_launches(lambda: step(0), fallback=0)
        dev_err = lib.device_error(clear=True)
    if dev_err:
        raise RuntimeError(f"device error word {dev_err} after the timed region")
    pk = peaks()
    Dt = m.route_token_dim
    att_bytes = Ml * (Rl * Dt * 2 + qd * 2 + m.readout_num_heads * (Dt + 2) * 4 + Rl)
    achieved = att_bytes / (att_ms / 1e3) / 1e9
    table_gb = c["routes"] * (1 << c["bits"]) ** c["ngrams"][0] * c["mem_dim"] * 2 / 1e9
    return {
        "metric": METRIC, "value": M * args.steps / (ms_max / 1e3), "unit": "positions/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) hidden states, N(0,0.02) tables)",
        "config": {"workload": "scaled", "batch": B, "seq_len": T, "d_model": d, "routes": c["routes"],
                   "routes_per_gpu": Rl, "bits": c["bits"], "ngrams": list(c["ngrams"]), "mem_dim": c["mem_dim"],
                   "table_gb": round(table_gb, 1),
                   "parallelism": (f"route {rs} x data {place.data_shards}: route-sharded groups of {rs} GPUs (NCCL "
                                   f"max all-reduce + bf16 reduce-scatter by sequence blocks, {chunks} "
                                   f"overlapped groups), sequences split across the groups")
                                  if world > 1 else "single GPU (whole table)",
                   "l2": f"inputs larger than L2 ({table_gb:.0f} GB table, 1.07 GB h + h_norm)"},
        "roofline": {"bound": "hbm", "kernel": "attend_mma_kernel (partial mode, this rank's routes)",
                     "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                     "peak_source": pk["source"], "traffic": None, "bytes_per_launch": att_bytes,
                     "ms_per_launch": att_ms},
        "gpu_launches": launches["per_step"] * args.steps, "launch_count": launches,
        "phases_ms": phases,
        "nccl_bytes_per_rank": None if rs == 1 else {
            "all_reduce_max_fp32": Ml * m.readout_num_heads * 4,
            "reduce_scatter_sent_bf16": int(Ml * m.readout_num_heads * (Dt + 1) * 2 * (rs - 1) / rs),
            "note": "per forward; each of the SCALED_CHUNKS groups moves its share"},
        "clocks": clk.summary(),
    }


def time_scaled_phases(pkg, shard, h, hn, world) -> dict:
    """Max-over-ranks CUDA-event time of each phase of the route-sharded forward on one sequence group,
    run back to back without overlap, scaled to the whole batch (the step overlaps the exchange)."""
    B, T = h.shape[:2]
    Bc = B // SCALED_CHUNKS
    hc, xc = h[:Bc], hn[:Bc]
    m = shard.full.module
    res = {}

    def tm(name, fn):
        fn()
        torch.cuda.synchronize()
        barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        out = fn()
        b.record()
        torch.cuda.synchronize()
        res[name] = round(max_over_ranks(a.elapsed_time(b), world) * SCALED_CHUNKS, 3)
        return out

    f = m.folded()
    tm("query_gemm (replicated)", lambda: m._linear(hc.reshape(Bc * T, -1), f["w_qk"]))
    if shard.packed:
        mloc, pack = tm("partial (codes + rms + query gemm + gather -> bf16 pack)", lambda: shard.partial_packed(hc, xc))
        mg = tm("all_reduce_max", lambda: pkg.sharded.all_reduce_max(mloc.clone(), shard.group_m))
        tm("rescale", lambda: shard.rescale(mloc, mg, pack))
    else:
        mloc, lloc, u = tm("partial (codes + rms + query gemm + gather)", lambda: shard.partial(hc, xc))
        mg = tm("all_reduce_max", lambda: pkg.sharded.all_reduce_max(mloc.clone(), shard.group_m or shard.group))
        pack = tm("pack", lambda: shard.pack(mloc, mg, lloc, u))
    mine = tm("reduce_scatter", lambda: pkg.sharded.reduce_scatter_rows(pack.view(Bc * T, -1), shard.group))
    tm("finish (unpack + output gemm + conv)", lambda: shard.finish(mine, Bc // shard.world, T))
    return res


# --------------------------------------------------------------------------- CPU baseline / reference arm
def host_cpu() -> dict:
    """The host's CPU model, core count and the threads torch uses (recorded beside every CPU figure)."""
    model = None
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"cpu_model": model, "os_cpu_count": os.cpu_count(), "torch_threads": torch.get_num_threads()}


def _port_threads() -> int:
    n = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    torch.set_num_threads(max(1, n))
    return torch.get_num_threads()


PORT_NOTE = ("torch-CPU restatement of the reference forward (oracle/torch_port.py): the same operator kinds "
             "as the reference's own torch forward, measured at its speed on the same cores with identical outputs")


_PORT_PARAMS: dict = {}


def _sb_port_params():
    """The SB layer's parameters for the torch-CPU port (made once per process)."""
    if "sb" not in _PORT_PARAMS:
        from oracle import torch_port as tp
        from tests.golden import cases

        _PORT_PARAMS["sb"] = tp.from_state(cases.memory_params("sb_slice"), cases.MEMORY_CASES["sb_slice"])
    return _PORT_PARAMS["sb"]


def cpu_sb_sample(budget_s: float = 12.0, max_seqs: int = 4) -> dict:
    """The reference memory-layer forward (torch CPU port) on whole SB sequences (B = 1 x T = 2048) until
    ``budget_s`` seconds have passed (at least one sequence, at most ``max_seqs``)."""
    from oracle import torch_port as tp
    from tests.golden import cases

    c = SB
    threads = _port_threads()
    p = _sb_port_params()
    w = 1.0 + 0.1 * torch.randn(c["d"], generator=torch.Generator().manual_seed(7))
    g = torch.Generator().manual_seed(0)
    n_pos, seqs = 0, 0
    t0 = time.perf_counter()
    while True:
        h = torch.randn(1, c["T"], c["d"], generator=g).to(torch.bfloat16).float()
        hn = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-5) * w       # attn_norm (fp32 model)
        tp.lngram_forward(h, hn, p)
        n_pos += c["T"]
        seqs += 1
        if time.perf_counter() - t0 >= budget_s or seqs >= max_seqs:
            break
    dt = time.perf_counter() - t0
    return dict({"value": n_pos / dt, "unit": "positions/s", "cores": threads, "kind": "port",
                 "sample": f"{seqs} x (1 x 2048) SB positions through the reference forward, fp32 ({PORT_NOTE})"},
                **host_cpu())


def cpu_tree_sample(budget_s: float = 12.0, max_seqs: int | None = None) -> dict:
    """The reference tree-verification memory block (``drafting/tree.py:178-195``, torch CPU port) with the
    SB layer: the nodes' router codes and the block for one sequence's 16-node tree after a 1024-position
    context, repeated for about ``budget_s`` seconds."""
    from oracle import torch_port as tp
    from tests.golden import cases

    threads = _port_threads()
    p = _sb_port_params()
    parent = cases.TREE_PARENT
    n, d, R = len(parent), SB["d"], SB["routes"]
    g = torch.Generator().manual_seed(1)
    hist, lp = max(SB["ngrams"]) - 1, 3 * max(SB["ngrams"])
    t0 = time.perf_counter()
    seqs = 0
    while True:
        h = torch.randn(1, n, d, generator=g).to(torch.bfloat16).float()
        x = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-5)
        history = torch.randint(0, 1 << SB["bits"], (1, hist, R), generator=g)
        conv_cache = torch.randn(1, lp, d, generator=g)
        tp.tree_block(h, x, parent, history, conv_cache, p)
        seqs += 1
        if time.perf_counter() - t0 >= budget_s or (max_seqs is not None and seqs >= max_seqs):
            break
    dt = time.perf_counter() - t0
    return dict({"value": seqs * n / dt, "unit": "tree nodes/s", "cores": threads, "kind": "port",
                 "sample": f"{seqs} x 16-node trees (1024-position context) through the reference tree block, "
                           f"fp32 ({PORT_NOTE})"}, **host_cpu())


def run_reference(args, rank, world) -> dict | None:
    """The reference algorithm on the host cores (rank 0 only), same metric / unit / config keys."""
    if rank != 0:
        return None
    wl = args.workload
    if wl == "scaled":
        return {"impl": "reference", "unavailable": "the scaled table (52 GB) has no bounded CPU sample: the "
                "reference CPU forward would have to generate and hold the whole table in host memory"}
    per_step, base = [], None
    for i in range(args.warmup + args.steps):
        if wl == "sb_prefill":
            r = cpu_sb_sample(budget_s=0.0)                 # one 2048-position sequence per step
        elif wl == "sdb_draft":
            r = cpu_sdb_sample(reps=1)                      # one draft of 4 tokens on every thread per step
        else:
            r = cpu_tree_sample(budget_s=0.0, max_seqs=1)   # one 16-node tree per step
        if i >= args.warmup:
            per_step.append(r["value"])
        base = r
    value = statistics.mean(per_step)
    units = {"sb_prefill": SB["T"], "sdb_draft": base["cores"] * SDB["gamma"], "tree_verify": 16}[wl]
    cfg = {"sb_prefill": lambda: sb_config(world), "sdb_draft": lambda: sdb_config(sdb_bundle()[0], world),
           "tree_verify": lambda: tree_config(world)}[wl]()
    return {"impl": "reference", "metric": METRIC, "value": value, "unit": base["unit"], "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": units / value * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded)", "config": cfg, "cpu_baseline": dict(base, value=value),
            "e2e": {"value": value, "unit": base["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


RUNNERS = {"sb_prefill": "run_ours", "sdb_draft": "run_sdb", "tree_verify": "run_tree", "scaled": "run_scaled"}
SUB_KEYS = ("value", "unit", "ms_per_step", "steps", "warmup", "scaling", "config", "roofline", "e2e", "cpu_baseline",
            "gpu_launches", "phases_ms", "nccl_bytes_per_rank", "clocks")


def summarize(res: dict) -> dict:
    """The keys of one workload's line that go into the default line's ``workloads`` sub-object."""
    return {k: res[k] for k in SUB_KEYS if k in res}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=tuple(RUNNERS), default="sb_prefill")
    ap.add_argument("--batch", type=int, default=SB["B"], help="sb_prefill sequences per GPU (32 = the SB configuration; "
                    "smaller for ncu)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-groups", type=int, default=E2E_GROUPS, help="sequence groups of the pipelined e2e call")
    ap.add_argument("--route-shards", type=int, default=SCALED_ROUTE_SHARDS,
                    help="scaled table at N > 1: GPUs per route-sharded group (the groups split the sequences; "
                    "0 = all N GPUs, the configuration's layout)")
    ap.add_argument("--scaled-chunks", type=int, default=SCALED_CHUNKS,
                    help="scaled table at N > 1: sequence groups pipelined through the route exchange")
    ap.add_argument("--no-extras", action="store_true", help="sb_prefill only: skip the SD-B / tree / scaled "
                    "sub-objects of the default line")
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
    line = globals()[RUNNERS[args.workload]](args, rank, world, local)
    cpu_arms = {"sb_prefill": cpu_sb_sample, "sdb_draft": cpu_sdb_sample, "tree_verify": cpu_tree_sample}
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload in cpu_arms:
        line["cpu_baseline"] = cpu_arms[args.workload]()
    if args.workload == "sb_prefill" and not args.no_extras:
        # the other parts of the metric, each on its own configuration, in the same JSON line
        sub = argparse.Namespace(**vars(args))
        sub.steps, sub.warmup = min(args.steps, 10), max(3, min(args.warmup, 3))
        line["workloads"] = {}
        runs = [("sdb_draft", "sdb_draft", None), ("tree_verify", "tree_verify", None),
                ("route_sharded", "scaled", 0)]
        if world > GRID_ROUTE_SHARDS and world % GRID_ROUTE_SHARDS == 0:
            runs.append(("route_data_grid", "scaled", GRID_ROUTE_SHARDS))
        for key, wl, shards in runs:
            torch.cuda.empty_cache()
            if shards is not None:
                sub.route_shards = shards
            res = globals()[RUNNERS[wl]](sub, rank, world, local)
            if rank == 0 and world == 1 and not args.no_cpu_baseline and wl in cpu_arms:
                res["cpu_baseline"] = cpu_arms[wl](budget_s=6.0)
            line["workloads"][key] = summarize(res)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

#!/usr/bin/env python
"""Block-scaled FP4 grouped GEMM benchmark on B200.

Default workload = BASELINE config 3, the expert-parallel MoE layer (4096
tokens, top-8 of 64 experts with Zipf(1.1) routing, N=4096, K=7168, NVFP4),
the one workload that runs at every GPU count: experts sharded over the
ranks, tokens dispatched and combined with NCCL collectives (strong
scaling).  Other configs: --config grouped (config 2: 8 groups,
M_g ~ U[64, 1024], N=4096, K=7168; replicas under torchrun), dense (config 4,
8192^3; N split over the ranks), decode (config 5, 256 groups,
M_g ~ U[1, 16], N=7168, K=2048; groups sharded by LPT), mlp (the gated
expert MLP), mx (the reference operator fp4_grouped_gemm at its campaign
point).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C]
                    [--impl ours|reference|reference-gpu]

Prints ONE JSON line on rank 0: barrier + synchronize around exactly K timed
steps after W warm-up steps, max over ranks.

  value       TFLOP/s of the public call with inputs resident in HBM
  e2e         the same call fed from pinned host buffers (H2D of the inputs
              and D2H of the output inside the timed region)
  roofline    the GEMM kernel against 4 x the measured dense bf16 peak
              (B200's dense FP4 rate is 4x its bf16 rate), or against the
              measured HBM copy bandwidth for the decode config
  cpu_baseline  the CPU oracle (dequantise + fp32 matmul, all host threads)
              on a bounded sample of the same workload, rank 0, N=1
  --impl reference      that CPU oracle alone on the same config
  --impl reference-gpu  the reference's own kernel (baseline/_ref) beside
              fp4_grouped_gemm on one B200 (config mx)
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
L2_BYTES = 126 * 1024 * 1024


# ------------------------------------------------------------------ workloads
def workload(name: str, seed: int = 0) -> dict:
    rng = np.random.default_rng(seed)
    if name == "grouped":
        ms = [int(v) for v in rng.integers(64, 1025, size=8)]
        return dict(name="grouped", desc="8 groups, M_g~U[64,1024] seed 0, N=4096, K=7168",
                    m=ms, n=4096, k=7168, w_std=1.0, bound="tensor")
    if name == "dense":
        return dict(name="dense", desc="single group M=N=K=8192", m=[8192], n=8192, k=8192,
                    w_std=1.0, bound="tensor")
    if name == "moe":
        return dict(name="moe", desc="MoE expert layer: 4096 tokens, top-8 of 64 experts "
                    "(Zipf s=1.1, seed 0), N=4096 (gate+up), K=7168, expert-parallel",
                    m=[4096 * 8], n=4096, k=7168, w_std=1.0, bound="tensor",
                    tokens=4096, experts=64, topk=8)
    if name == "mlp":
        ms = [int(v) for v in rng.integers(64, 1025, size=8)]
        return dict(name="mlp", desc="gated expert MLP, 8 experts, M_g~U[64,1024] seed 0: "
                    "gate+up N=4096 (I=2048) K=7168 with the SiLU*up epilogue, NVFP4 "
                    "quantisation of the intermediate, down N=7168 K=2048",
                    m=ms, n=2 * 2048, k=7168, inter=2048, w_std=1.0, bound="tensor")
    if name == "mx":
        return dict(name="mx", desc="the reference operator fp4_grouped_gemm (MXFP8 x MXFP4) at "
                    "its campaign point: 8 experts x 4096 rows (segments padded to 224, "
                    "M_total=34048), N=K=4096", m=[4096] * 8, n=4096, k=4096, w_std=1.0,
                    bound="tensor", ref_us=375.6)
    if name == "decode":
        ms = [int(v) for v in rng.integers(1, 17, size=256)]
        return dict(name="decode", desc="256 groups, M_g~U[1,16] seed 0, N=7168, K=2048",
                    m=ms, n=7168, k=2048, w_std=0.02, bound="hbm")
    raise SystemExit(f"unknown config {name}")


def flops(wl) -> float:
    if wl["name"] == "mlp":  # gate+up GEMM, then the down projection
        return 2.0 * sum(wl["m"]) * (wl["n"] * wl["k"] + wl["k"] * wl["inter"])
    return 2.0 * sum(wl["m"]) * wl["n"] * wl["k"]


def alg_bytes(wl) -> float:
    """Algorithmic HBM bytes of one call: read A codes+scales, B codes+scales,
    write C (bf16)."""
    n, k, G = wl["n"], wl["k"], len(wl["m"])
    sm = sum(wl["m"])
    return sm * (k / 2 + k / 16) + G * n * (k / 2 + k / 16) + sm * n * 2


def set_bytes(wl) -> float:
    return alg_bytes(wl)


# ------------------------------------------------------------------ helpers
def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"bf16": float(d["bf16_tflops"]), "bf16_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "hbm": float(d["hbm_gbs"]), "src": "measured"}
    return {"bf16": 1590.0, "bf16_sustained": 1400.0, "hbm": 6650.0, "src": "fallback"}


_SAMPLER_SRC = r"""
import json, select, sys, time
import pynvml
pynvml.nvmlInit()
h = pynvml.nvmlDeviceGetHandleByUUID(sys.argv[1])
print("ready", flush=True)
out, err = [], None
while not select.select([sys.stdin], [], [], 0)[0]:
    try:
        out.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                    pynvml.nvmlDeviceGetCurrentClocksEventReasons(h),
                    pynvml.nvmlDeviceGetPowerUsage(h)))
    except Exception as e:
        err = str(e)
        break
    time.sleep(0.0005)
print(json.dumps({"samples": out, "err": err}), flush=True)
"""


class ClockSampler:
    """SM clock, power and throttle reasons sampled through NVML (the source
    nvidia-smi reads) every ~1 ms while the timed region runs.  The sampler is
    a child process, so the timed loop's Python work cannot starve it.  The
    GPU is found by UUID, so CUDA_VISIBLE_DEVICES remapping is harmless."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))

    def __init__(self, device: int):
        self.device = device
        self.err = None
        self.nv = None
        self.max_mhz = None
        self.proc = None
        try:
            import pynvml

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            h = pynvml.nvmlDeviceGetHandleByUUID(self.uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self.nv = pynvml
        except Exception as e:  # no NVML: report why instead of clocks
            self.err = f"nvml unavailable: {e}"

    def start(self):
        if self.nv is None:
            return
        import subprocess

        self.proc = subprocess.Popen([sys.executable, "-c", _SAMPLER_SRC, self.uuid],
                                     stdin=subprocess.PIPE, stdout=subprocess.PIPE, text=True)
        if self.proc.stdout.readline().strip() != "ready":
            self.err = "clock sampler did not start"
            self.proc.kill()
            self.proc = None

    def stop(self) -> dict:
        samples = []
        if self.proc is not None:
            try:
                out, _ = self.proc.communicate(input="x", timeout=30)
                d = json.loads(out.strip().splitlines()[-1])
                samples = d["samples"]
                self.err = d["err"] or self.err
            except Exception as e:
                self.proc.kill()
                self.err = f"clock sampler failed: {e}"
        if self.nv is None or not samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "note": self.err}
        reasons = set()
        for _, bits, _ in samples:
            for name, attr in self.REASONS:
                if bits & getattr(self.nv, attr, 0):
                    reasons.add(name)
        sm = [c for c, _, _ in samples]
        return {"sm_mhz": statistics.median(sm), "sm_min_mhz": min(sm),
                "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(p for _, _, p in samples) / 1000.0,
                "source": "NVML in a child process, ~0.5 ms polling during the timed region"}


def dist_init():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return ws, rank, local


def max_over_ranks(x: float, ws: int, dev) -> float:
    if ws == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(ws: int):
    if ws > 1:
        import torch.distributed as dist

        dist.barrier()


# ------------------------------------------------------------------ inputs
def shard(wl, ws: int, rank: int) -> dict:
    """This rank's part of the workload.  grouped / mlp / mx: every rank runs
    the whole workload (independent replicas, weak scaling).  dense: the
    weight rows (output columns) split evenly, the activations replicated
    (strong scaling).  decode: whole groups placed by longest-processing-time
    on their weight bytes (strong scaling)."""
    sub = dict(wl)
    sub["groups"] = list(range(len(wl["m"])))
    sub["w_rows"] = (0, wl["n"])
    if ws == 1:
        sub["split"] = "none"
        return sub
    if wl["name"] == "dense":
        if wl["n"] % (256 * ws):
            raise SystemExit(f"N={wl['n']} does not split into {ws} slices of 256-row tiles")
        per = wl["n"] // ws
        sub["n"] = per
        sub["w_rows"] = (rank * per, (rank + 1) * per)
        sub["split"] = f"N split: weight rows [{rank * per}, {(rank + 1) * per}) of {wl['n']}"
        return sub
    if wl["name"] == "decode":
        wbytes = wl["n"] * (wl["k"] // 2 + wl["k"] // 16)   # every group's weights
        load = [0] * ws
        owner = []
        for g in sorted(range(len(wl["m"])), key=lambda g: (-wbytes, g)):
            r = min(range(ws), key=lambda r: (load[r], r))
            owner.append((g, r))
            load[r] += wbytes
        sub["groups"] = sorted(g for g, r in owner if r == rank)
        sub["m"] = [wl["m"][g] for g in sub["groups"]]
        sub["split"] = f"groups by LPT on weight bytes: {len(sub['groups'])} of {len(wl['m'])}"
        return sub
    sub["split"] = "replica"
    return sub


def make_set(wl, seed: int, dev):
    """One input set on the device: N(0,1) activations and N(0, w_std) weights,
    each quantised to NVFP4 with its own global scale by the device quantiser.
    Every group draws from its own seeded stream, so a group's data does not
    depend on how the groups are sharded; the dense split takes its rows of
    one seeded weight tensor.  The activation codes and scales of all groups
    live in one contiguous buffer (the per-group tensors are row views of it)."""
    import ratchet_b200 as rb

    n, k = wl["n"], wl["k"]
    groups = wl.get("groups", list(range(len(wl["m"]))))
    r0, r1 = wl.get("w_rows", (0, n))
    ms = list(wl["m"])
    rows = sum(ms)
    a_all = torch.empty((rows, k // 2), dtype=torch.uint8, device=dev)
    sf_all = torch.empty((rows, k // 16), dtype=torch.uint8, device=dev)
    B, BSF, alpha = [], [], []
    at = 0
    for g, m in zip(groups, ms):
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed * 100003 + 2 * g)
        x = torch.randn((m, k), generator=gen, device=dev, dtype=torch.float32)
        qa, sa, ga = rb.quantize_nvfp4(x)
        a_all[at:at + m].copy_(qa)
        sf_all[at:at + m].copy_(sa.view(torch.uint8))
        at += m
        gen.manual_seed(seed * 100003 + 2 * g + 1)
        w = torch.randn((r1 if wl["name"] == "dense" else n, k), generator=gen, device=dev,
                        dtype=torch.float32)[r0:r1 if wl["name"] == "dense" else n]
        w = w * wl["w_std"]
        qb, sb, gb = rb.quantize_nvfp4(w.contiguous())
        del x, w
        B.append(qb)
        BSF.append(sb)
        alpha.append(ga * gb)
    off = torch.zeros(len(ms) + 1, dtype=torch.int32)
    off[1:] = torch.cumsum(torch.tensor(ms, dtype=torch.int64), 0).to(torch.int32)
    return dict(a=list(a_all.split(ms)), a_sf=[t.view(torch.float8_e4m3fn) for t in sf_all.split(ms)],
                a_all=a_all, sf_all=sf_all.view(torch.float8_e4m3fn), offsets=off.to(dev),
                out=torch.empty((rows, r1 - r0 if wl["name"] == "dense" else n),
                                dtype=torch.bfloat16, device=dev),
                b=B, b_sf=BSF, alpha=torch.stack(alpha).float(), sizes=[(m, n, k) for m in ms],
                max_m=max(ms) if ms else 0)


# The public entry a step calls: "rows" = nvfp4_grouped_gemm_rows over the
# contiguous activations with device offsets (the reference operator's own
# M-grouped layout; host work independent of the group count), "list" = the
# per-group-list operator.
CALL = "rows"


def public_call(s, out=None, call=None):
    """The public operator call a step makes (CALL unless `call` is given),
    writing the set's own output buffer unless `out` is given (a serving loop
    reuses its output buffers).  Decode-shaped sets (every M_g <= 16) pass
    that bound, which selects the decode tiles."""
    import ratchet_b200 as rb

    if out is None:
        out = s["out"]
    if (call or CALL) == "rows":
        if "pack" not in s:
            s["pack"] = rb.pack_weights(s["b"], s["b_sf"])
        return rb.nvfp4_grouped_gemm_rows(s["a_all"], s["sf_all"], s["offsets"], pack=s["pack"],
                                          alpha=s["alpha"], out=out,
                                          max_group_rows=16 if s["max_m"] <= 16 else 0)
    return rb.nvfp4_grouped_gemm(s["a"], s["a_sf"], s["b"], s["b_sf"], s["sizes"], s["alpha"],
                                 out=out)


def time_value(sets, steps, warmup, dev, ws, entry=None):
    """Device time per step (CUDA events around exactly `steps` calls) and the
    host's time per call (wall clock of the same loop, which only enqueues
    work: while the device is the bottleneck this is the host cost itself)."""
    import ratchet_b200 as rb

    R = len(sets)
    call = lambda s: public_call(s, call=entry)
    for i in range(warmup):
        call(sets[i % R])
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    h0 = time.perf_counter()
    for i in range(steps):
        call(sets[i % R])
    host_us = (time.perf_counter() - h0) * 1e6 / steps
    e1.record(st)
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    rb.last_status()
    return e0.elapsed_time(e1) / steps, host_us


def time_kernel_only(sets, steps, dev):
    """Average duration of the GEMM kernel alone: each set prepared once, then
    K launches of the GEMM half on rotating sets, events on the launch stream."""
    import ratchet_b200 as rb
    from ratchet_b200 import _lib, ops

    L = _lib.lib()
    st = torch.cuda.current_stream()
    handles = []
    for s in sets:
        pack = rb.pack_weights(s["b"], s["b_sf"])
        G = len(s["a"])
        n, k = pack.n, pack.k
        ms = [int(t.shape[0]) for t in s["a"]]
        out = torch.empty((sum(ms), n), dtype=torch.bfloat16, device=dev)
        m_arr = np.asarray(ms, dtype=np.int32)
        pa = ops._ptr_array([t.view(torch.uint8) for t in s["a"]])
        psf = ops._ptr_array([t.view(torch.uint8) for t in s["a_sf"]])
        prob = _lib.FggNvfp4Problem(G, n, k, m_arr.ctypes.data, pa.ctypes.data, psf.ctypes.data,
                                    s["alpha"].data_ptr(), out.data_ptr())
        nbytes = int(L.fgg_nvfp4_workspace_bytes(prob))
        wsb = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        _lib.check(L.fgg_nvfp4_prepare(prob, wsb.data_ptr(), nbytes, st.cuda_stream), "prepare")
        handles.append((prob, pack, wsb, nbytes, out, m_arr, pa, psf))
    for i in range(3):
        prob, pack, wsb, nb = handles[i % len(handles)][:4]
        _lib.check(L.fgg_nvfp4_gemm(prob, pack.buf.data_ptr(), wsb.data_ptr(), nb, st.cuda_stream), "gemm")
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(steps):
        prob, pack, wsb, nb = handles[i % len(handles)][:4]
        _lib.check(L.fgg_nvfp4_gemm(prob, pack.buf.data_ptr(), wsb.data_ptr(), nb, st.cuda_stream), "gemm")
    e1.record(st)
    torch.cuda.synchronize()
    for h in handles:
        rc = L.fgg_read_device_status(h[2].data_ptr(), st.cuda_stream)
        _lib.check(rc, "kernel-only status")
    return e0.elapsed_time(e1) / steps


def time_e2e(sets, steps, warmup, dev, ws):
    """The public call fed from pinned host memory, pipelined over three
    streams the way a serving loop runs it.  Step i: one H2D copy of its
    activation codes + scales (one pinned buffer per input set) on the copy
    stream, nvfp4_grouped_gemm on the compute stream (out= a per-set device
    buffer), one D2H copy of the whole bf16 output on the read-back stream.
    Step i's H2D overlaps step i-1's GEMM and step i-2's D2H; events keep
    each set's buffers from being reused before their last reader is done.
    Timed with events from the first H2D to the last D2H."""
    import ratchet_b200 as rb

    R = len(sets)
    n = sets[0]["sizes"][0][1]
    k = sets[0]["sizes"][0][2]
    bufs = []
    for s in sets:
        rows = int(s["a_all"].shape[0])
        codes = s["a_all"].cpu().pin_memory()
        scales = s["sf_all"].view(torch.uint8).cpu().pin_memory()
        out = torch.empty((rows, n), dtype=torch.bfloat16, device=dev)
        hout = torch.empty((rows, n), dtype=torch.bfloat16).pin_memory()
        # the step's H2D lands in the set's own contiguous activation buffers
        bufs.append(dict(codes=codes, scales=scales, d_codes=s["a_all"],
                         d_scales=s["sf_all"].view(torch.uint8), out=out, hout=hout))
    h2d = bufs[0]["codes"].numel() + bufs[0]["scales"].numel()
    d2h = bufs[0]["hout"].numel() * 2
    s_in, s_run, s_back = (torch.cuda.Stream(dev) for _ in range(3))
    ev = lambda: torch.cuda.Event()
    ready = [ev() for _ in range(R)]      # set b's inputs are on the device
    computed = [ev() for _ in range(R)]   # set b's GEMM is done
    drained = [ev() for _ in range(R)]    # set b's output is back on the host
    used = [False] * R

    def step(i):
        b = i % R
        s, B = sets[b], bufs[b]
        with torch.cuda.stream(s_in):
            if used[b]:
                s_in.wait_event(computed[b])  # the previous GEMM on set b has read its inputs
            B["d_codes"].copy_(B["codes"], non_blocking=True)
            B["d_scales"].copy_(B["scales"], non_blocking=True)
            ready[b].record(s_in)
        with torch.cuda.stream(s_run):
            s_run.wait_event(ready[b])
            if used[b]:
                s_run.wait_event(drained[b])  # the previous read-back of set b's output
            public_call(s, out=B["out"])
            computed[b].record(s_run)
        with torch.cuda.stream(s_back):
            s_back.wait_event(computed[b])
            B["hout"].copy_(B["out"], non_blocking=True)
            drained[b].record(s_back)
        used[b] = True

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    s_run.wait_event(e0)
    s_back.wait_event(e0)
    for i in range(steps):
        step(warmup + i)
    s_back.wait_stream(s_in)
    s_back.wait_stream(s_run)
    e1.record(s_back)
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps, h2d, d2h


def cpu_sample(wl, budget_s: float = 10.0, seed: int = 1234):
    """The CPU oracle on a bounded sample of the workload: whole groups in
    order, dequantise (torch CPU) + fp32 matmul + bf16, repeated over the
    group list until about budget_s of work has been timed."""
    from oracle import nvfp4 as ref

    torch.set_num_threads(os.cpu_count() or 1)
    rng = np.random.default_rng(seed)
    n, k = wl["n"], wl["k"]
    G = len(wl["m"])
    t_total, f_total, done = 0.0, 0.0, 0
    while t_total < budget_s and done < 64 * G:
        m = wl["m"][done % G]
        # the CPU cost does not depend on the values: random codes and scales
        qa, sa, qb, sb = _random_codes(rng, m, n, k)
        ga = gb = np.float32(1.0 / 2688.0)
        t0 = time.perf_counter()
        a = ref.nvfp4_dequantize_torch(qa, sa)
        b = ref.nvfp4_dequantize_torch(qb, sb)
        c = ((a @ b.T) * float(ga * gb)).to(torch.bfloat16)
        t_total += time.perf_counter() - t0
        f_total += 2.0 * m * n * k
        done += 1
        del c
    return {"value": f_total / t_total / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{done} group GEMMs ({done / G:.1f} passes over the {G} groups, N={n}, "
                      f"K={k}): torch-CPU dequantise + fp32 matmul + bf16, {t_total:.1f} s timed"}


def mx_inputs(wl, dev, seed: int = 0):
    """The MX campaign inputs in the reference's layout: per-expert row
    segments padded to 224 rows (m_indices = -1 on padding), E4M3 activations
    with power-of-two 1x128 scales, packed E2M1 weights with 1x32 scales."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    n, k, G = wl["n"], wl["k"], len(wl["m"])
    idx = []
    for e, r in enumerate(wl["m"]):
        idx += [e] * r + [-1] * ((-r) % 224)
    m_total = len(idx)
    mi = torch.tensor(idx, dtype=torch.int32, device=dev)
    a = torch.randint(0, 256, (m_total, k), dtype=torch.uint8, device=dev, generator=gen)
    a = torch.where((a & 0x7F) == 0x7F, a ^ 1, a).view(torch.float8_e4m3fn)  # no NaN codes
    a_sf = torch.exp2(torch.randint(-3, 4, (m_total, k // 128), device=dev, generator=gen).float())
    b = torch.randint(0, 256, (G, n, k // 2), dtype=torch.uint8, device=dev, generator=gen)
    b_sf = torch.exp2(torch.randint(-4, 3, (G, n, k // 32), device=dev, generator=gen).float())
    return a, a_sf, b, b_sf, mi


def mx_cpu_sample(wl, budget_s: float = 10.0, seed: int = 1234):
    """The MX oracle (oracle/mx.py) on a bounded sample: one expert segment
    of 224 rows per step, dequantise + fp32 matmul + bf16 on the host cores."""
    from oracle import mx as mref

    torch.set_num_threads(os.cpu_count() or 1)
    n, k = wl["n"], wl["k"]
    prob = mref.random_problem([224], n, k, seed=seed)
    t_total, f_total, done = 0.0, 0.0, 0
    while t_total < budget_s and done < 64:
        t0 = time.perf_counter()
        mref.fp4_grouped_gemm(prob["a"], prob["a_sf"], prob["b"], prob["b_sf"], prob["m_indices"])
        t_total += time.perf_counter() - t0
        f_total += 2.0 * 224 * n * k
        done += 1
    return {"value": f_total / t_total / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{done} expert segments of 224 rows (N={n}, K={k}): numpy dequantise + "
                      f"torch-CPU fp32 matmul + bf16, {t_total:.1f} s timed"}


def _random_codes(rng, m, n, k):
    """Random NVFP4 codes and E4M3 scales (bytes 0x30..0x5F, values 0.75..28)."""
    qa = torch.from_numpy(rng.integers(0, 256, size=(m, k // 2), dtype=np.uint8))
    sa = torch.from_numpy(rng.integers(0x30, 0x60, size=(m, k // 16), dtype=np.uint8))
    qb = torch.from_numpy(rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8))
    sb = torch.from_numpy(rng.integers(0x30, 0x60, size=(n, k // 16), dtype=np.uint8))
    return qa, sa, qb, sb


def traffic_from_profiles(config: str):
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text()).get(config)
        except json.JSONDecodeError:
            return None
    return None


# ------------------------------------------------------------------ arms
def run_reference(args, wl):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    if wl["name"] == "mx":
        return run_reference_mx(args, wl)
    from oracle import nvfp4 as ref

    torch.set_num_threads(os.cpu_count() or 1)
    rng = np.random.default_rng(0)
    n, k = wl["n"], wl["k"]
    G = len(wl["m"])
    data = []
    for gi in range(min(G, 4)):
        m = min(wl["m"][gi], 1024)  # bounded sample per step
        qa, sa, qb, sb = _random_codes(rng, m, n, k)
        data.append((m, qa, sa, qb, sb, float(np.float32(1.0 / 2688.0) ** 2)))

    def step(i):
        m, qa, sa, qb, sb, al = data[i % len(data)]
        a = ref.nvfp4_dequantize_torch(qa, sa)
        b = ref.nvfp4_dequantize_torch(qb, sb)
        ((a @ b.T) * al).to(torch.bfloat16)
        return 2.0 * m * n * k

    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    fl = 0.0
    for i in range(args.steps):
        fl += step(i)
    dt = time.perf_counter() - t0
    val = fl / dt / 1e12
    line = {
        "impl": "reference", "metric": "grouped-GEMM TFLOPS", "value": val, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong" if wl["name"] == "moe" else "weak",
        "vs_baseline": None, "dtype": "f32 (dequantised NVFP4)", "data": "synthetic",
        "config": {"workload": wl["desc"], "parallelism": "cpu"},
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": "each step one group of at most 1024 rows (cycling over "
                                   f"the first {len(data)} groups): dequantise + fp32 matmul + "
                                   "bf16"},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_reference_mx(args, wl):
    """The reference arm at the MX campaign point: the oracle's restatement of
    kernel.py:2788 on the host cores, a bounded sample per step."""
    from oracle import mx as mref

    torch.set_num_threads(os.cpu_count() or 1)
    n, k = wl["n"], wl["k"]
    prob = mref.random_problem([224], n, k, seed=0)
    step = lambda: mref.fp4_grouped_gemm(prob["a"], prob["a_sf"], prob["b"], prob["b_sf"],
                                         prob["m_indices"])
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    val = 2.0 * 224 * n * k * args.steps / dt / 1e12
    line = {
        "impl": "reference", "metric": "grouped-GEMM TFLOPS", "value": val, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (dequantised MXFP8 x MXFP4)", "data": "synthetic",
        "config": {"workload": wl["desc"], "parallelism": "cpu"},
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": "each step one expert segment of 224 rows: numpy dequantise "
                                   "+ torch-CPU fp32 matmul + bf16"},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


REF_KERNEL = ROOT / "baseline" / "_ref" / "kernels" / "gemm" / "fp4_grouped_gemm" / "b200" / "kernel.py"
MX_CAMPAIGN_SEED = 2026


def load_reference_kernel():
    """The reference's own B200 kernel module (kernels/gemm/fp4_grouped_gemm/
    b200/kernel.py, unmodified), from the reference install under
    baseline/_ref (not part of this repository).  Returns (module, None) or
    (None, why)."""
    import importlib.util

    if not REF_KERNEL.exists():
        return None, f"reference kernel not installed at {REF_KERNEL.relative_to(ROOT)}"
    try:
        spec = importlib.util.spec_from_file_location("reference_fp4_grouped_gemm", str(REF_KERNEL))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    except Exception as e:  # the DSL it needs is missing or incompatible
        return None, f"reference kernel did not import: {type(e).__name__}: {e}"
    return mod, None


def mx_campaign_on_device(dev, seed: int = MX_CAMPAIGN_SEED):
    """The MX campaign problem (oracle/mx.py campaign_problem, numpy) on the device."""
    from oracle import mx as mref

    p = mref.campaign_problem(seed)
    t = {k: torch.from_numpy(v).to(dev) for k, v in p.items()}
    return (t["a"].view(torch.float8_e4m3fn), t["a_sf"], t["b"], t["b_sf"], t["m_indices"]), p


def _device_close(got, want):
    """The operator tolerance evaluated on the device (no host copy of the outputs)."""
    g, w = got.float(), want.float()
    d = (g - w).abs()
    scale = float(w.abs().max())
    bad = int((d > 2e-2 * w.abs() + 1e-2 * scale).sum())
    rel = float(d.max()) / scale if scale > 0 else float(d.max())
    return {"rel": rel, "bad": bad, "max_ref": scale, "bitexact_frac": float((g == w).float().mean()),
            "ok": rel <= 1e-2 and bad == 0}


def run_reference_gpu_mx(args, wl):
    """The reference's own kernel.py next to fp4_grouped_gemm on the same B200,
    same inputs, same timing protocol: warm-up calls, then alternating windows
    of `steps` back-to-back calls per arm (CUDA events), median per arm.  Also
    compares the two outputs on every valid row and both with the CPU oracle on
    sampled rows."""
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if ws > 1:
        if rank == 0:
            print(json.dumps({"impl": "reference-gpu", "unavailable": "the reference kernel arm "
                              "runs on one GPU only"}))
        return 0
    mod, why = load_reference_kernel()
    if mod is None:
        print(json.dumps({"impl": "reference-gpu", "unavailable": why}))
        return 0
    import hashlib

    import ratchet_b200 as rb
    from oracle import mx as mref
    from oracle import nvfp4 as ref

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    args_t, prob = mx_campaign_on_device(dev)
    valid = args_t[4] >= 0
    arms = {"reference": lambda: mod.fp4_grouped_gemm(*args_t),
            "ours": lambda: rb.fp4_grouped_gemm(*args_t)}
    t0 = time.perf_counter()
    c_ref = arms["reference"]()
    torch.cuda.synchronize()
    first_ref_s = time.perf_counter() - t0
    c_ours = arms["ours"]()
    torch.cuda.synchronize()
    rb.last_status()
    parity = {"ours_vs_reference": _device_close(c_ours[valid], c_ref[valid])}
    rows = np.flatnonzero(prob["m_indices"] >= 0)[::1024]
    want = mref.campaign_rows_output(MX_CAMPAIGN_SEED, rows)
    ridx = torch.from_numpy(rows).to(dev)
    for name, c in (("oracle_vs_reference", c_ref), ("oracle_vs_ours", c_ours)):
        ok, st = ref.check_close(c.index_select(0, ridx).cpu(), want)
        parity[name] = dict(st, ok=ok, rows=int(rows.size))
    del c_ref, c_ours
    for _ in range(args.warmup):
        for f in arms.values():
            f()
    torch.cuda.synchronize()
    windows = {k: [] for k in arms}
    sampler = ClockSampler(0)
    sampler.start()
    for w in range(5):
        for name in (("reference", "ours") if w % 2 == 0 else ("ours", "reference")):
            f = arms[name]
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            for _ in range(args.steps):
                f()
            e1.record()
            torch.cuda.synchronize()
            windows[name].append(e0.elapsed_time(e1) / args.steps)
    clocks = sampler.stop()
    rb.last_status()
    fl = flops(wl)
    med = {k: statistics.median(v) for k, v in windows.items()}
    line = {
        "impl": "reference-gpu", "metric": "grouped-GEMM TFLOPS", "unit": "TFLOP/s",
        "value": fl / (med["reference"] * 1e-3) / 1e12, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": med["reference"], "higher_is_better": True,
        "config": {"workload": wl["desc"], "m_total": int(prob["m_indices"].size),
                   "seed": MX_CAMPAIGN_SEED,
                   "l2": "one 0.36 GB input set (> L2), back-to-back calls"},
        "reference": {"ms": med["reference"], "windows_ms": windows["reference"],
                      "tflops": fl / (med["reference"] * 1e-3) / 1e12,
                      "first_call_s_with_compile": first_ref_s,
                      "kernel_sha256": hashlib.sha256(REF_KERNEL.read_bytes()).hexdigest()},
        "ours": {"ms": med["ours"], "windows_ms": windows["ours"],
                 "tflops": fl / (med["ours"] * 1e-3) / 1e12},
        "ours_speedup": med["reference"] / med["ours"],
        "parity": parity, "clocks": clocks,
        "protocol": f"{args.warmup} warm-up calls per arm, then 5 alternating windows of "
                    f"{args.steps} back-to-back calls per arm (CUDA events), median",
    }
    print(json.dumps(line), flush=True)
    return 0


def run_mx(args, wl):
    """fp4_grouped_gemm, the reference's own operator, at its campaign point
    (kernel.py:213, :286-288: 0.3756 ms on the reference's B200).  One GPU, or
    independent replicas under torchrun.  A step is one call; the scale repack
    is cached on tensor identity as the reference caches it, so a step is the
    GEMM kernel."""
    ws, rank, local = dist_init()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import ratchet_b200 as rb

    a, a_sf, b, b_sf, mi = mx_inputs(wl, dev, seed=1000 * rank)
    call = lambda: rb.fp4_grouped_gemm(a, a_sf, b, b_sf, mi)
    for _ in range(args.warmup):
        call()
    sampler = ClockSampler(local)  # started before the barrier (see run_moe)
    sampler.start()
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        call()
    e1.record()
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    rb.last_status()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, ws, dev)
    fl = flops(wl)  # the 32768 real rows; padding rows are not counted
    value = fl * ws / (ms * 1e-3) / 1e12

    # end to end: each step copies this rank's activations and their scales
    # from pinned host memory into the call's input tensors (new contents, so
    # the operator repacks the activation scales, as it must for new
    # inputs), calls the operator and reads the whole output back
    e2e = None
    if not args.no_e2e:
        h_a = a.view(torch.uint8).cpu().pin_memory()
        h_sf = a_sf.cpu().pin_memory()
        h_c = torch.empty((int(a.shape[0]), wl["n"]), dtype=torch.bfloat16).pin_memory()
        a_u8 = a.view(torch.uint8)

        def e2e_step():
            a_u8.copy_(h_a, non_blocking=True)
            a_sf.copy_(h_sf, non_blocking=True)
            h_c.copy_(call(), non_blocking=True)

        for _ in range(2):
            e2e_step()
        n_e2e = max(3, min(args.steps, 10))  # each step moves about 0.4 GB over the host link
        torch.cuda.synchronize()
        barrier(ws)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(n_e2e):
            e2e_step()
        e1.record()
        torch.cuda.synchronize()
        barrier(ws)
        e2e_ms = max_over_ranks(e0.elapsed_time(e1) / n_e2e, ws, dev)
        e2e = {"value": fl * ws / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": int(h_a.numel() + h_sf.numel() * 4) * ws,
               "d2h_bytes_per_step": int(h_c.numel() * 2) * ws, "ms_per_step": e2e_ms,
               "steps": n_e2e}
    pk = peaks()
    achieved = fl / (ms * 1e-3) / 1e12
    peak = 2.0 * pk["bf16"]  # .kind::mxf8f6f4 runs at the FP8 rate, twice bf16
    ref_value = fl / (wl["ref_us"] * 1e-6) / 1e12
    if rank == 0:
        line = {
            "metric": "grouped-GEMM TFLOPS", "value": value, "unit": "TFLOP/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak",
            "vs_baseline": achieved / ref_value,
            "vs_baseline_basis": "the reference's published 0.3756 ms device time at this "
                                 "config (kernels/gemm/fp4_grouped_gemm/b200/kernel.py:213, "
                                 ":286), on its own B200",
            "dtype": "mxf8f6f4 (e4m3 x e2m1, ue8m0 scales 1x128 / 1x32, fp32 acc, bf16 out)",
            "data": "synthetic (seeded random E4M3 / E2M1 codes, power-of-two scales)",
            "config": {"workload": wl["desc"], "m_total": int(a.shape[0]), "n": wl["n"],
                       "k": wl["k"], "experts": len(wl["m"]), "parallelism": f"replicas x{ws}",
                       "l2": "back-to-back calls on one 0.5 GB input set (> L2)"},
            "clocks": clocks,
            "e2e": e2e,
            "gpu_launches": args.steps,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak, "traffic": None,
                         "peak_basis": f"2 x {pk['src']} dense bf16 ({pk['bf16']:.0f} TF/s)",
                         "kernel_ms": ms, "kernel": "fgg_gemm_pair_kernel<PairCfg<MX>>"},
            "cpu_baseline": (mx_cpu_sample(wl) if (ws == 1 and not args.no_cpu) else None),
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


def run_ours(args, wl):
    ws, rank, local = dist_init()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import ratchet_b200 as rb  # noqa: F401  (fails loudly without the native library)

    sub = shard(wl, ws, rank)
    # dense and decode split one problem over the ranks (at every N, 1 included)
    strong = wl["name"] in ("dense", "decode")
    # replicas draw their own data; a split workload draws the same problem on every rank
    seed0 = 0 if strong else 1000 * rank
    per_set = set_bytes(sub)
    R = max(1, min(8, int(np.ceil(2.0 * L2_BYTES / per_set)) + (1 if per_set < L2_BYTES else 0)))
    sets = [make_set(sub, seed0 + s, dev) for s in range(R)]
    torch.cuda.synchronize()

    sampler = ClockSampler(local)
    sampler.start()
    ms, host_us = time_value(sets, args.steps, args.warmup, dev, ws)
    clocks = sampler.stop()
    ms = max_over_ranks(ms, ws, dev)
    host_us = max_over_ranks(host_us, ws, dev)
    # the other public entry on the same sets, for its step and host cost
    other = "list" if CALL == "rows" else "rows"
    o_ms, o_host = time_value(sets, args.steps, args.warmup, dev, ws, entry=other)
    o_ms, o_host = max_over_ranks(o_ms, ws, dev), max_over_ranks(o_host, ws, dev)
    fl_rank = flops(sub)
    fl = flops(wl) if strong else fl_rank * ws     # work of the whole job
    value = fl / (ms * 1e-3) / 1e12

    k_ms = time_kernel_only(sets, args.steps, dev)
    pk = peaks()
    # the roofline of the slowest rank's GEMM kernel against its own work
    if wl["bound"] == "tensor":
        achieved = fl_rank / (k_ms * 1e-3) / 1e12
        frac = max_over_ranks(-achieved / (4.0 * pk["bf16"]), ws, dev) * -1.0
        k_ms = max_over_ranks(k_ms, ws, dev)
        roof = {"bound": "tensor", "achieved": frac * 4.0 * pk["bf16"], "peak": 4.0 * pk["bf16"],
                "unit": "TFLOP/s", "frac": frac, "traffic": traffic_from_profiles(wl["name"]),
                "peak_basis": f"4 x {pk['src']} dense bf16 ({pk['bf16']:.0f} TF/s)",
                "kernel_ms": k_ms, "alg_bytes": alg_bytes(sub),
                "kernel": "the GEMM launch alone (fgg_nvfp4_gemm after one prepare per set; "
                          "the same tile kernel both public entries launch)"}
    else:
        achieved = alg_bytes(sub) / (k_ms * 1e-3) / 1e9
        frac = max_over_ranks(-achieved / pk["hbm"], ws, dev) * -1.0
        k_ms = max_over_ranks(k_ms, ws, dev)
        roof = {"bound": "hbm", "achieved": frac * pk["hbm"], "peak": pk["hbm"], "unit": "GB/s",
                "frac": frac, "traffic": traffic_from_profiles(wl["name"]),
                "peak_basis": f"{pk['src']} HBM copy", "kernel_ms": k_ms,
                "alg_bytes": alg_bytes(sub)}

    if args.no_e2e:
        e2e_ms, h2d, d2h = float("nan"), 0, 0
    else:
        e2e_ms, h2d, d2h = time_e2e(sets, args.steps, args.warmup, dev, ws)
        e2e_ms = max_over_ranks(e2e_ms, ws, dev)

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        cpu = cpu_sample(wl)

    if rank == 0:
        line = {
            "metric": "grouped-GEMM TFLOPS", "value": value, "unit": "TFLOP/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong" if strong else "weak",
            "vs_baseline": None,
            "dtype": "nvfp4 (e2m1 x e2m1, e4m3/16 scales, fp32 acc, bf16 out)",
            "data": "synthetic (seeded N(0,1) activations, N(0,w_std) weights, NVFP4-quantised)",
            "config": {"workload": wl["desc"], "groups": len(wl["m"]), "sum_m": sum(wl["m"]),
                       "n": wl["n"], "k": wl["k"],
                       "parallelism": (f"replicas x{ws}" if not strong else
                                       ("N split" if wl["name"] == "dense" else "groups sharded")
                                       + f" over {ws}"),
                       "rank0_part": sub["split"],
                       "call": ("nvfp4_grouped_gemm_rows (contiguous rows, device offsets)"
                                if CALL == "rows" else "nvfp4_grouped_gemm (per-group lists)"),
                       "l2": f"{R} rotating input sets of {per_set / 1e6:.0f} MB per rank "
                             "(> L2 in total)"},
            "clocks": clocks,
            "e2e": None if args.no_e2e else {
                "value": fl / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": h2d * ws, "d2h_bytes_per_step": d2h * ws,
                "ms_per_step": e2e_ms},
            "gpu_launches": 2 * args.steps,
            "host_us_per_call": host_us,
            "other_entry": {"call": other, "ms_per_step": o_ms, "host_us_per_call": o_host},
            "roofline": roof,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


def moe_setup(wl, ws: int, rank: int, dev) -> dict:
    """Config 3's seeded inputs for one rank of an ws-way expert-parallel run:
    Zipf(1.1) top-8 routing of all tokens (seed 0), LPT placement of the
    experts on their expected routed load (sampled independently of the
    batch), this rank's experts' weights (each drawn from its own seed, so
    they do not depend on ws) and this rank's share of the tokens, quantised
    to NVFP4 on the device."""
    import ratchet_b200 as rb
    from ratchet_b200 import moe

    T, E, topk, n, k = wl["tokens"], wl["experts"], wl["topk"], wl["n"], wl["k"]
    tl = T // ws
    ids_all, w_all = moe.zipf_routing(T, E, topk, s=1.1, seed=0)
    owner, slot = moe.place_experts(moe.routed_load(E, topk, s=1.1, seed=0), ws)
    mine = sorted(np.flatnonzero(owner == rank).tolist(), key=lambda e: slot[e])
    wc, wsf, wg = [], [], []
    for e in mine:
        gen = torch.Generator(device=dev)
        gen.manual_seed(7000 + e)
        q, sf, g = rb.quantize_nvfp4(torch.randn((n, k), generator=gen, device=dev))
        wc.append(q)
        wsf.append(sf)
        wg.append(g)
    gen = torch.Generator(device=dev)
    gen.manual_seed(9000 + rank)
    xc, xs, xg = rb.quantize_nvfp4(torch.randn((tl, k), generator=gen, device=dev))
    ids = torch.from_numpy(ids_all[rank * tl:(rank + 1) * tl]).to(dev)
    wts = torch.from_numpy(w_all[rank * tl:(rank + 1) * tl]).to(dev)
    return dict(tl=tl, ids_all=ids_all, w_all=w_all, owner=owner, slot=slot, mine=mine,
                wc=wc, wsf=wsf, wg=wg, xc=xc, xs=xs, xg=xg, ids=ids, wts=wts)


def run_moe(args, wl):
    """one expert-parallel MoE projection over N ranks.
    The 4096 tokens are split evenly over the ranks (each rank routes its own
    share); the 64 experts are placed by expected load (LPT, equal counts).
    A step = pack + all-gather dispatch + expand + grouped GEMM + weighted
    reduce + all-to-all combine + partial sum, with no host synchronisation,
    replayed from one CUDA graph.  Total work is fixed, so the scaling is
    strong; value = all FLOPs / the slowest rank's step time.  The line also
    carries a per-phase breakdown of the same forward issued eagerly (CUDA
    events between the phases on the compute stream, mean over the steps,
    max over ranks)."""
    from ratchet_b200 import moe

    ws, rank, local = dist_init()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import ratchet_b200 as rb

    T, E, topk, n, k = wl["tokens"], wl["experts"], wl["topk"], wl["n"], wl["k"]
    if T % ws or E % ws:
        raise SystemExit(f"--gpus {ws} must divide {T} tokens and {E} experts")
    d = moe_setup(wl, ws, rank, dev)
    tl, ids_all, mine = d["tl"], d["ids_all"], d["mine"]
    xc, xs, xg, ids, wts = d["xc"], d["xs"], d["xg"], d["ids"], d["wts"]
    layer = moe.ExpertParallelMoE(d["wc"], d["wsf"], d["wg"], d["owner"], d["slot"], max_tokens=tl,
                                  combine=args.combine, transport=args.transport)
    torch.cuda.synchronize()
    fl = 2.0 * T * topk * n * k

    # 1. eager forwards with CUDA events between the phases: the per-phase
    #    breakdown and the host's enqueue time per forward (not the value)
    for _ in range(args.warmup):
        layer.forward(xc, xs, xg, ids, wts)
    torch.cuda.synchronize()
    barrier(ws)
    evs = [dict() for _ in range(args.steps)]
    h0 = time.perf_counter()
    for i in range(args.steps):
        layer.forward(xc, xs, xg, ids, wts, events=evs[i])
    host_ms = (time.perf_counter() - h0) * 1e3 / args.steps
    torch.cuda.synchronize()
    barrier(ws)
    layer.check()
    names = list(moe.PHASES) + ["end"]
    phases = {}
    for a, b in zip(names[:-1], names[1:]):
        mean = sum(ev[a].elapsed_time(ev[b]) for ev in evs) / args.steps
        phases[a] = max_over_ranks(mean, ws, dev)
    eager_steps = [ev["pack"].elapsed_time(ev["end"]) for ev in evs]
    eager_ms = max_over_ranks(statistics.median(eager_steps), ws, dev)
    host_ms = max_over_ranks(host_ms, ws, dev)

    # 2. the timed steps: the whole layer (kernels and collectives) replayed
    #    from one CUDA graph per step
    replay, out_g = layer.capture(xc, xs, xg, ids, wts)
    for _ in range(args.warmup):
        replay()
    # the sampler starts before the barrier: a rank still spawning it would
    # hold the others' first collective
    sampler = ClockSampler(local)
    sampler.start()
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        replay()
    e1.record()
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    layer.check()
    rb.last_status()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, ws, dev)
    g_ms = phases["gemm"]
    # GEMM rows on this rank (the kernel's FLOPs): the routes of its experts from every rank
    counts = np.bincount(ids_all.ravel(), minlength=E)
    my_rows = int(counts[np.asarray(mine)].sum())
    g_fl = max_over_ranks(2.0 * my_rows * n * k, ws, dev)
    pk = peaks()
    achieved = g_fl / (g_ms * 1e-3) / 1e12
    peak = 4.0 * pk["bf16"]
    roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
            "frac": achieved / peak, "traffic": traffic_from_profiles("moe"),
            "peak_basis": f"4 x {pk['src']} dense bf16 ({pk['bf16']:.0f} TF/s)",
            "kernel_ms": g_ms, "kernel": "grouped GEMM inside the layer (device-offset prepare + "
                                        "fgg_gemm_pair_kernel), slowest rank, eager pass"}

    # 3. end to end: this rank's activations from pinned host memory into the
    #    graph's input tensors, the replay, the output back to pinned memory,
    #    pipelined the way a serving loop runs it: two input/output sets, each
    #    with its own captured graph; step i's H2D (copy stream) overlaps step
    #    i-1's replay and step i-2's D2H (read-back stream), and events keep a
    #    set's buffers from being reused before their last reader is done
    xc2, xs2 = xc.clone(), xs.clone()
    replay2, out_g2 = layer.capture(xc2, xs2, xg, ids, wts)
    for _ in range(args.warmup):
        replay2()
    h_xc = xc.cpu().pin_memory()
    h_xs = xs.view(torch.uint8).cpu().pin_memory()
    slots = [(xc, xs.view(torch.uint8), replay, out_g), (xc2, xs2.view(torch.uint8), replay2, out_g2)]
    h_outs = [torch.empty((tl, n), dtype=torch.bfloat16).pin_memory() for _ in slots]
    e2e_steps = args.steps
    cur = torch.cuda.current_stream()
    s_in, s_back = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ready = [torch.cuda.Event() for _ in slots]     # set b's inputs are on the device
    consumed = [torch.cuda.Event() for _ in slots]  # set b's replay is done
    drained = [torch.cuda.Event() for _ in slots]   # set b's output is back on the host
    used = [False] * len(slots)

    def e2e_step(i):
        bi = i % len(slots)
        d_xc, d_xs, rep, out_b = slots[bi]
        with torch.cuda.stream(s_in):
            if used[bi]:
                s_in.wait_event(consumed[bi])   # the last replay on set b has read its inputs
            d_xc.copy_(h_xc, non_blocking=True)
            d_xs.copy_(h_xs, non_blocking=True)
            ready[bi].record(s_in)
        cur.wait_event(ready[bi])
        if used[bi]:
            cur.wait_event(drained[bi])         # set b's last output has been read back
        rep()
        consumed[bi].record(cur)
        with torch.cuda.stream(s_back):
            s_back.wait_event(consumed[bi])
            h_outs[bi].copy_(out_b, non_blocking=True)
            drained[bi].record(s_back)
        used[bi] = True

    for i in range(3):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    e0.record(cur)
    s_in.wait_event(e0)
    s_back.wait_event(e0)
    for i in range(e2e_steps):
        e2e_step(3 + i)
    cur.wait_stream(s_in)
    cur.wait_stream(s_back)
    e1.record(cur)
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps, ws, dev)
    h_out = h_outs[0]
    # the graphs hold the collectives' captured work: drop every reference
    # before the layer and the process group go
    del replay2, slots
    del replay
    layer.release()
    if args.transport == "p2p":
        # dispatch (pack + peer stores), wait, expand (2), GEMM (2), reduce, signal, wait, sum
        launches = 10
        dispatch_desc = ("peer stores of token records into every rank's buffer by the "
                         "library's dispatch kernel (CUDA IPC, no multicast), bounded flag wait")
        combine_desc = ("router-weighted partial rows kept where they are computed, "
                        "bounded flag wait, fp32 sum reading them over NVLink")
    else:
        launches = 7 if ws > 1 else 5
        dispatch_desc = ("NCCL all-gather of token records (capacity = tokens per rank)"
                         if ws > 1 else "none (one rank)")
        combine_desc = (("NCCL reduce-scatter of router-weighted partial rows"
                         if args.combine == "reduce_scatter" else
                         "NCCL all-to-all of router-weighted partial rows, fp32 sum")
                        if ws > 1 else "router-weighted sum on the rank")

    if rank == 0:
        line = {
            "metric": "grouped-GEMM TFLOPS", "value": fl / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "nvfp4 (e2m1 x e2m1, e4m3/16 scales, fp32 acc, bf16 out)",
            "data": "synthetic (seeded N(0,1) tokens and expert weights, NVFP4-quantised; "
                    "Zipf(1.1) top-8 routing)",
            "config": {"workload": wl["desc"], "tokens": T, "experts": E, "topk": topk,
                       "n": n, "k": k, "parallelism": f"ep{ws}",
                       "placement": "LPT on expected routed load (top-8 inclusion probability), equal expert counts",
                       "dispatch": dispatch_desc,
                       "combine": combine_desc,
                       "l2": f"expert weights {E * n * k * 0.5625 / ws / 1e6:.0f} MB per rank "
                             "read every step"},
            "phases_ms": phases,
            "eager": {"ms_per_step_median": eager_ms, "host_enqueue_ms": host_ms,
                      "note": "the same forward issued kernel by kernel (phases_ms come from it); "
                              "the timed steps replay it from one CUDA graph"},
            "clocks": clocks,
            "e2e": {"value": fl / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": int(h_xc.numel() + h_xs.numel()) * ws,
                    "d2h_bytes_per_step": int(h_out.numel() * 2) * ws, "ms_per_step": e2e_ms,
                    "pipeline": "two input/output slots, each with its own graph; H2D, replay "
                                "and D2H on three streams, overlapped across steps"},
            "gpu_launches": launches * args.steps,
            "roofline": roof,
            "cpu_baseline": cpu_sample(wl) if (ws == 1 and not args.no_cpu) else None,
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


def run_mlp(args, wl):
    """The gated expert MLP (nvfp4_expert_mlp) on one GPU, or as independent
    replicas under torchrun.  A step = gate+up grouped GEMM with the SiLU*up
    epilogue, amax + NVFP4 quantisation of the intermediate, down grouped
    GEMM: the whole call is timed (it is the kernel time too)."""
    ws, rank, local = dist_init()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import ratchet_b200 as rb

    gen = torch.Generator(device=dev)
    gen.manual_seed(1000 * rank + 5)
    hid, inter = wl["k"], wl["inter"]
    A, ASF, a13, W13, W13SF, W2, W2SF, w2g = [], [], [], [], [], [], [], []
    for m in wl["m"]:
        qa, sa, ga = rb.quantize_nvfp4(torch.randn((m, hid), generator=gen, device=dev))
        q13, s13, g13 = rb.quantize_nvfp4(torch.randn((2 * inter, hid), generator=gen, device=dev))
        q13, s13 = rb.interleave_gate_up(q13, s13)
        q2, s2, g2 = rb.quantize_nvfp4(torch.randn((hid, inter), generator=gen, device=dev))
        A.append(qa)
        ASF.append(sa)
        a13.append(ga * g13)
        W13.append(q13)
        W13SF.append(s13)
        W2.append(q2)
        W2SF.append(s2)
        w2g.append(g2)
    alpha13 = torch.stack(a13).float()
    w2s = torch.stack(w2g).float()
    call = lambda: rb.nvfp4_expert_mlp(A, ASF, alpha13, W13, W13SF, W2, W2SF, w2s)
    for _ in range(args.warmup):
        call()
    sampler = ClockSampler(local)  # started before the barrier (see run_moe)
    sampler.start()
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        call()
    e1.record()
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    rb.last_status()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, ws, dev)
    fl = flops(wl)
    value = fl * ws / (ms * 1e-3) / 1e12
    pk = peaks()
    achieved = fl / (ms * 1e-3) / 1e12
    peak = 4.0 * pk["bf16"]
    wbytes = sum(t.numel() for t in W13 + W13SF + W2 + W2SF)
    if rank == 0:
        line = {
            "metric": "grouped-GEMM TFLOPS", "value": value, "unit": "TFLOP/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "nvfp4 (e2m1 x e2m1, e4m3/16 scales, fp32 acc, bf16 out)",
            "data": "synthetic (seeded N(0,1) activations and weights, NVFP4-quantised)",
            "config": {"workload": wl["desc"], "groups": len(wl["m"]), "sum_m": sum(wl["m"]),
                       "hidden": hid, "inter": inter, "parallelism": f"replicas x{ws}",
                       "l2": f"expert weights {wbytes / 1e6:.0f} MB read every step (> L2)"},
            "clocks": clocks,
            "e2e": None,
            "gpu_launches": 6 * args.steps,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak, "traffic": None,
                         "peak_basis": f"4 x {pk['src']} dense bf16 ({pk['bf16']:.0f} TF/s)",
                         "kernel_ms": ms,
                         "kernel": "whole call: two prepare + two GEMM kernels, amax, quantise"},
            "cpu_baseline": None,
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


def _one_line_stdout():
    """Keep the process's stdout for the JSON line alone: file descriptor 1
    (where native libraries print, e.g. NCCL's version banner) goes to stderr,
    and Python's print writes to the original stdout."""
    real = os.dup(1)
    sys.stdout.flush()
    os.dup2(2, 1)
    sys.stdout = os.fdopen(real, "w", buffering=1)


def main():
    _one_line_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference", "reference-gpu"], default="ours")
    ap.add_argument("--config", choices=["grouped", "dense", "decode", "moe", "mlp", "mx"],
                    default="moe")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline sample")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--combine", choices=["a2a", "reduce_scatter"], default="a2a",
                    help="the MoE layer's combine collective (--config moe)")
    ap.add_argument("--call", choices=["rows", "list"], default="rows",
                    help="the public entry a GEMM step calls (configs other than moe / mx)")
    ap.add_argument("--transport", choices=["nccl", "p2p"], default="nccl",
                    help="the MoE layer's exchange: NCCL collectives or the library's "
                         "peer-store kernels (--config moe)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    global CALL
    CALL = args.call
    wl = workload(args.config)
    if args.impl == "reference" and wl["name"] == "mlp":
        print(json.dumps({"impl": "reference", "unavailable": "the reference operator has no "
                          "gated expert MLP; its CPU arm covers the GEMM configs"}))
        return 0
    if args.impl == "reference-gpu":
        if wl["name"] != "mx":
            print(json.dumps({"impl": "reference-gpu", "unavailable": "the reference's GPU kernel "
                              "is the MX operator: use --config mx"}))
            return 0
        return run_reference_gpu_mx(args, wl)
    if args.impl == "reference":
        return run_reference(args, wl)
    if wl["name"] == "moe":
        return run_moe(args, wl)
    if wl["name"] == "mlp":
        return run_mlp(args, wl)
    if wl["name"] == "mx":
        return run_mx(args, wl)
    return run_ours(args, wl)


if __name__ == "__main__":
    sys.exit(main())

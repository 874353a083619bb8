#!/usr/bin/env python
"""Benchmark of the SCA2 / Laplace long-head scan on B200 (sm_100a kernels).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload (one step = one pass of the hot path over one batch, inputs resident in HBM):
  the phase-coded delta scan of the LapA long head, forward + backward,
  B=8, T=4096, H=16, d_head=64 (Mh=32 complex modes, K=2Mh=64, V=64), per-mode decay
  lam = min(softplus(N(0,1)), 1/16), erase gate beta = sigmoid(N(0,1)), phases
  p*omega_rope + N(0,1), v and dO ~ N(0,1) in bf16, fp32 state.  Synthetic seeded data.
  Multi-GPU (torchrun): every rank runs its own (batch x head) shard of the same size
  (weak scaling, no data-path collective); time = max over ranks.

Printed: one JSON line (rank 0) with the contract keys plus roofline (dominant kernel),
cpu_baseline (numpy oracle on the host cores), e2e (public API, host buffers), clocks,
gpu_launches, a decode block (batch 256, H=16, K=V=128, 512 steps after a 4096 prefill) and an
sp_prefill block (one 131072-token sequence, H=16, d_head=64, split over the ranks: slab maps
all-gathered over NCCL, sequence-parallel prefill), a gdn_delta block (the delta rule in the
gated-delta-rule form with explicit keys: B=4, T=8192, H=8, d_k=d_v=128, bf16 fwd+bwd), and the
D-head, short-head, layer and LM blocks.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORK = dict(B=8, T=4096, H=16, Mh=32, V=64)
DECODE = dict(B=256, T=4096, H=16, Mh=64, V=128, steps=512)
SP = dict(B=1, T=131072, H=16, Mh=32, V=64)  # one long sequence, split over the ranks
DHEAD = dict(B=8, T=4096, M=16, G=8, V=64)   # D head of the reference LayerCfg (Md=16, G=8, dv=d/2)
SHORT = dict(B=8, T=4096, L=16, dv=64, decode_B=256)  # short head, LapA default window L=16
# delta-rule (GDN form) scan: explicit L2-normalised keys, per-token scalar decay and beta
GDN = dict(B=4, T=8192, H=8, K=128, V=128)
# one SCA2 layer (GatedLayer: 16 gated heads of d_head 64 + D head + mix + FFN), d_model 1024
LAYER = dict(B=8, T=4096, d=1024, heads=16, Mh=32, dvh=64, Md=4, G=8, ff=4096)
# 12-layer SCA2 LM training step (GatedLayer stack), d_model 768, 12 heads of d_head 64,
# vocab 16384, T=2048, 32 sequences per GPU, Zipf(1.1) tokens, bf16 autocast, AdamW
LMCFG = dict(B=32, T=2048, d=768, heads=12, Mh=32, dvh=64, Md=4, G=8, ff=3072, n_layers=12, vocab=16384,
             steps=3, warmup=2, decode_B=64, prompt=128, decode_steps=64)
# Algorithmic bytes per token per head (inputs read + outputs written once):
#   fwd: phi, psi fp32 (2*Mh*4) + v bf16 (V*2) + beta (4) + o bf16 (2*V*2)
#   bwd: dO bf16 (2*V*2) + inputs re-read (2*Mh*4 + V*2 + 4) + dphi, dpsi fp32 (2*Mh*4) + dv bf16 (V*2) + dbeta (4)
# what `value` times: the scan op of the hot path, not a whole layer (that is the "layer" block)
METRIC = "scan fwd+bwd tokens/s"
FWD_BYTES_TOK = lambda Mh, V: 2 * Mh * 4 + V * 2 + 4 + 2 * V * 2
BWD_BYTES_TOK = lambda Mh, V: 2 * V * 2 + (2 * Mh * 4 + V * 2 + 4) + (2 * Mh * 4 + V * 2 + 4)
# Algorithmic MACs per token per head of the delta form, R=2 read columns, chunk C=64:
#   R (C K/2 + C V/2 + K V) + K V + C K/2 (Gram) + K V (read-back) + C V/2 (solve); fwd+bwd = 3x
FWD_MAC_TOK = lambda K, V, C=64, R=2: R * (C * K / 2 + C * V / 2 + K * V) + K * V + C * K / 2 + K * V + C * V / 2


# --------------------------------------------------------------------------------------
#  CPU baseline: the numpy oracle on the host cores (spawned pool, one sequence per task)
# --------------------------------------------------------------------------------------
def _cpu_one(args):
    seed, T, Mh, V = args
    import numpy as np
    from oracle import scan as ora
    rng = np.random.default_rng(seed)
    p = np.arange(T, dtype=np.float32)[:, None]
    om = (np.pi * 1e4 ** (-np.arange(Mh) / (Mh - 1))).astype(np.float32)
    phw = (p * om + rng.standard_normal((T, Mh))).astype(np.float32)[None, :, None]
    phq = (p * om + rng.standard_normal((T, Mh))).astype(np.float32)[None, :, None]
    v = rng.standard_normal((1, T, 1, V)).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((1, T, 1))))).astype(np.float32)
    lam = np.minimum(np.log1p(np.exp(rng.standard_normal((1, Mh)))), 1 / 16).astype(np.float32)
    wr, wi = np.ones((1, Mh), np.float32), np.zeros((1, Mh), np.float32)
    do = rng.standard_normal((1, T, 1, 2, V)).astype(np.float32)
    t0 = time.perf_counter()
    k, Q = ora.phase_codes(phw, phq, wr, wi)
    lamf = np.concatenate([lam, lam], -1)
    ora.forward_chunked(k, Q, v, beta, None, lamf, float(Mh), None, C=64, dtype=np.float32)
    ora.backward_chunked(k, Q, v, beta, None, lamf, float(Mh), None, do, None, C=64, dtype=np.float32)
    return time.perf_counter() - t0


def cpu_pool():
    import multiprocessing as mp
    for var in ("OMP_NUM_THREADS", "MKL_NUM_THREADS", "OPENBLAS_NUM_THREADS"):
        os.environ[var] = "1"
    n = len(os.sched_getaffinity(0))
    return mp.get_context("spawn").Pool(n), n


def cpu_sample(pool, n, seed=0):
    """One bounded sample: n sequences of the workload (one (b,h) each, T tokens) fwd+bwd in
    parallel; returns (tokens/s of the layer = sequence-tokens / H per second, wall s)."""
    W = WORK
    nseq = min(n, W["B"] * W["H"])
    t0 = time.perf_counter()
    pool.map(_cpu_one, [(seed + i, W["T"], W["Mh"], W["V"]) for i in range(nseq)])
    wall = time.perf_counter() - t0
    return nseq * W["T"] / W["H"] / wall, wall, nseq


# --------------------------------------------------------------------------------------
#  clocks
# --------------------------------------------------------------------------------------
class Clocks:
    """SM clock and clock-event reasons sampled DURING the timed region: NVML (read-only
    queries) every 10 ms on a thread, plus one sample at start and at stop, so that even a
    timed region of a few ms is covered; nvidia-smi -lms 200 when NVML is unavailable."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, index):
        import threading
        self.rows, self.p, self.h = [], None, None
        try:
            import pynvml as N
            N.nvmlInit()
            self.N = N
            self.h = (N.nvmlDeviceGetHandleByUUID(index) if isinstance(index, str)
                      else N.nvmlDeviceGetHandleByIndex(index))
            self.bits = (N.nvmlClocksEventReasonHwSlowdown, N.nvmlClocksEventReasonHwThermalSlowdown,
                         N.nvmlClocksEventReasonSwThermalSlowdown, N.nvmlClocksEventReasonSwPowerCap)
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM)
            self.stop_ev = threading.Event()
            self._sample()
            self.t = threading.Thread(target=self._loop, daemon=True)
            self.t.start()
            return
        except Exception:
            self.h = None
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(index), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def _sample(self):
        N = self.N
        mhz = N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM)
        r = N.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        self.rows.append((float(mhz), float(self.max_mhz), [n for n, b in zip(self.NAMES, self.bits) if r & b]))

    def _loop(self):
        while not self.stop_ev.wait(0.01):
            try:
                self._sample()
            except Exception:
                return

    def stop(self):
        if self.h is not None:
            self.stop_ev.set()
            self.t.join(2)
            try:
                self._sample()
            except Exception:
                pass
            rows = self.rows
            if not rows:
                return None
            return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                    "reasons": sorted({n for r in rows for n in r[2]}), "samples": len(rows), "source": "nvml"}
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(5)
        except Exception:
            self.p.kill()
        self.f.flush()
        rows = []
        with open(self.f.name) as fh:
            for line in fh:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = sorted({n for r in rows for n, val in zip(self.NAMES, r[5:9]) if val.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "source": "nvidia-smi"}


# --------------------------------------------------------------------------------------
#  GPU arm
# --------------------------------------------------------------------------------------
def make_inputs(torch, seed, dev, B, T, H, Mh, V, dtype, with_grad_out=True):
    g = torch.Generator(device=dev).manual_seed(seed)
    rn = lambda *s: torch.randn(*s, device=dev, generator=g)
    p = torch.arange(T, device=dev, dtype=torch.float32)[:, None]
    om = math.pi * 1e4 ** (-torch.arange(Mh, device=dev, dtype=torch.float32) / (Mh - 1))
    pw = (p * om)[None, :, None, :]
    phw = (pw + rn(B, T, H, Mh)).contiguous()
    phq = (pw + rn(B, T, H, Mh)).contiguous()
    v = rn(B, T, H, V).to(dtype)
    beta = torch.sigmoid(rn(B, T, H))
    lam = torch.nn.functional.softplus(rn(H, Mh)).clamp(max=1 / 16)
    wr, wi = 1 + 0.3 * rn(H, Mh), 0.3 * rn(H, Mh)
    dO = rn(B, T, H, 2, V).to(dtype) if with_grad_out else None
    return dict(phw=phw, phq=phq, v=v, beta=beta, lam=lam, wr=wr, wi=wi, dO=dO)


def run_gpu(args, rank, world, local_rank, dist):
    import torch
    from sca2_b200 import ops

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    W = WORK
    B, T, H, Mh, V = W["B"], W["T"], W["H"], W["Mh"], W["V"]
    x = make_inputs(torch, 1234 + rank, dev, B, T, H, Mh, V, torch.bfloat16)
    plan = ops.PhaseScanPlan(x["phw"], x["phq"], x["v"], x["beta"], None, x["lam"], x["wr"], x["wi"])
    st = torch.cuda.current_stream()

    def step(ev=None):
        if ev is not None:
            ev[0].record(st)
        plan.fwd()
        if ev is not None:
            ev[1].record(st)
        plan.zero_grads()
        if ev is not None:
            ev[2].record(st)
        plan.bwd(x["dO"], zero=False)
        if ev is not None:
            ev[3].record(st)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    uuid = getattr(torch.cuda.get_device_properties(dev), "uuid", None)
    clocks = Clocks(f"GPU-{uuid}" if uuid is not None else torch.cuda.current_device()) if rank == 0 else None
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        step(evs[i])
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    clk = clocks.stop() if clocks is not None else None
    total_ms = evs[0][0].elapsed_time(evs[-1][3])
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    zero_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    bwd_ms = statistics.mean(e[2].elapsed_time(e[3]) for e in evs)
    if dist is not None:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_step = total_ms / args.steps

    # ---- end to end through the public API: host (pinned) inputs -> device, fwd + bwd, result -> host.
    # Two device input sets: the next step's host-to-device copies run on a copy stream while
    # the current step computes (every step's inputs still cross PCIe inside the timed region).
    e2e = None
    if not args.no_e2e:
        # The heads' own call: the projections K(h), K(z) in bf16 (theta = 1 per mode, so the phases
        # K theta + p omega have the workload's distribution) through ops.phase_scan_proj, which
        # forms the phases inside the kernels and returns dK(h), dK(z).
        g = torch.Generator(device=dev).manual_seed(4321 + rank)
        kh = torch.randn(B, T, H, Mh, device=dev, generator=g).bfloat16()
        kz = torch.randn(B, T, H, Mh, device=dev, generator=g).bfloat16()
        theta = torch.ones(H, Mh, device=dev)
        omega = (math.pi * 1e4 ** (-torch.arange(Mh, device=dev, dtype=torch.float32) / (Mh - 1))).expand(H, Mh)
        omega = omega.contiguous()
        pos0 = torch.zeros((), device=dev)
        src = dict(kh=kh, kz=kz, v=x["v"], beta=x["beta"], dO=x["dO"])
        keys = tuple(src)
        host = {k: src[k].cpu().pin_memory() for k in keys}
        h2d = sum(t.numel() * t.element_size() for t in host.values())
        # every step's results come back to pinned host memory: the read o, the final state and
        # the gradients of every per-token input (K(h), K(z), v, beta)
        pin = lambda *s, dt=torch.float32: torch.empty(*s, dtype=dt).pin_memory()
        res = dict(o=pin(B, T, H, 2, V, dt=torch.bfloat16), S=pin(B, H, 2 * Mh, V),
                   kh=pin(B, T, H, Mh, dt=torch.bfloat16), kz=pin(B, T, H, Mh, dt=torch.bfloat16),
                   v=pin(B, T, H, V, dt=torch.bfloat16), beta=pin(B, T, H))
        d2h = sum(t.numel() * t.element_size() for t in res.values())
        bufs = [{k: torch.empty_like(src[k]) for k in keys} for _ in range(2)]
        del kh, kz, src
        cs = torch.cuda.Stream(device=dev)
        ds = torch.cuda.Stream(device=dev)  # device -> host copies of the results
        ready = [torch.cuda.Event() for _ in range(2)]
        free = [torch.cuda.Event() for _ in range(2)]
        used = [False, False]

        def copy_in(i):
            sl = i % 2
            with torch.cuda.stream(cs):
                if used[sl]:
                    cs.wait_event(free[sl])
                for k in keys:
                    bufs[sl][k].copy_(host[k], non_blocking=True)
                ready[sl].record(cs)

        def compute(i):
            sl = i % 2
            st.wait_event(ready[sl])
            d = dict(bufs[sl])
            for k in ("kh", "kz", "v", "beta"):
                d[k] = d[k].detach().requires_grad_(True)  # leaf over the buffer's storage
            o, S = ops.phase_scan_proj(d["kh"], d["kz"], theta, omega, pos0, d["v"], d["beta"], None, x["lam"],
                                       x["wr"], x["wi"])
            torch.autograd.backward(o, d["dO"])
            out = dict(o=o.detach(), S=S.detach(), kh=d["kh"].grad, kz=d["kz"].grad, v=d["v"].grad,
                       beta=d["beta"].grad)
            done = torch.cuda.Event()
            done.record(st)
            free[sl].record(st)
            used[sl] = True
            # the results leave on their own stream while the next step computes
            ds.wait_event(done)
            with torch.cuda.stream(ds):
                for k, t in out.items():
                    t.record_stream(ds)
                    res[k].copy_(t, non_blocking=True)

        def run(n):
            copy_in(0)
            for i in range(n):
                if i + 1 < n:
                    copy_in(i + 1)
                compute(i)

        run(max(1, args.warmup))
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        # a pipelined run: the first step's input copy and the last step's result copy overlap
        # nothing (about 6 ms each way at the benchmark shape), so enough steps that this fill
        # and drain stays a small part of the average (every step's copies are still timed)
        n_e2e = max(30, args.steps)
        e0.record(st)
        cs.wait_stream(st)  # the first copy starts inside the timed region
        run(n_e2e)
        st.wait_stream(ds)  # the last step's results are on the host
        e1.record(st)
        torch.cuda.synchronize()
        em = e0.elapsed_time(e1) / n_e2e
        if dist is not None:
            t = torch.tensor([em], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            em = float(t.item())
        e2e = {"value": world * B * T / (em / 1e3), "unit": "tokens/s", "ms_per_step": em,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "api": "ops.phase_scan_proj + torch.autograd.backward (the heads' call: bf16 K(h), K(z), v, dO; "
                      "fp32 beta; phases formed in the kernels)",
               "copied_out": "o, S, dK(h), dK(z), dv, d beta",
               "pipelining": "next step's H2D on a copy stream and the previous step's D2H on another "
                             "overlap the current step's compute",
               "steps": n_e2e}
        del host, bufs

    # ---- decode (config: batch 256, H=16, K=V=128, 4096-token prefill, 512 steps)
    decode = None
    if not args.no_decode:
        del plan
        torch.cuda.empty_cache()
        decode = run_decode(torch, ops, dev, rank, world, dist)
    sp = None
    if not args.no_sp:
        torch.cuda.empty_cache()
        sp = run_sp(torch, dev, rank, world, dist)
    dh = None
    if not args.no_dhead:
        torch.cuda.empty_cache()
        dh = run_dhead(torch, ops, dev, rank, world, dist)
    sh = None
    if not args.no_short:
        torch.cuda.empty_cache()
        sh = run_short(torch, ops, dev, rank, world, dist)
    gd = None
    if not args.no_gdn:
        torch.cuda.empty_cache()
        gd = run_gdn(torch, ops, dev, rank, world, dist)
    ly = lt = None
    if not args.no_layer:
        torch.cuda.empty_cache()
        ly = run_layer(torch, dev, rank, world, dist)
        if world > 1:
            torch.cuda.empty_cache()
            lt = run_layer_tp(torch, dev, rank, world, dist)
    lmr = None
    if not args.no_lm:
        torch.cuda.empty_cache()
        lmr = run_lm(torch, dev, rank, world, local_rank, dist)
    return dict(ms_step=ms_step, fwd_ms=fwd_ms, bwd_ms=bwd_ms, zero_ms=zero_ms, clocks=clk, e2e=e2e,
                decode=decode, sp=sp, dhead=dh, short=sh, gdn=gd, layer=ly, layer_tp=lt, lm=lmr)


def run_decode(torch, ops, dev, rank, world, dist):
    D = DECODE
    B, T, H, Mh, V, n = D["B"], D["T"], D["H"], D["Mh"], D["V"], D["steps"]
    x = make_inputs(torch, 777 + rank, dev, B, T, H, Mh, V, torch.bfloat16, with_grad_out=False)
    with torch.no_grad():
        _, S = ops.phase_scan(x["phw"], x["phq"], x["v"], x["beta"], None, x["lam"], x["wr"], x["wi"])
    del x
    torch.cuda.empty_cache()
    y = make_inputs(torch, 999 + rank, dev, B, n, H, Mh, V, torch.float32, with_grad_out=False)
    S = S.contiguous()
    plan = ops.PhaseStepPlan(y["phw"], y["phq"], y["v"], y["beta"], None, y["lam"], y["wr"], y["wi"], S)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for t in range(3):
            plan.step(t)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for t in range(n):
            plan.step(t)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st = torch.cuda.current_stream()
    e0.record(st)
    graph.replay()
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    us_step = ms * 1e3 / n
    state_bytes = B * H * 2 * Mh * V * 4
    io_bytes = B * H * (2 * Mh * 4 + V * 4 + 4 + 2 * V * 4)
    gbs = (2 * state_bytes + io_bytes) / (us_step * 1e-6) / 1e9
    del graph
    return {"value": world * B * n / (ms / 1e3), "unit": "tokens/s", "us_per_step": us_step,
            "config": {"batch": B, "H": H, "K": 2 * Mh, "V": V, "prefill": T, "steps": n},
            "achieved_gbs": gbs, "bytes_per_step": 2 * state_bytes + io_bytes}


def sp_slab(torch, dev, r, T, S=SP):
    """Inputs of slab r (tokens [r T, (r + 1) T)) of the long sequence: per-token inputs from
    seed 555 + r with positions continuing the previous slabs, and the per-head parameters
    (lam, wr, wi) from one seed shared by every slab."""
    x = make_inputs(torch, 555 + r, dev, S["B"], T, S["H"], S["Mh"], S["V"], torch.bfloat16, with_grad_out=False)
    om = math.pi * 1e4 ** (-torch.arange(S["Mh"], device=dev, dtype=torch.float32) / (S["Mh"] - 1))
    x["phw"] += (r * T) * om
    x["phq"] += (r * T) * om
    shared = make_inputs(torch, 555, dev, 1, 1, S["H"], S["Mh"], S["V"], torch.bfloat16, with_grad_out=False)
    x.update(lam=shared["lam"], wr=shared["wr"], wi=shared["wi"])
    return x


def sp_parity(torch, ops, dev, rank, world, dist, T_rank=4096, H=4):
    """Correctness of the sequence-parallel prefill across the ranks, on a problem whose state
    carries across the slabs: additive write, no decay on half the modes (the LapA long head's
    persistent half), 1/16 on the rest, T_rank tokens per rank, H heads.  Every rank runs the
    sequence-parallel prefill of its slab, regenerates every slab and runs the single-GPU scan of
    the whole sequence, and compares its outputs (unit-RMS max-abs, cosine) and the final state
    (relative error) at the bf16 bar.  (The benchmark's own inputs forget within about 16 tokens,
    so there the slabs' incoming states vanish and the comparison would be trivially exact.)"""
    from sca2_b200.sp import sp_phase_prefill
    Mh, V = SP["Mh"], SP["V"]
    om = math.pi * 1e4 ** (-torch.arange(Mh, device=dev, dtype=torch.float32) / (Mh - 1))

    def slab(r):
        x = make_inputs(torch, 900 + r, dev, 1, T_rank, H, Mh, V, torch.bfloat16, with_grad_out=False)
        return x["phw"] + (r * T_rank) * om, x["phq"] + (r * T_rank) * om, x["v"]
    shared = make_inputs(torch, 900, dev, 1, 1, H, Mh, V, torch.bfloat16, with_grad_out=False)
    lam = torch.full((H, Mh), 1.0 / 16, device=dev)
    lam[:, : Mh // 2] = 0.0
    wr, wi = shared["wr"], shared["wi"]
    phw, phq, v = slab(rank)
    o, S_end = sp_phase_prefill(phw, phq, v, None, None, lam, wr, wi)
    parts = [slab(r) for r in range(world)]
    with torch.no_grad():
        ro, rS = ops.phase_scan(*(torch.cat([p[k] for p in parts], 1) for k in range(3)), None, None, lam, wr, wi)
    a, b = o.float(), ro[:, rank * T_rank:(rank + 1) * T_rank].float()
    err = float((a - b).abs().max() / b.abs().max())  # max-abs over max |reference| of the raw read
    cos = float((a * b).sum() / (a.norm() * b.norm()))
    rms = lambda t: t / t.square().mean(-1, keepdim=True).add(1e-6).sqrt()
    err_u = float((rms(a.reshape(1, T_rank, H, -1)) - rms(b.reshape(1, T_rank, H, -1))).abs().max())
    s_err = float((S_end - rS).abs().max() / rS.abs().max())
    ok = err < 2e-2 and cos > 0.9999 and s_err < 2e-2
    flags = torch.tensor([0.0 if ok else 1.0, err, 1.0 - cos, s_err, err_u], device=dev)
    if dist is not None:
        dist.all_reduce(flags, op=dist.ReduceOp.MAX)
    return {"parity_ok": bool(flags[0] == 0),
            "parity": {"case": f"additive write, lam 0 on half the modes and 1/16 on the rest, {T_rank} tokens "
                               f"per rank, H={H}, bf16 values",
                       "vs": "single-GPU scan of the whole sequence",
                       "bar": "read: max-abs / max |ref| < 2e-2 and cosine > 0.9999; final state: relative < 2e-2",
                       "read_rel": float(flags[1]), "one_minus_cosine": float(flags[2]),
                       "final_state_rel": float(flags[3]), "read_unit_rms_max_abs": float(flags[4])}}


def run_sp(torch, dev, rank, world, dist, reps=7):
    """Sequence-parallel prefill of one 131072-token sequence (bf16 v, fp32 state): every rank
    holds T / N tokens; slab maps all-gathered over NCCL.  Each prefill is timed on its own
    (CUDA events on the launching stream); the reported time is the median over the prefills
    of the max over ranks, so one prefill held up by the host (the prefill is a few dozen
    launches around two scans) does not set the number; every prefill's time is listed.
    Afterwards sp_parity checks the cross-rank path on a long-memory problem; parity_ok holds
    on every rank or is false."""
    from sca2_b200 import ops
    from sca2_b200.sp import sp_phase_prefill
    S = SP
    T = S["T"] // world
    x = sp_slab(torch, dev, rank, T, S)
    args = (x["phw"], x["phq"], x["v"], x["beta"], None, x["lam"], x["wr"], x["wi"])
    for _ in range(2):
        sp_phase_prefill(*args)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    st = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for e0, e1 in ev:
        e0.record(st)
        o, S_end = sp_phase_prefill(*args)
        e1.record(st)
    torch.cuda.synchronize()
    each = [e0.elapsed_time(e1) for e0, e1 in ev]
    if dist is not None:
        t = torch.tensor(each, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        each = [float(v) for v in t.tolist()]
    ms = statistics.median(each)
    del x, args
    out = {"value": S["B"] * S["T"] / (ms / 1e3), "unit": "tokens/s", "ms_per_prefill": ms,
           "ms_each": [round(v, 3) for v in each], "timing": "median over prefills of the max over ranks",
           "config": {"batch": S["B"], "seq_len": S["T"], "tokens_per_rank": T, "H": S["H"], "d_head": 2 * S["Mh"],
                      "ranks": world, "fwd_only": True}}
    out.update(sp_parity(torch, ops, dev, rank, world, dist))
    return out


def _quiet_stdout(fn):
    """Run fn with file descriptor 1 on /dev/null (C-level prints included)."""
    import ctypes
    sys.stdout.flush()
    saved, null = os.dup(1), os.open(os.devnull, os.O_WRONLY)
    os.dup2(null, 1)
    try:
        return fn()
    finally:
        try:
            ctypes.CDLL(None).fflush(None)
        except OSError:
            pass
        os.dup2(saved, 1)
        os.close(saved)
        os.close(null)


def run_dhead(torch, ops, dev, rank, world, dist, reps=5):
    """D-head diagonal scan fwd+bwd (separable read, fp32) on the reference layer's D-head
    shape; algorithmic bytes: fwd reads a (2 M G), v (V), c (2 M) and writes [A|Bv] (2 V)
    fp32 per token, bwd re-reads the inputs, reads d[A|Bv] and writes every input gradient."""
    D = DHEAD
    B, T, M, G, V = D["B"], D["T"], D["M"], D["G"], D["V"]
    g = torch.Generator(device=dev).manual_seed(31 + rank)
    rn = lambda *sh: torch.randn(*sh, device=dev, generator=g)
    ph = rn(B, T, M, G)
    mag = torch.exp(-torch.nn.functional.softplus(rn(B, T, M, G)))
    x = [(mag * torch.cos(ph)).requires_grad_(True), (mag * torch.sin(ph)).requires_grad_(True),
         rn(B, T, V).requires_grad_(True), rn(B, T, M).requires_grad_(True), rn(B, T, M).requires_grad_(True)]
    dab = rn(B, T, 2, V)

    def step():
        ab, (sr, si) = ops.dscan(*x, sep=True)
        torch.autograd.backward(ab, dab)
    for _ in range(3):
        step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        step()
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    fwd_b = (2 * M * G + V + 2 * M + 2 * V) * 4
    bwd_b = fwd_b - 2 * V * 4 + 2 * V * 4 + (2 * M * G + V + 2 * M) * 4
    gbs = (fwd_b + bwd_b) * B * T / (ms * 1e-3) / 1e9
    return {"value": world * B * T / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
            "config": {"batch": B, "seq_len": T, "M": M, "G": G, "dv": V, "read": "separable", "fwd+bwd": True},
            "achieved_gbs": gbs, "algorithmic_bytes_per_step": (fwd_b + bwd_b) * B * T}


def run_gdn(torch, ops, dev, rank, world, dist, reps=3):
    """Delta-rule scan in the gated-delta-rule form (explicit keys, K = V = 128), fwd+bwd,
    bf16 q/k/v/dO with fp32 state; q, k L2-normalised per head, beta = sigmoid(N(0,1)),
    g = -softplus(N(0,1)).  Algorithmic bytes per token and head: fwd q, k, v (3 x 128 bf16)
    + g, beta (2 x 4) read, o (128 bf16) written = 1,032 B; bwd dO read, inputs re-read,
    dq, dk, dv, dg, dbeta written = 1,808 B."""
    D = GDN
    B, T, H, K, V = D["B"], D["T"], D["H"], D["K"], D["V"]
    gen = torch.Generator(device=dev).manual_seed(51 + rank)
    rn = lambda *sh: torch.randn(*sh, device=dev, generator=gen)
    nrm = lambda x: (x / x.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    q = nrm(rn(B, T, H, K)).requires_grad_(True)
    k = nrm(rn(B, T, H, K)).requires_grad_(True)
    v = rn(B, T, H, V).to(torch.bfloat16).requires_grad_(True)
    beta = torch.sigmoid(rn(B, T, H)).requires_grad_(True)
    g = (-torch.nn.functional.softplus(rn(B, T, H))).requires_grad_(True)
    dO = rn(B, T, H, V).to(torch.bfloat16)

    def step():
        o, _ = ops.key_scan(q, k, v, g, beta)
        torch.autograd.backward(o, dO)
        for t in (q, k, v, beta, g):
            t.grad = None
    ms = _timed(torch, dist, dev, step, reps)
    fwd_b, bwd_b = 3 * K * 2 + 8 + V * 2, V * 2 + (3 * K * 2 + 8) + (3 * K * 2 + 8)
    tokh = B * T * H
    mac = FWD_MAC_TOK(K, V, R=1) * tokh
    hbm = peaks()[0]
    gbs = (fwd_b + bwd_b) * tokh / (ms * 1e-3) / 1e9
    return {"value": world * B * T / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
            "config": {"batch": B, "seq_len": T, "heads": H, "d_k": K, "d_v": V, "dtype": "bf16",
                       "form": "gated delta rule (v_times_beta), scalar decay g", "fwd+bwd": True},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                         "basis": "algorithmic bytes of the whole fwd+bwd step / step time"},
            "achieved_gbs": gbs,
            "algorithmic_bytes_per_step": (fwd_b + bwd_b) * tokh,
            "achieved_tflops": 3 * 2 * mac / (ms * 1e-3) / 1e12}


def _timed(torch, dist, dev, fn, reps):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        fn()
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def _graph_timed(torch, dist, dev, fn, reps):
    """Time `fn` (a forward + backward of small kernels, whose Python launch cost would
    otherwise exceed their GPU time) as replays of one CUDA graph captured from it."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    ms = _timed(torch, dist, dev, graph.replay, reps)
    del graph
    return ms


def run_short(torch, ops, dev, rank, world, dist, reps=10):
    """Short-head window read (fp32) on the LapA short-head shape: prefill fwd+bwd over
    B x T tokens, and one decode token for decode_B sequences.  Algorithmic bytes per token:
    fwd K(h), K(z) (2 L) + V(z) (dv) read, o (2 dv) written; bwd dO (2 dv) read, inputs
    re-read, their gradients written (all fp32)."""
    S = SHORT
    B, T, L, dv = S["B"], S["T"], S["L"], S["dv"]
    n = L - 1
    g = torch.Generator(device=dev).manual_seed(41 + rank)
    rn = lambda *sh: torch.randn(*sh, device=dev, generator=g)
    omega = (torch.arange(L, dtype=torch.float64) * (2 * math.pi / L)).float().to(dev)
    par = [(0.3 * rn(L)).requires_grad_(True), (1 + 0.1 * rn(L)).requires_grad_(True), (0.1 * rn(L)).requires_grad_(True)]
    x = [rn(B, T, L).requires_grad_(True), rn(B, T, L).requires_grad_(True), rn(B, T, dv).requires_grad_(True)]
    ph = rn(B, n, L)
    st = (ph.cos(), ph.sin(), rn(B, n, dv))
    pos = torch.tensor(5, device=dev)
    dO = rn(B, T, 2 * dv)

    def step():
        o, _ = ops.short_read(x[0], x[1], x[2], par[0], omega, par[1], par[2], st, pos)
        torch.autograd.backward(o, dO)
    ms = _graph_timed(torch, dist, dev, step, reps)
    fwd_b = (2 * L + dv + 2 * dv) * 4
    bwd_b = (2 * dv + 2 * L + dv + 2 * L + dv) * 4
    Bd = S["decode_B"]
    xd = [rn(Bd, 1, L), rn(Bd, 1, L), rn(Bd, 1, dv)]
    phd = rn(Bd, n, L)
    std = [phd.cos(), phd.sin(), rn(Bd, n, dv)]

    # one decode token as a CUDA graph (read, then the new ring buffer copied over the old)
    def dbody():
        with torch.no_grad():
            o, new = ops.short_read(xd[0], xd[1], xd[2], par[0], omega, par[1], par[2], tuple(std), pos)
            for a, b in zip(std, new):
                a.copy_(b)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            dbody()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        dbody()
    dms = _timed(torch, dist, dev, graph.replay, 200)
    del graph
    return {"value": world * B * T / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
            "config": {"batch": B, "seq_len": T, "L": L, "dv": dv, "fwd+bwd": True, "dtype": "f32",
                       "cuda_graph": True},
            "achieved_gbs": (fwd_b + bwd_b) * B * T / (ms * 1e-3) / 1e9,
            "algorithmic_bytes_per_step": (fwd_b + bwd_b) * B * T,
            "decode": {"batch": Bd, "us_per_token_step": dms * 1e3, "cuda_graph": True,
                       "tokens_per_s": world * Bd / (dms / 1e3)}}


def _gated_cfg(C, max_len):
    from sca2_b200.layers import LayerCfg
    return LayerCfg(d=C["d"], Mc=C["heads"] * C["Mh"], Md=C["Md"], G=C["G"], ff=C["ff"], freq="rope",
                    theta_scale=0.02, max_len=max_len, dv=C["heads"] * C["dvh"], c_heads=C["heads"], c_decay=True)


def run_layer(torch, dev, rank, world, dist, reps=5):
    """One SCA2 layer (GatedLayer with this package's heads) forward + backward under bf16
    autocast on B x T tokens per GPU: norm, 16-head gated C head (projections, phase scan on
    the tensor-core kernels, read-out), D head, mix, FFN.  Weights N(0, 0.02^2)."""
    from sca2_b200 import layers, lm as L
    C = LAYER
    torch.manual_seed(7 + rank)
    layer = layers.GatedLayer(_gated_cfg(C, C["T"])).to(dev)
    L.init_weights(layer)
    x = torch.randn(C["B"], C["T"], C["d"], device=dev, requires_grad=True)
    dy = torch.randn(C["B"], C["T"], C["d"], device=dev)

    def step():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = layer(x)
        torch.autograd.backward(y, dy)
    ms = _timed(torch, dist, dev, step, reps)
    n_par = sum(p.numel() for p in layer.parameters())
    tok = C["B"] * C["T"]
    return {"value": world * tok / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
            "config": {"layer": "GatedLayer", "batch": C["B"], "seq_len": C["T"], "d_model": C["d"],
                       "heads": C["heads"], "d_head": 2 * C["Mh"], "ff": C["ff"], "dtype": "bf16 autocast",
                       "fwd+bwd": True},
            "params": n_par}


def run_layer_tp(torch, dev, rank, world, dist, reps=5):
    """The GatedLayer of the layer block with its 16 C heads sharded over the N ranks
    (tensor-parallel heads, sca2_b200.tp) for a batch smaller than N: B = 1, T = 4096, bf16
    autocast, forward + backward with the sharded gradients summed; time = max over ranks."""
    from sca2_b200 import layers, lm as L, tp
    C = LAYER
    torch.manual_seed(7)  # the same weights on every rank
    layer = tp.shard_layer(layers.GatedLayer(_gated_cfg(C, C["T"])).to(dev), None)
    L.init_weights(layer)
    g = torch.Generator(device=dev).manual_seed(8)
    x = torch.randn(1, C["T"], C["d"], device=dev, generator=g, requires_grad=True)
    dy = torch.randn(1, C["T"], C["d"], device=dev, generator=g)

    def step():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = layer(x)
        torch.autograd.backward(y, dy)
        tp.reduce_sharded_grads(layer)
    ms = _timed(torch, dist, dev, step, reps)
    return {"value": C["T"] / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
            "config": {"layer": "GatedLayer, C heads sharded over the ranks", "batch": 1, "seq_len": C["T"],
                       "d_model": C["d"], "heads": C["heads"], "heads_per_rank": C["heads"] // world,
                       "ranks": world, "dtype": "bf16 autocast", "fwd+bwd": True}}


def run_lm(torch, dev, rank, world, local_rank, dist):
    """12-layer SCA2 LM training step (GatedLM) with AdamW under bf16 autocast, DDP over the
    ranks when N > 1 (gradient all-reduce over NCCL, overlapped with the backward); then
    greedy decoding of decode_B sequences with the whole stack's step in one CUDA graph."""
    from sca2_b200 import lm as L
    C = LMCFG
    torch.manual_seed(11)
    model = L.GatedLM(C["vocab"], _gated_cfg(C, C["T"]), n_layers=C["n_layers"]).to(dev)
    L.init_weights(model)
    n_par = sum(p.numel() for p in model.parameters())
    net = model
    if dist is not None:
        net = torch.nn.parallel.DistributedDataParallel(model, device_ids=[local_rank])
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, fused=True)
    tok = L.zipf_tokens(C["B"], C["T"] + 1, C["vocab"], seed=100 + rank, device=dev)
    for _ in range(C["warmup"]):
        L.train_step(net, opt, tok)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(C["steps"]):
        loss = L.train_step(net, opt, tok)
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / C["steps"]
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    tokens = C["B"] * C["T"]
    flops = 6.0 * n_par * tokens * world
    bf16_peak = _bf16_sustained()
    out = {"value": world * tokens / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
           "loss": float(loss),
           "config": {"model": "GatedLM (12 x GatedLayer)", "n_layers": C["n_layers"], "d_model": C["d"],
                      "heads": C["heads"], "d_head": 2 * C["Mh"], "vocab": C["vocab"], "ff": C["ff"],
                      "seq_len": C["T"], "batch_per_gpu": C["B"], "dtype": "bf16 autocast", "optimizer": "AdamW",
                      "data": "Zipf(1.1) token ids, seeded", "parallelism": f"ddp{world}" if world > 1 else "single"},
           "params": n_par,
           "model_tflops_per_s": flops / (ms * 1e-3) / 1e12,
           "frac_of_bf16_peak": (flops / (ms * 1e-3) / 1e12) / (world * bf16_peak[0]),
           "bf16_peak_tflops": bf16_peak[0], "bf16_peak_source": bf16_peak[1],
           "flop_convention": "6 x parameters x tokens (scan FLOP not added)"}
    del opt, net
    torch.cuda.empty_cache()
    # decode: prefill a prompt, then greedy tokens from one CUDA graph of the whole step
    Bd = C["decode_B"]
    model.eval()
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16, cache_enabled=False):
        prompt = L.zipf_tokens(Bd, C["prompt"], C["vocab"], seed=200 + rank, device=dev)
        logits, state = model.prefill(prompt)
        dec = L.GraphDecoder(model, state)
        first = logits[:, -1].argmax(-1)
        for _ in range(3):
            dec.step(first)
        torch.cuda.synchronize()
        e0.record(st)
        tok_ = first
        for _ in range(C["decode_steps"]):
            tok_ = dec.step(tok_)
        e1.record(st)
        torch.cuda.synchronize()
    dms = e0.elapsed_time(e1) / C["decode_steps"]
    if dist is not None:
        t = torch.tensor([dms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dms = float(t.item())
    out["decode"] = {"batch": Bd, "prompt": C["prompt"], "ms_per_token_step": dms,
                     "tokens_per_s": world * Bd / (dms / 1e3), "cuda_graph": True}
    del dec
    return out


def _traffic(kernel, B):
    """DRAM bytes per launch of `kernel` from the committed ncu summary (captured at B=2,
    scaled by the number of sequences), or None."""
    try:
        with open(os.path.join(ROOT, "profiles", "roofline_traffic.json")) as f:
            t = json.load(f)
        return t[kernel]["captured_bytes_B2"] * B / 2
    except Exception:
        return None


def _bf16_sustained():
    """bf16 dense peak for a kernel mix timed inside a long step: the sustained cuBLAS figure."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return float(m.get("bf16_tflops_sustained", m["bf16_tflops"])), "measured (sustained)"
    except Exception:
        return 1400.0, "fallback (sustained)"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return float(m["hbm_gbs"]), float(m["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-sp", action="store_true")
    ap.add_argument("--no-dhead", action="store_true")
    ap.add_argument("--no-short", action="store_true")
    ap.add_argument("--no-layer", action="store_true")
    ap.add_argument("--no-lm", action="store_true")
    ap.add_argument("--no-gdn", action="store_true")
    ap.add_argument("--gdn-only", action="store_true",
                    help="run only the delta-rule (K = V = 128) block on one GPU and print its JSON (profiling)")
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences per GPU (default 8); smaller values make profiler-sized cases")
    args = ap.parse_args()
    if args.batch is not None:
        WORK["B"] = args.batch

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    W = WORK
    if args.gdn_only:
        import torch
        from sca2_b200 import ops
        dev = torch.device("cuda", local_rank)
        torch.cuda.set_device(dev)
        print(json.dumps({"gdn_delta": run_gdn(torch, ops, dev, 0, 1, None, reps=max(1, args.steps))}))
        return
    config = {"workload": "LapA long-head phase-coded delta scan fwd+bwd (phases, per-mode decay, "
                          f"delta gate), B={WORK['B']} T=4096 H=16 d_head=64 (Mh=32, K=V=64) per GPU",
              "batch_per_gpu": W["B"], "seq_len": W["T"], "heads": W["H"], "d_head": 2 * W["Mh"],
              "parallelism": f"(batch x head) shards, {world} rank(s)",
              "l2": "inputs larger than L2 (~0.7 GB touched per step), no flush"}

    if args.impl == "reference":
        if rank != 0:
            return
        pool, n = cpu_pool()
        try:
            cpu_sample(pool, n, seed=0)  # warm the workers
            for i in range(args.warmup):
                cpu_sample(pool, n, seed=1 + i)
            vals, walls = [], []
            for i in range(args.steps):
                v, w, nseq = cpu_sample(pool, n, seed=100 + i)
                vals.append(v)
                walls.append(w)
        finally:
            pool.close()
        tot = sum(walls)
        value = args.steps * nseq * W["T"] / W["H"] / tot
        line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": 1e3 * tot / args.steps, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
                "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": n, "kind": "port",
                                 "sample": f"{nseq} (b,h) sequences x {W['T']} tokens fwd+bwd per step, "
                                           f"numpy oracle float32, one process per core"},
                "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    # CPU pool first (spawned before any CUDA work)
    pool = None
    if rank == 0 and world == 1 and not args.no_cpu:
        pool, ncpu = cpu_pool()
    dist = None
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist_

        def setup():  # NCCL prints a banner on the first communicator; keep stdout to the JSON line
            dist_.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                     device_id=torch.device("cuda", local_rank))
            dist_.barrier()
        _quiet_stdout(setup)
        dist = dist_
    try:
        r = run_gpu(args, rank, world, local_rank, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()
    if rank != 0:
        if pool is not None:
            pool.close()
        return
    cpu = None
    if pool is not None:
        try:
            cpu_sample(pool, ncpu, seed=0)
            v, w, nseq = cpu_sample(pool, ncpu, seed=7)
            cpu = {"value": v, "unit": "tokens/s", "cores": ncpu, "kind": "port",
                   "sample": f"{nseq} (b,h) sequences x {W['T']} tokens fwd+bwd (of the {W['B'] * W['H']} "
                             f"per step), numpy oracle float32, one process per core, {w:.1f} s wall"}
        finally:
            pool.close()

    hbm, tfl, src = peaks()
    tokh = W["B"] * W["T"] * W["H"]
    fwd_b, bwd_b = FWD_BYTES_TOK(W["Mh"], W["V"]) * tokh, BWD_BYTES_TOK(W["Mh"], W["V"]) * tokh
    kern = {"scan_fwd": (r["fwd_ms"], fwd_b), "scan_bwd": (r["bwd_ms"], bwd_b)}
    name = max(kern, key=lambda k: kern[k][0])
    ms, by = kern[name]
    achieved = by / (ms * 1e-3) / 1e9
    mac = FWD_MAC_TOK(2 * W["Mh"], W["V"]) * tokh
    line = {
        "metric": METRIC, "value": world * W["B"] * W["T"] / (r["ms_step"] / 1e3),
        "metric_note": "the scan op alone (the hot path: LapA long-head scan forward + backward); the "
                       "whole GatedLayer step (projections, D head, mix, FFN under torch) is the 'layer' "
                       "block and the 12-layer LM step the 'lm_train' block",
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": r["ms_step"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic", "config": config,
        "roofline": {"bound": "hbm", "kernel": name, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "peak_source": f"{src} (MEASURED_PEAKS.json hbm_gbs)",
                     "traffic": _traffic(name, W["B"]), "traffic_source": "ncu dram bytes per launch, "
                     "profiles/roofline_traffic.json (B=2 capture x B/2)",
                     "algorithmic_bytes_per_launch": by, "ms_per_launch": ms},
        "kernels_ms": {"scan_fwd": r["fwd_ms"], "grad_zero_fill": r["zero_ms"], "scan_bwd": r["bwd_ms"]},
        "flops": {"algorithmic_tflop_per_step": 3 * 2 * mac / 1e12,
                  "achieved_tflops": 3 * 2 * mac / (r["ms_step"] * 1e-3) / 1e12, "peak_tflops": tfl},
        "cpu_baseline": cpu, "e2e": r["e2e"], "clocks": r["clocks"], "gpu_launches": 3 * args.steps,
        "decode": r["decode"],
        "sp_prefill": r["sp"],
        "d_head": r["dhead"],
        "short_head": r["short"],
        "gdn_delta": r["gdn"],
        "layer": r["layer"],
        "layer_tp": r["layer_tp"],
        "lm_train": r["lm"],
    }
    print(json.dumps(line))


if __name__ == "__main__":
    main()

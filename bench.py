#!/usr/bin/env python
"""GDN-2 B200 benchmark (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Headline workload (the configuration the north star's
1 -> 8 GPU target is quoted on): chunkwise GDN-2 forward + backward, bf16
activations, fp32 decay / state / accumulation, B=1 T=262,144 H=32 K=V=128,
chunk 64, scalar beta and log-decay per (token, head) broadcast through the
channel-wise API, seeded synthetic inputs (no dataset is involved).  A step
is one forward and one backward over the whole sequence.  The total work is
fixed as N grows (strong scaling): at N=1 the step is ``chunk_gdn2`` + its
backward on one GPU (which runs one sequence with 32 heads overlapped: the
sequence cut into 16 pieces whose state passes run on a second stream beside
the intra-chunk kernels of the neighbouring pieces); at N>1 rank r owns
tokens [r T/N, (r+1) T/N) and runs
``chunk_gdn2_cp`` (span pre-scan, one NCCL all-gather of the span maps per
direction, merge, state pass).  The inputs are drawn in 4,096-token blocks
with one seed per block, so every N times the same sequence.  The reported
time is the max over ranks.

* ``value``: tokens/s of the whole job with inputs resident in HBM, through
  the public API with autograd; every library phase is bracketed by CUDA
  events on the launch stream (``phase_timing``), which gives the per-phase
  breakdown and the live roofline of the dominant kernel.  On the overlapped
  path the phases overlap, so their sum exceeds the step; the roofline's
  ``achieved`` then comes from the dominant kernel's launches that had the
  GPU to themselves, and ``all_launches`` gives the figure over every one.
* ``e2e``: the same step as a training step sees it: every step copies its
  inputs from pinned host memory -- this rank's q, k, v, the upstream
  gradient dO, and the per-(token, head) beta and log-decay, broadcast
  channel-wise on the device -- runs the forward, forms the loss
  sum(o * dO), runs the backward into device gradients and reads the loss
  back to the host.  The next step's copy runs on a second stream while the
  current step computes; every copy is inside the timed region.
* ``sp_parity`` (N>1): rel-L2 of two heads' outputs, final state and all six
  input gradients, gathered over the ranks, against ``chunk_gdn2`` run on the
  whole sequence of those heads on rank 0's GPU.
* ``heads`` (N>1): the head-sharded variant of config 4 (H/N heads of the
  whole sequence per rank, no collective).
* ``config1``: BASELINE config 1 (B=8 T=4096 H=16, fwd+bwd) per rank, batch-
  sharded (weak), its four kernel phases through the C ABI with their own
  roofline, its own end-to-end leg and CPU baseline.
* ``decode``: BASELINE config 2 (B=256 H=16 K=V=128 fp32 state, in-place
  recurrent step, bf16 inputs), state read+write GB/s, and the CPU decode
  step timed beside it.
* ``config3``: BASELINE config 3, a 24-layer decoder (hidden 2048, 16 heads
  of 128, SwiGLU 5632, vocab 151,936, bf16) with the drop-in block in every
  layer: one optimizer step over B=8 x T=8192 token ids per GPU, data-
  parallel (DDP, NCCL gradient all-reduce) at N>1; tokens/s/GPU.
* ``config0``: BASELINE config 0 (fp32 forward, B=1 T=512 H=4 K=V=64): GPU
  latency of ``chunk_gdn2`` and the CPU chunk and recurrent paths' times.
* ``block_ops``: the block's prologue / epilogue kernels at config-1 shapes.
* ``cpu_baseline``: the reference algorithm's CPU path (PyTorch restatement
  in oracle/gdn2_torch_port.py, fp32, autograd backward), all host threads,
  on a bounded slice of the workload; rank 0 at N=1 only.

``--impl reference`` times only that CPU path (the reference itself is pure
Python and cannot run on the GPU box), on the same metric and unit.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

K, V, C = 128, 128, 64
B1, T1, H1 = 8, 4096, 16            # config 1
T4, H4, BLOCK4 = 262144, 32, 4096   # config 4 and its input block
DEC_B, DEC_H, DEC_STEPS, DEC_SETS = 256, 16, 1024, 32
FALLBACK_HBM_GBS, FALLBACK_TFLOPS = 6650.0, 1590.0
PARITY_HEADS = (0, 17)

# Algorithmic bytes per token-head moved by each kernel (bf16 token tensors,
# fp32 decay/gl, 64-token chunks, K = V = 128):
#   fwd_intra : reads q,k,b,v,w (5x256) + g (512); writes Qg,Kd,W,U (4x256)
#               + Aqk, A (2x128) + gl (8)                               = 3080
#   fwd_state : reads Qg,Kd,W (768) + U (256) + Aqk (128) + gl (8);
#               writes o (256) + VN (256) + h checkpoint (K*V*2/64 = 512) = 2184
#   bwd_state : reads Qg,Kd,W,Aqk,gl (904) + dO (256);
#               writes dh checkpoint (512) + dVN (256)                  = 1928
#   bwd_intra : reads q,k,b,g,v,w (1792) + dO (256) + A (128) + VN (256)
#               + h (512) + dh (512) + dVN (256) + gl (8);
#               writes dq,dk,db (768) + dg (512) + dv,dw (512)          = 5512
PHASE_BYTES = {"fwd_intra": 3080, "fwd_state": 2184, "bwd_state": 1928, "bwd_intra": 5512}
# Algorithmic FLOPs per token-head (C = 64, K = V = 128), for context.
PHASE_FLOPS = {
    "fwd_intra": 6 * C * K + 2 * C * V,
    "fwd_state": 6 * K * V + 2 * C * V,
    "bwd_state": 6 * K * V + 2 * C * V,
    "bwd_intra": 6 * K * V + 6 * C * V + 12 * C * K + 4 * C * C,
}
# Library phases that are one kernel launch each (the rest of a step's
# phases -- the span-map folds, the NCCL all-gathers -- are torch / NCCL).
NATIVE_PHASES = ("fwd_intra", "fwd_prescan", "fwd_merge", "fwd_unfold", "fwd_state",
                 "bwd_prescan", "bwd_merge", "bwd_unfold", "bwd_state", "bwd_intra")
# The metric's "% TC peak": the reference schedule's fwd+bwd FLOPs per
# token-head, 20CK + 14CV + 22KV + 4C^2 = 655,360, over the step time, against
# the measured bf16 peak and against the HBM-limited ceiling min(peak, AI x
# HBM GB/s) with AI = 655,360 / 6,900 minimum bytes per token-head.
STEP_FLOPS = 20 * C * K + 14 * C * V + 22 * K * V + 4 * C * C
STEP_MIN_BYTES = 6900
# DRAM traffic (read + write) of the dominant kernel, k_bwd_intra16, per
# token-head, from ncu --set full captures: a config-4-shaped slice (B=1,
# T=32,768, H=32: 5.743 GB over 1,048,576 token-heads) and config-1 shapes at
# batch 2 (689.5 MB over 131,072 token-heads).  The kernel runs one CTA per
# (chunk, head) whatever the sequence layout, so its traffic grows with
# token-heads and scales to a full config-4 or config-1 launch.  Summaries
# under profiles/.
NCU_TRAFFIC_PER_TOKEN_HEAD = {"config4": 5476.6, "config1": 5260.8}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops", 1643.0)), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_TFLOPS, "fallback"


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def host_threads():
    """Cores this process may run on (the container's share, not the host's)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------
# clocks sampling during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        time.sleep(0.3)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sms, mx, reasons = [], 0.0, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sms:
            return None
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sms)}


# ---------------------------------------------------------------------------
# inputs
# ---------------------------------------------------------------------------
def _draw(gen, dev, shape_bt, H):
    """One block of the config-0 recipe: q, k ~ N(0,1) L2-normalised, v ~
    N(0,1), beta = sigmoid(N(0,1)), g = logsigmoid(N(3,1)) per token and
    head, dO ~ N(0,1).  Returns bf16 q, k, v, dO, fp32 beta and g."""
    Bs, Ts = shape_bt
    bf = torch.bfloat16
    q = F.normalize(torch.randn(Bs, Ts, H, K, device=dev, generator=gen), dim=-1).to(bf)
    k = F.normalize(torch.randn(Bs, Ts, H, K, device=dev, generator=gen), dim=-1).to(bf)
    v = torch.randn(Bs, Ts, H, V, device=dev, generator=gen).to(bf)
    beta = torch.sigmoid(torch.randn(Bs, Ts, H, device=dev, generator=gen))
    gs = F.logsigmoid(torch.randn(Bs, Ts, H, device=dev, generator=gen) + 3.0)
    do = torch.randn(Bs, Ts, H, V, device=dev, generator=gen).to(bf)
    return dict(q=q, k=k, v=v, do=do, beta=beta, gs=gs)


def broadcast_gates(beta, gs):
    """Channel-wise b, w (token dtype) and g (fp32) from per-(token, head)
    beta and log-decay, as the reference module's scalar gates reach the
    kernel API."""
    Bs, Ts, H = beta.shape
    b = beta[..., None].expand(Bs, Ts, H, K).to(torch.bfloat16).contiguous()
    w = beta[..., None].expand(Bs, Ts, H, V).to(torch.bfloat16).contiguous()
    g = gs.float()[..., None].expand(Bs, Ts, H, K).contiguous()
    return b, w, g


def make_config1(device, seed):
    """Config-1 inputs [B1, T1, H1, *] (config-0 recipe), plus the per-(token,
    head) beta (bf16) and log-decay the host holds for the end-to-end leg."""
    gen = torch.Generator(device=device).manual_seed(seed)
    d = _draw(gen, device, (B1, T1), H1)
    b, w, g = broadcast_gates(d["beta"], d["gs"])
    x = dict(q=d["q"], k=d["k"], v=d["v"], g=g, b=b, w=w, do=d["do"])
    return x, dict(beta=d["beta"].to(torch.bfloat16), g=d["gs"])


def config4_scalars(dev, t0, t1, heads=None):
    """Config-4 inputs for tokens [t0, t1) (multiples of BLOCK4) and the given
    heads (all 32 when None): every 4,096-token block is drawn for all heads
    from its own seed, so any split of the sequence sees the same data.
    Returns bf16 q, k, v, dO and per-(token, head) beta (bf16) and g (fp32)."""
    hs = list(range(H4)) if heads is None else list(heads)
    n = t1 - t0
    bf = torch.bfloat16
    out = dict(q=torch.empty(1, n, len(hs), K, device=dev, dtype=bf),
               k=torch.empty(1, n, len(hs), K, device=dev, dtype=bf),
               v=torch.empty(1, n, len(hs), V, device=dev, dtype=bf),
               do=torch.empty(1, n, len(hs), V, device=dev, dtype=bf),
               beta=torch.empty(1, n, len(hs), device=dev, dtype=bf),
               g=torch.empty(1, n, len(hs), device=dev, dtype=torch.float32))
    for blk in range(t0 // BLOCK4, t1 // BLOCK4):
        gen = torch.Generator(device=dev).manual_seed(1000 + blk)
        d = _draw(gen, dev, (1, BLOCK4), H4)
        a = blk * BLOCK4 - t0
        sl = slice(a, a + BLOCK4)
        for n_ in ("q", "k", "v", "do"):
            out[n_][:, sl] = d[n_][:, :, hs]
        out["beta"][:, sl] = d["beta"][:, :, hs].to(bf)
        out["g"][:, sl] = d["gs"][:, :, hs]
    return out


def leaves_of(x):
    """Differentiable channel-wise API inputs from the scalar-gate draw."""
    b, w, g = broadcast_gates(x["beta"], x["g"])
    return [t.detach().requires_grad_() for t in (x["q"], x["k"], x["v"], g, b, w)]


# ---------------------------------------------------------------------------
# timing helpers
# ---------------------------------------------------------------------------
def phase_summary(records, steps):
    """Mean ms per step of every phase name (records of ``steps`` steps)."""
    tot: dict[str, float] = {}
    cnt: dict[str, int] = {}
    for name, s, e in records:
        tot[name] = tot.get(name, 0.0) + s.elapsed_time(e)
        cnt[name] = cnt.get(name, 0) + 1
    return {n: {"ms": round(t / steps, 4), "launches": cnt[n]} for n, t in tot.items()}


def roofline_of(phases, token_heads, hbm, peak_kind, shape):
    """Live roofline of the slowest phase with known algorithmic bytes
    (``shape``: "config4" or "config1", the ncu capture its traffic uses)."""
    known = [p for p in PHASE_BYTES if p in phases]
    dom = max(known, key=lambda p: phases[p]["ms"])
    ach = PHASE_BYTES[dom] * token_heads / (phases[dom]["ms"] / 1e3) / 1e9
    per = NCU_TRAFFIC_PER_TOKEN_HEAD.get(shape)
    traffic = round(per * token_heads) if per and dom == "bwd_intra" else None
    for p in known:
        t_s = phases[p]["ms"] / 1e3
        phases[p]["GBps"] = round(PHASE_BYTES[p] * token_heads / t_s / 1e9, 1)
        phases[p]["TFLOPs"] = round(PHASE_FLOPS[p] * token_heads / t_s / 1e12, 2)
    return {"bound": "hbm", "kernel": dom, "achieved": round(ach, 1), "peak": hbm,
            "unit": "GB/s", "frac": round(ach / hbm, 4), "traffic": traffic,
            "peak_source": peak_kind, "bytes_per_token_head": PHASE_BYTES[dom],
            "token_heads_per_launch": token_heads}


def solo_launches(records, t0_event, name="bwd_intra", beside="bwd_state"):
    """Durations (ms) of the ``name`` launches that started after the step's
    last ``beside`` launch had ended, i.e. that had the GPU to themselves.
    On the overlapped path (pieces of one long sequence, state passes on a
    second stream) the earlier ``name`` launches share the SMs with a state
    pass by design.  Times are taken against ``t0_event`` (recorded before
    the first step), so events of both streams compare.  Returns
    ``(solo durations, all durations, launches per step)``."""
    steps, cur = [], []
    for r in records:
        if r[0] == "fwd_intra" and cur and cur[-1][0].startswith("bwd"):
            steps.append(cur)
            cur = []
        cur.append(r)
    if cur:
        steps.append(cur)
    solo, every = [], []
    for st in steps:
        ends = [t0_event.elapsed_time(e) for n, _, e in st if n == beside]
        last = max(ends) if ends else float("-inf")
        for n, s, e in st:
            if n != name:
                continue
            d = s.elapsed_time(e)
            every.append(d)
            if t0_event.elapsed_time(s) >= last:
                solo.append(d)
    per_step = len(every) // max(len(steps), 1)
    return solo, every, per_step


def tc_peak_line(token_heads, ms, peak_tflops, hbm_gbs):
    """Whole-step tensor-core fraction as the metric names it."""
    tf = STEP_FLOPS * token_heads / (ms / 1e3) / 1e12
    ceiling = min(peak_tflops, STEP_FLOPS / STEP_MIN_BYTES * hbm_gbs / 1e3)
    return {"flops_per_token_head": STEP_FLOPS, "tflops": round(tf, 1),
            "frac_of_bf16_peak": round(tf / peak_tflops, 4),
            "hbm_ceiling_tflops": round(ceiling, 1), "frac_of_ceiling": round(tf / ceiling, 4)}


class E2ELoader:
    """Double-buffered host -> device loader for the end-to-end legs: step
    i+1's inputs are copied from pinned host memory on a second stream while
    step i computes."""

    def __init__(self, host, dev, stream):
        self.host = host
        self.stream = stream
        self.bufs = [{n: torch.empty_like(t, device=dev) for n, t in host.items()}
                     for _ in range(2)]
        self.copy_stream = torch.cuda.Stream(dev)
        self.ev_copied = [torch.cuda.Event() for _ in range(2)]
        self.ev_consumed = [torch.cuda.Event() for _ in range(2)]
        self.used = [False, False]
        self.h2d = sum(t.numel() * t.element_size() for t in host.values())

    def issue(self, i, after=None):
        j = i % 2
        with torch.cuda.stream(self.copy_stream):
            if after is not None:
                self.copy_stream.wait_event(after)
            if self.used[j]:
                self.copy_stream.wait_event(self.ev_consumed[j])
            for n, t in self.host.items():
                self.bufs[j][n].copy_(t, non_blocking=True)
            self.ev_copied[j].record(self.copy_stream)
        self.used[j] = True

    def take(self, i):
        j = i % 2
        self.stream.wait_event(self.ev_copied[j])
        return self.bufs[j]

    def release(self, i):
        self.ev_consumed[i % 2].record(self.stream)


def run_e2e(world, dev, host, step_fn, steps, warmup):
    """Time ``steps`` end-to-end steps; ``step_fn(bufs) -> loss`` (device
    scalar).  Returns (ms per step, max over ranks; h2d bytes; d2h bytes)."""
    stream = torch.cuda.current_stream(dev)
    ld = E2ELoader(host, dev, stream)
    loss_host = torch.empty((), dtype=torch.float32, pin_memory=True)

    def run(n, start=None):
        ld.issue(0, start)
        for i in range(n):
            if i + 1 < n:
                ld.issue(i + 1)
            loss = step_fn(ld.take(i))
            loss_host.copy_(loss.detach(), non_blocking=True)
            ld.release(i)

    run(warmup)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    run(steps, e0)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    return ms, ld.h2d, loss_host.numel() * loss_host.element_size()


# ---------------------------------------------------------------------------
# config 4 (headline)
# ---------------------------------------------------------------------------
def config4_step_fn(world, rank):
    from qwendopamine_b200 import chunk_gdn2
    from qwendopamine_b200.gdn2_ops.cp import chunk_gdn2_cp, gather_span_maps

    if world == 1:
        def fwd(leaves):
            o, _ = chunk_gdn2(*leaves, use_qk_l2norm_in_kernel=True)
            return o
    else:
        def fwd(leaves):
            o, _ = chunk_gdn2_cp(*leaves, rank=rank, world=world,
                                 gather=lambda t: gather_span_maps(t, None))
            return o
    return fwd


def run_config4(args, world, rank, local, clocks_out):
    from qwendopamine_b200 import _native as N

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    N.load()
    Tr = T4 // world
    t0 = rank * Tr
    x = config4_scalars(dev, t0, t0 + Tr)
    leaves = leaves_of(x)
    do = x["do"]
    fwd = config4_step_fn(world, rank)

    def step():
        o = fwd(leaves)
        torch.autograd.grad(o, leaves, do)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    barrier(world)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with N.phase_timing() as rec:
        torch.cuda.nvtx.range_push("config4_timed")  # lets a profiler select the timed steps
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    barrier(world)
    if sampler:
        clocks_out.append(sampler.stop())
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    phases = phase_summary(rec, args.steps)
    launches = sum(1 for n, _, _ in rec if n in NATIVE_PHASES)
    solo = solo_launches(rec, e0)
    del rec

    # ---- end to end: host buffers, copies inside the timed region ---------
    host = {n: x[n].cpu().pin_memory() for n in ("q", "k", "v", "do", "beta", "g")}

    def e2e_step(d):
        lv = leaves_of(d)
        o = fwd(lv)
        loss = (o * d["do"]).sum(dtype=torch.float32)
        torch.autograd.grad(loss, lv)
        return loss

    e2e_ms, h2d, d2h = run_e2e(world, dev, host, e2e_step, max(1, min(args.steps, 5)),
                               min(args.warmup, 2))
    del host
    return dict(ms=ms, phases=phases, launches=launches, e2e_ms=e2e_ms, h2d=h2d, d2h=d2h,
                token_heads=Tr * H4, x=x, leaves=leaves, solo=solo)


def sp_parity(world, rank, local, x, fwd):
    """N>1: one more sequence-parallel step on the timed inputs; two heads'
    outputs, final state and input gradients are gathered to rank 0 and
    compared with chunk_gdn2 on the whole sequence of those heads there."""
    import torch.distributed as dist

    from qwendopamine_b200 import chunk_gdn2
    from qwendopamine_b200.gdn2_ops.cp import chunk_gdn2_cp, gather_span_maps

    dev = torch.device("cuda", local)
    hs = list(PARITY_HEADS)
    leaves = leaves_of(x)
    o, ht = chunk_gdn2_cp(*leaves, rank=rank, world=world,
                          gather=lambda t: gather_span_maps(t, None))
    grads = torch.autograd.grad(o, leaves, x["do"])
    parts = {"o": o.detach()[:, :, hs]}
    parts.update({f"d{n}": gr[:, :, hs] for n, gr in zip("qkvgbw", grads)})
    gathered = {n: gather_span_maps(t.contiguous(), None) for n, t in parts.items()}
    ht_last = ht.detach()[:, hs].contiguous()
    dist.broadcast(ht_last, src=world - 1)
    out = None
    if rank == 0:
        full = config4_scalars(dev, 0, T4, heads=hs)
        lv = leaves_of(full)
        o_ref, ht_ref = chunk_gdn2(*lv, output_final_state=True, use_qk_l2norm_in_kernel=True)
        g_ref = torch.autograd.grad(o_ref, lv, full["do"])
        refs = {"o": o_ref.detach()}
        refs.update({f"d{n}": gr for n, gr in zip("qkvgbw", g_ref)})

        def rel(a, b):
            a, b = a.double(), b.double()
            return float((a - b).norm() / b.norm().clamp_min(1e-30))

        sig = lambda x: float(f"{x:.3e}")
        out = {n: sig(rel(torch.cat(list(gathered[n].unbind(0)), 1), refs[n])) for n in refs}
        out["ht"] = sig(rel(ht_last, ht_ref))
        out["heads"] = hs
        out["reference"] = "chunk_gdn2 on the whole 262,144-token sequence on one GPU"
        out["tolerance"] = 2e-2
        out["ok"] = all(v <= 2e-2 for k_, v in out.items() if isinstance(v, float))
    barrier(world)
    return out


def run_heads(args, world, rank, local):
    """N>1: config 4 head-sharded -- H/N heads of the whole sequence per rank,
    chunk_gdn2 on one GPU each, no collective."""
    from qwendopamine_b200 import chunk_gdn2

    dev = torch.device("cuda", local)
    hper = H4 // world
    x = config4_scalars(dev, 0, T4, heads=range(rank * hper, (rank + 1) * hper))
    leaves = leaves_of(x)

    def step():
        o, _ = chunk_gdn2(*leaves, use_qk_l2norm_in_kernel=True)
        torch.autograd.grad(o, leaves, x["do"])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    from qwendopamine_b200.gdn2_ops.cp import sub_spans_single
    from qwendopamine_b200.gdn2_ops.overlap import overlap_pieces

    S = sub_spans_single(1, T4, hper, K, V, torch.bfloat16)
    P = overlap_pieces(1, T4, hper, K, V, torch.bfloat16, dev)
    if S > 1:
        path, per_step = (f"single-GPU sub-span path, {S} pieces (pre-scan, unfold, state "
                          "passes on the pieces)"), 8
    elif P > 1:
        path, per_step = (f"overlapped path, {P} pieces (state passes on a second stream "
                          "beside the intra kernels)"), 4 * P
    else:
        path, per_step = "plain chunk path", 4
    return {"workload": f"config4 head-sharded: {hper} of {H4} heads of the whole sequence "
                        f"per rank, no collective; {path}",
            "ms_per_step": round(ms, 3), "value": round(T4 / (ms / 1e3), 1),
            "unit": "tokens/s", "gpu_launches": per_step * args.steps}


# ---------------------------------------------------------------------------
# config 1 (nested record)
# ---------------------------------------------------------------------------
def run_config1(args, world, rank, local):
    from qwendopamine_b200 import _native as N
    from qwendopamine_b200 import chunk_gdn2

    dev = torch.device("cuda", local)
    lib = N.load()
    x, x_scalar = make_config1(dev, 1234 + rank)
    tables = N.seq_tables(B1, T1, dev)
    prob = N.ChunkProblem(H1, K, V, N.dtype_code(torch.bfloat16), 1, K ** -0.5, tables.struct())
    sbytes = lib.gdn2_chunk_saved_bytes(prob)
    wbytes = lib.gdn2_chunk_bwd_workspace_bytes(prob)
    saved = torch.empty(sbytes, dtype=torch.uint8, device=dev)
    ws = torch.empty(wbytes, dtype=torch.uint8, device=dev)
    o = torch.empty_like(x["v"])
    grads = {n: torch.empty_like(x[n]) for n in ("q", "k", "v", "g", "b", "w")}
    P = {n: N.ptr(t) for n, t in x.items()}
    G = {n: N.ptr(t) for n, t in grads.items()}
    st = N.stream_of(dev)
    stream = torch.cuda.current_stream(dev)
    phases = ("fwd_intra", "fwd_state", "bwd_state", "bwd_intra")

    def step(evs):
        evs[0].record(stream)
        N.check(lib.gdn2_chunk_fwd_intra(prob, P["q"], P["k"], P["v"], P["g"], P["b"], P["w"],
                                         N.ptr(saved), sbytes, st), "fwd_intra")
        evs[1].record(stream)
        N.check(lib.gdn2_chunk_fwd_state(prob, None, N.ptr(o), None, N.ptr(saved), sbytes, st),
                "fwd_state")
        evs[2].record(stream)
        N.check(lib.gdn2_chunk_bwd_state(prob, N.ptr(saved), sbytes, P["do"], None, None,
                                         N.ptr(ws), wbytes, st), "bwd_state")
        evs[3].record(stream)
        N.check(lib.gdn2_chunk_bwd_intra(prob, P["q"], P["k"], P["v"], P["g"], P["b"], P["w"],
                                         N.ptr(saved), sbytes, P["do"], G["q"], G["k"], G["v"],
                                         G["g"], G["b"], G["w"], N.ptr(ws), wbytes, st),
                "bwd_intra")
        evs[4].record(stream)

    mk = lambda: [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    for _ in range(args.warmup):
        step(mk())
    torch.cuda.synchronize()
    barrier(world)
    evlist = [mk() for _ in range(args.steps)]
    for evs in evlist:
        step(evs)
    torch.cuda.synchronize()
    barrier(world)
    total_ms = evlist[0][0].elapsed_time(evlist[-1][4])
    phase_ms = {ph: {"ms": round(statistics.mean(e[i].elapsed_time(e[i + 1]) for e in evlist), 4),
                     "launches": args.steps}
                for i, ph in enumerate(phases)}
    ms_step = max_over_ranks(total_ms / args.steps, world)
    del saved, ws, o, grads

    # end to end through chunk_gdn2 + autograd with host buffers
    host = {n: x[n].cpu().pin_memory() for n in ("q", "k", "v", "do")}
    host.update({n: t.cpu().pin_memory() for n, t in x_scalar.items()})

    def e2e_step(d):
        b_, w_, g_ = broadcast_gates(d["beta"], d["g"])
        lv = [t.detach().requires_grad_() for t in (d["q"], d["k"], d["v"], g_, b_, w_)]
        out, _ = chunk_gdn2(*lv, use_qk_l2norm_in_kernel=True)
        loss = (out * d["do"]).sum(dtype=torch.float32)
        torch.autograd.grad(loss, lv)
        return loss

    e2e_ms, h2d, d2h = run_e2e(world, dev, host, e2e_step, max(1, min(args.steps, 5)),
                               min(args.warmup, 2))
    del host
    th = B1 * T1 * H1
    hbm, tflops_peak, kind = peaks()
    roof = roofline_of(phase_ms, th, hbm, kind, "config1")
    return {
        "workload": "config1: chunk_gdn2 forward+backward, B=8 T=4096 H=16 K=V=128 bf16 per "
                    f"rank, batch-sharded x{world} (weak, no data-path collective); the four "
                    "phases of gdn2_chunk_fwd / gdn2_chunk_bwd through the C ABI",
        "value": round(B1 * T1 * world / (ms_step / 1e3), 1), "unit": "tokens/s",
        "ms_per_step": round(ms_step, 4), "scaling": "weak", "steps": args.steps,
        "gpu_launches": 4 * args.steps,
        "phases": phase_ms, "roofline": roof,
        "tc_peak": tc_peak_line(th * world, ms_step, tflops_peak, hbm),
        "e2e": {"value": round(B1 * T1 * world / (e2e_ms / 1e3), 1), "unit": "tokens/s",
                "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "l2": "inputs (>1 GB per step) exceed L2; no flush",
    }


def run_step4(args):
    """Only the headline's timed loop: config-4 forward + backward steps on
    one GPU through ``chunk_gdn2`` (the overlapped path), ``--warmup`` +
    ``--steps`` steps with per-phase CUDA events; no end-to-end leg, CPU
    baseline or sub-record (a short program for ncu launch lists)."""
    from qwendopamine_b200 import _native as N

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    N.load()
    x = config4_scalars(dev, 0, T4)
    leaves = leaves_of(x)
    fwd = config4_step_fn(1, 0)

    def step():
        torch.autograd.grad(fwd(leaves), leaves, x["do"])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with N.phase_timing() as rec:
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    return {"ms_per_step": round(ms, 4), "tokens_per_s": round(T4 / (ms / 1e3), 1),
            "phases": phase_summary(rec, args.steps),
            "gpu_launches": sum(1 for n, _, _ in rec if n in NATIVE_PHASES)}


def run_profile_case(args, local):
    """Small case for ncu captures: the step's four phases through the C ABI
    at ``--batch`` x ``--seq`` tokens x ``--heads`` heads (config-1 shapes by
    default; ``--batch 1 --seq 32768 --heads 32`` is a config-4-shaped slice),
    inputs still larger than L2, ``--warmup`` + ``--steps`` steps, nothing
    else."""
    from qwendopamine_b200 import _native as N

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    lib = N.load()
    Bp, Tp, Hp = args.batch, args.seq, args.heads
    gen = torch.Generator(device=dev).manual_seed(99)
    d = _draw(gen, dev, (Bp, Tp), Hp)
    b, w, g = broadcast_gates(d["beta"], d["gs"])
    x = dict(q=d["q"], k=d["k"], v=d["v"], g=g, b=b, w=w, do=d["do"])
    tables = N.seq_tables(Bp, Tp, dev)
    prob = N.ChunkProblem(Hp, K, V, N.dtype_code(torch.bfloat16), 1, K ** -0.5, tables.struct())
    sbytes = lib.gdn2_chunk_saved_bytes(prob)
    wbytes = lib.gdn2_chunk_bwd_workspace_bytes(prob)
    saved = torch.empty(sbytes, dtype=torch.uint8, device=dev)
    ws = torch.empty(wbytes, dtype=torch.uint8, device=dev)
    o = torch.empty_like(x["v"])
    gr = {n: torch.empty_like(x[n]) for n in ("q", "k", "v", "g", "b", "w")}
    P = {n: N.ptr(t) for n, t in x.items()}
    G = {n: N.ptr(t) for n, t in gr.items()}
    st = N.stream_of(dev)
    for _ in range(args.warmup + args.steps):
        N.check(lib.gdn2_chunk_fwd(prob, P["q"], P["k"], P["v"], P["g"], P["b"], P["w"], None,
                                   N.ptr(o), None, N.ptr(saved), sbytes, st), "fwd")
        N.check(lib.gdn2_chunk_bwd(prob, P["q"], P["k"], P["v"], P["g"], P["b"], P["w"],
                                   N.ptr(saved), sbytes, P["do"], None, G["q"], G["k"], G["v"],
                                   G["g"], G["b"], G["w"], None, N.ptr(ws), wbytes, st), "bwd")
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": {"batch": Bp, "T": Tp, "H": Hp, "K": K, "V": V,
                                       "launches_per_step": 4,
                                       "steps": args.warmup + args.steps}}))


# ---------------------------------------------------------------------------
# decode (config 2), config 0, block kernels
# ---------------------------------------------------------------------------
def run_decode(dev, lib, N, steps=DEC_STEPS, warm=16):
    """Config 2: one in-place recurrent step over B=256 sequences per call."""
    gen = torch.Generator(device=dev).manual_seed(7)
    bf = torch.bfloat16
    state = torch.randn(DEC_B, DEC_H, K, V, device=dev, generator=gen) * 0.02
    sets = []
    for _ in range(DEC_SETS):
        d = _draw(gen, dev, (DEC_B, 1), DEC_H)
        b, w, g = broadcast_gates(d["beta"], d["gs"])
        sets.append(dict(q=d["q"], k=d["k"], v=d["v"], g=g, b=b, w=w,
                         o=torch.empty(DEC_B, 1, DEC_H, V, device=dev, dtype=bf)))
    prob = N.RecurrentProblem(DEC_B, 1, DEC_H, DEC_H, K, V, N.dtype_code(bf), 1, K ** -0.5, DEC_B,
                              None, None, 0)
    st = N.stream_of(dev)
    stream = torch.cuda.current_stream(dev)
    ptrs = [tuple(N.ptr(s[n]) for n in ("q", "k", "v", "g", "b", "w", "o")) for s in sets]

    def one(i):
        p = ptrs[i % DEC_SETS]
        N.check(lib.gdn2_recurrent_fwd(prob, *p[:6], N.ptr(state), p[6], N.ptr(state), st),
                "decode")

    for i in range(warm):
        one(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        one(i)
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / steps
    nbytes = 2 * DEC_B * DEC_H * K * V * 4
    hbm, _, kind = peaks()
    gbs = nbytes / (us / 1e6) / 1e9
    return {"workload": "config2: B=256 H=16 K=V=128 fp32 state, in-place step, bf16 inputs",
            "steps": steps, "us_per_step": round(us, 2), "GBps": round(gbs, 1),
            "frac": round(gbs / hbm, 4), "state_bytes_per_step": nbytes,
            "peak_source": kind, "gpu_launches": steps, "kernel": "k_recurrent_stream"}


def run_config0(dev, iters=50, warm=5):
    """Config 0 on the GPU: fp32 forward of B=1 T=512 H=4 K=V=64 (seed 0,
    draw order q, k, v, beta, g; zero initial state) through chunk_gdn2,
    latency per call; returns the record and the output for the CPU check."""
    from qwendopamine_b200 import chunk_gdn2

    x = config0_inputs()
    xd = [t.to(dev) for t in x]
    stream = torch.cuda.current_stream(dev)
    for _ in range(warm):
        chunk_gdn2(*xd, output_final_state=True, use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(iters):
        o, ht = chunk_gdn2(*xd, output_final_state=True, use_qk_l2norm_in_kernel=True)
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / iters
    rec = {"workload": "config0: chunk_gdn2 forward, fp32, B=1 T=512 H=4 K=V=64, zero "
                       "initial state, seed 0 (public API, two launches per call)",
           "gpu_us_per_call": round(us, 2), "calls": iters, "gpu_launches": 2 * iters}
    return rec, (o.cpu(), ht.cpu())


def config0_inputs():
    gen = torch.Generator().manual_seed(0)
    Bs, Ts, H, D = 1, 512, 4, 64
    q = F.normalize(torch.randn(Bs, Ts, H, D, generator=gen), dim=-1)
    k = F.normalize(torch.randn(Bs, Ts, H, D, generator=gen), dim=-1)
    v = torch.randn(Bs, Ts, H, D, generator=gen)
    beta = torch.sigmoid(torch.randn(Bs, Ts, H, generator=gen))
    g = F.logsigmoid(torch.randn(Bs, Ts, H, generator=gen) + 3.0)
    return (q, k, v, g[..., None].expand(Bs, Ts, H, D).contiguous(),
            beta[..., None].expand(Bs, Ts, H, D).contiguous(),
            beta[..., None].expand(Bs, Ts, H, D).contiguous())


def run_block_ops(dev, lib, N, iters=20, warm=3):
    """Conv + SiLU and gated RMSNorm kernels at config-1 shapes (bf16)."""
    bf = torch.bfloat16
    gen = torch.Generator(device=dev).manual_seed(9)
    D, Wc, rows = H1 * K, 4, B1 * T1 * H1
    st = N.stream_of(dev)
    stream = torch.cuda.current_stream(dev)
    hbm, _, kind = peaks()
    sets = [dict(x=torch.randn(B1, T1, D, device=dev, generator=gen).to(bf),
                 dy=torch.randn(B1, T1, D, device=dev, generator=gen).to(bf)) for _ in range(2)]
    w = torch.randn(D, Wc, device=dev, generator=gen) * 0.5
    y, dx = torch.empty_like(sets[0]["x"]), torch.empty_like(sets[0]["x"])
    cp = N.ConvProblem(B1, T1, D, Wc, N.dtype_code(bf), 1)
    cws = torch.empty(lib.gdn2_conv_bwd_workspace_bytes(cp), dtype=torch.uint8, device=dev)
    dw = torch.empty(D, Wc, device=dev)
    nw = 1 + 0.1 * torch.randn(V, device=dev, generator=gen).to(bf)
    npb = N.NormProblem(rows, V, N.dtype_code(bf), N.dtype_code(bf), 1e-5, 0)
    nws = torch.empty(lib.gdn2_gated_norm_bwd_workspace_bytes(npb), dtype=torch.uint8, device=dev)
    ndw = torch.empty(V, device=dev)
    nsets = [dict(x=s["x"].view(rows, V), z=s["dy"].view(rows, V)) for s in sets]
    ny, ndx, ndz = (torch.empty(rows, V, device=dev, dtype=bf) for _ in range(3))

    calls = {
        "conv_fwd": (lambda s: lib.gdn2_conv_fwd(cp, N.ptr(s["x"]), N.ptr(w), None, None,
                                                 N.ptr(y), None, st), 2),
        "conv_bwd": (lambda s: lib.gdn2_conv_bwd(cp, N.ptr(s["x"]), N.ptr(w), None, None,
                                                 N.ptr(s["dy"]), N.ptr(dx), N.ptr(dw), None, None,
                                                 N.ptr(cws), cws.numel(), st), 3),
        "norm_fwd": (lambda s: lib.gdn2_gated_norm_fwd(npb, N.ptr(s["x"]), N.ptr(s["z"]),
                                                       N.ptr(nw), N.ptr(ny), st), 3),
        "norm_bwd": (lambda s: lib.gdn2_gated_norm_bwd(npb, N.ptr(s["x"]), N.ptr(s["z"]),
                                                       N.ptr(nw), N.ptr(ny), N.ptr(ndx),
                                                       N.ptr(ndz), N.ptr(ndw), N.ptr(nws),
                                                       nws.numel(), st), 5),
    }
    out = {"workload": "config1 shapes, bf16: conv+SiLU over [8,4096,2048] (W=4), gated "
                       "RMSNorm over [524288,128]", "peak_source": kind}
    tensor_bytes = B1 * T1 * D * 2
    for name, (fn, ntensors) in calls.items():
        src = nsets if name.startswith("norm") else sets
        for i in range(warm):
            N.check(fn(src[i % 2]), name)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(iters):
            N.check(fn(src[i % 2]), name)
        e1.record(stream)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / iters
        gbs = ntensors * tensor_bytes / (us / 1e6) / 1e9
        out[name] = {"us": round(us, 1), "GBps": round(gbs, 1), "frac": round(gbs / hbm, 4),
                     "bytes": ntensors * tensor_bytes, "launches": iters}
    return out


# ---------------------------------------------------------------------------
# config 3: a 24-layer decoder with the drop-in block in every layer, DDP
# ---------------------------------------------------------------------------
C3 = dict(layers=24, hidden=2048, heads=16, head_dim=128, mlp=5632, vocab=151936, batch=8,
          seq=8192, micro=1, warmup=2, steps=3)


def build_config3_model(dev):
    """Random-init decoder shaped as BASELINE config 3 (the reference host's
    block structure, gdn2_gpt/model.py:176-248 and :251-380): embedding, 24 x
    [RMSNorm -> GatedDeltaNet2 -> residual -> RMSNorm -> SwiGLU -> residual],
    final RMSNorm, LM head; bf16 parameters."""
    from torch import nn

    from qwendopamine_b200 import GatedDeltaNet2

    class RMSNorm(nn.Module):
        def __init__(self, n, eps=1e-5):
            super().__init__()
            self.weight = nn.Parameter(torch.ones(n))
            self.eps = eps

        def forward(self, x):
            return F.rms_norm(x, (x.shape[-1],), self.weight, self.eps)

    class Block(nn.Module):
        def __init__(self, i):
            super().__init__()
            d = C3["hidden"]
            self.norm_1, self.norm_2 = RMSNorm(d), RMSNorm(d)
            self.attn = GatedDeltaNet2(hidden_size=d, num_heads=C3["heads"],
                                       head_dim=C3["head_dim"], layer_idx=i)
            self.w1 = nn.Linear(d, C3["mlp"], bias=False)
            self.w2 = nn.Linear(d, C3["mlp"], bias=False)
            self.w3 = nn.Linear(C3["mlp"], d, bias=False)

        def forward(self, x):
            x = x + self.attn(self.norm_1(x))[0]
            n2 = self.norm_2(x)
            return x + self.w3(F.silu(self.w1(n2)) * self.w2(n2))

    class Decoder(nn.Module):
        def __init__(self):
            super().__init__()
            self.wte = nn.Embedding(C3["vocab"], C3["hidden"])
            self.h = nn.ModuleList([Block(i) for i in range(C3["layers"])])
            self.ln_f = RMSNorm(C3["hidden"])
            self.lm_head = nn.Linear(C3["hidden"], C3["vocab"], bias=False)

        def forward(self, idx, targets):
            x = self.wte(idx)
            for blk in self.h:
                x = blk(x)
            x = self.ln_f(x)
            loss = 0.0
            for a in range(0, idx.shape[1], 2048):  # bounded logits memory
                logits = self.lm_head(x[:, a:a + 2048]).float()
                loss = loss + F.cross_entropy(logits.flatten(0, 1), targets[:, a:a + 2048].flatten(),
                                              reduction="sum")
            return loss / idx.numel()

    with torch.device(dev):
        model = Decoder()
    return model.to(torch.bfloat16)


def run_config3(world, rank, local):
    """Config 3: one optimizer step per timed step over B=8 x T=8192 token ids
    per GPU (micro-batches of one sequence, gradients accumulated, NCCL
    all-reduce of the gradients by DDP at N>1), AdamW on bf16 parameters."""
    dev = torch.device("cuda", local)
    torch.manual_seed(0)
    model = build_config3_model(dev)
    n_params = sum(p.numel() for p in model.parameters())
    gdn_params = sum(p.numel() for blk in model.h for p in blk.attn.parameters())
    ddp = model
    if world > 1:
        from torch.nn.parallel import DistributedDataParallel as DDP

        ddp = DDP(model, device_ids=[local], bucket_cap_mb=256, gradient_as_bucket_view=True)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, fused=True)
    gen = torch.Generator(device=dev).manual_seed(3 + rank)
    idx = torch.randint(0, C3["vocab"], (C3["batch"], C3["seq"] + 1), device=dev, generator=gen)
    nmb = C3["batch"] // C3["micro"]

    def step():
        for m in range(nmb):
            sl = slice(m * C3["micro"], (m + 1) * C3["micro"])
            ctx = ddp.no_sync() if (world > 1 and m + 1 < nmb) else _nullctx()
            with ctx:
                loss = ddp(idx[sl, :-1], idx[sl, 1:])
                (loss / nmb).backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        return loss

    for _ in range(C3["warmup"]):
        step()
    torch.cuda.synchronize()
    barrier(world)
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(C3["steps"]):
        loss = step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / C3["steps"], world)
    tokens_gpu = C3["batch"] * C3["seq"]
    # dense work: 6 N tokens (fwd + bwd of every weight), plus the gdn2 core
    flops = 6 * n_params * tokens_gpu + C3["layers"] * STEP_FLOPS * C3["heads"] * tokens_gpu
    peak = peaks()[1]
    out = {"workload": "config3: 24 x [RMSNorm, GatedDeltaNet2 (B200 kernels), RMSNorm, "
                       "SwiGLU 5632] decoder, hidden 2048, 16 heads x 128, vocab 151936, bf16; "
                       "B=8 x T=8192 token ids per GPU as 8 micro-batches of one sequence, "
                       "AdamW (fused, bf16 parameters) step included",
           "parallelism": (f"data-parallel x{world} (DDP, NCCL all-reduce of gradients)"
                           if world > 1 else "single GPU"),
           "params": n_params, "gdn2_block_params": gdn_params,
           "ms_per_step": round(ms, 2), "steps": C3["steps"], "warmup": C3["warmup"],
           "tokens_per_s_per_gpu": round(tokens_gpu / (ms / 1e3), 1),
           "tokens_per_s": round(world * tokens_gpu / (ms / 1e3), 1),
           "model_tflops_per_gpu": round(flops / (ms / 1e3) / 1e12, 1),
           "frac_of_bf16_peak": round(flops / (ms / 1e3) / 1e12 / peak, 4),
           "loss": round(float(loss.detach()), 4)}
    del ddp, model, opt
    torch.cuda.empty_cache()
    return out


class _nullctx:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


# ---------------------------------------------------------------------------
# CPU baselines (reference algorithm, PyTorch CPU restatement)
# ---------------------------------------------------------------------------
CPU_SAMPLE_T, CPU_SAMPLE_HEADS = 8192, 8


def _cpu_sample_step(threads):
    """One fwd+bwd of the reference CPU path on a bounded slice of the
    workload: one sequence of 8,192 tokens x 8 heads, K=V=128 (fp32,
    autograd).  The chunk algorithm's cost is linear in tokens x heads, so
    the slice's token-heads per second scale to either config."""
    from oracle import gdn2_torch_port as P

    torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(0)
    h, Ts = CPU_SAMPLE_HEADS, CPU_SAMPLE_T
    q = F.normalize(torch.randn(1, Ts, h, K, generator=gen), dim=-1).requires_grad_()
    k = F.normalize(torch.randn(1, Ts, h, K, generator=gen), dim=-1).requires_grad_()
    v = torch.randn(1, Ts, h, V, generator=gen).requires_grad_()
    beta = torch.sigmoid(torch.randn(1, Ts, h, generator=gen))
    gs = F.logsigmoid(torch.randn(1, Ts, h, generator=gen) + 3.0)
    g = gs[..., None].expand(1, Ts, h, K).contiguous().requires_grad_()
    b = beta[..., None].expand(1, Ts, h, K).contiguous().requires_grad_()
    w = beta[..., None].expand(1, Ts, h, V).contiguous().requires_grad_()
    do = torch.randn(1, Ts, h, V, generator=gen)
    t0 = time.perf_counter()
    o, _ = P.chunk_fwd(q, k, v, g, b, w, chunk_size=C)
    torch.autograd.grad(o, (q, k, v, g, b, w), do)
    return time.perf_counter() - t0


def _sample_text(t, n, what):
    return (f"fwd+bwd of 1 sequence x T={CPU_SAMPLE_T} x {CPU_SAMPLE_HEADS} heads, K=V={K}, "
            f"fp32, reference CPU algorithm (torch_chunk_gdn2 + autograd) restated in "
            f"oracle/gdn2_torch_port.py; {t:.2f} s per sample, {what} of {n}; tokens x heads "
            "per second scaled to the config's tokens")


def cpu_baseline_chunk(samples=4):
    """Returns token-heads/s of the CPU chunk path, the per-sample seconds
    and the threads used."""
    threads = host_threads()
    _cpu_sample_step(threads)
    ts = [_cpu_sample_step(threads) for _ in range(samples)]
    t = min(ts)
    return CPU_SAMPLE_T * CPU_SAMPLE_HEADS / t, t, threads, samples


def cpu_config_line(th_per_s, t, threads, samples, heads):
    return {"value": round(th_per_s / heads, 2), "unit": "tokens/s", "cores": threads,
            "kind": "port", "sample": _sample_text(t, samples, "best")}


def cpu_decode(samples=3):
    """torch_recurrent_gdn2 at T=1 (restated as gdn2_torch_port.recurrent_step)
    over the config-2 state, all host threads."""
    from oracle import gdn2_torch_port as P

    threads = host_threads()
    torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(7)
    state = torch.randn(DEC_B, DEC_H, K, V, generator=gen) * 0.02
    d = _draw(gen, torch.device("cpu"), (DEC_B, 1), DEC_H)
    b, w, g = broadcast_gates(d["beta"], d["gs"])
    args = [t.float() for t in (d["q"], d["k"], d["v"], g, b, w)]
    ts = []
    for i in range(samples + 1):
        t0 = time.perf_counter()
        P.recurrent_step(*args, state)
        ts.append(time.perf_counter() - t0)
    t = min(ts[1:])
    nbytes = 2 * DEC_B * DEC_H * K * V * 4
    return {"us_per_step": round(t * 1e6, 1), "GBps": round(nbytes / t / 1e9, 3),
            "unit": "GB/s of state traffic", "cores": threads, "kind": "port",
            "sample": f"one T=1 step of oracle/gdn2_torch_port.recurrent_step (the reference's "
                      f"torch_recurrent_gdn2 token loop) over the whole config-2 state, fp32, "
                      f"best of {samples} after one warm-up"}


def cpu_config0(gpu_out, samples=3):
    """Config 0 on the CPU: the chunk path and the recurrent path (reference
    torch_chunk_gdn2 / torch_recurrent_gdn2, restated), all host threads,
    and the rel-L2 of the GPU output against the CPU chunk path's."""
    from oracle import gdn2_torch_port as P

    threads = host_threads()
    torch.set_num_threads(threads)
    x = config0_inputs()

    def best(fn):
        ts = []
        for _ in range(samples + 1):
            t0 = time.perf_counter()
            r = fn()
            ts.append(time.perf_counter() - t0)
        return min(ts[1:]), r

    t_chunk, (o_c, ht_c) = best(lambda: P.chunk_fwd(*x, chunk_size=C))
    t_rec, (o_r, _) = best(lambda: P.recurrent_step(*x, torch.zeros(1, 4, 64, 64)))

    def rel(a, b):
        return float((a.double() - b.double()).norm() / b.double().norm())

    return {"cpu_chunk_ms": round(t_chunk * 1e3, 2), "cpu_recurrent_ms": round(t_rec * 1e3, 2),
            "cores": threads, "kind": "port",
            "rel_l2_gpu_vs_cpu_chunk": {"o": round(rel(gpu_out[0], o_c), 8),
                                        "ht": round(rel(gpu_out[1], ht_c), 8)},
            "rel_l2_cpu_chunk_vs_recurrent": round(rel(o_c, o_r), 8)}


def run_reference(args, world, rank):
    if rank != 0:
        return
    threads = host_threads()
    for _ in range(args.warmup):
        _cpu_sample_step(threads)
    ts = [_cpu_sample_step(threads) for _ in range(args.steps)]
    t = statistics.mean(ts)
    th_per_s = CPU_SAMPLE_T * CPU_SAMPLE_HEADS / t
    value = th_per_s / H4
    line = {
        "impl": "reference",
        "metric": "gdn2 fwd+bwd tokens/s (BASELINE config 4)",
        "value": round(value, 2),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t * 1e3, 2),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded; config-0 recipe at config-4 shapes)",
        "config": {"workload": "config4: chunk_gdn2 forward+backward", "batch": 1,
                   "seq_len": T4, "heads": H4, "head_k": K, "head_v": V, "chunk": C},
        "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": threads,
                         "kind": "port",
                         "sample": "each step: " + _sample_text(t, args.steps, "mean")},
        "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# main B200 arm
# ---------------------------------------------------------------------------
def run_b200(args, world, rank, local):
    from qwendopamine_b200 import _native as N

    dev = torch.device("cuda", local)
    clocks = []
    c4 = run_config4(args, world, rank, local, clocks)
    parity = heads = None
    if world > 1:
        parity = sp_parity(world, rank, local, c4["x"], config4_step_fn(world, rank))
        del c4["x"], c4["leaves"]
        torch.cuda.empty_cache()
        heads = run_heads(args, world, rank, local)
    else:
        del c4["x"], c4["leaves"]
    torch.cuda.empty_cache()
    c1 = run_config1(args, world, rank, local)
    torch.cuda.empty_cache()
    c3 = run_config3(world, rank, local) if not args.skip_model else None
    dec = c0 = blk = None
    if rank == 0 and world == 1:
        lib = N.load()
        dec = run_decode(dev, lib, N)
        c0, c0_out = run_config0(dev)
        blk = run_block_ops(dev, lib, N)
    barrier(world)
    if rank != 0:
        return
    hbm, tflops_peak, peak_kind = peaks()
    phases = c4["phases"]
    roof = roofline_of(phases, c4["token_heads"], hbm, peak_kind, "config4")
    solo, every, per_step = c4["solo"]
    if roof["kernel"] == "bwd_intra" and per_step > 1 and solo:
        # overlapped path: the kernel's own rate is that of the launches that
        # had the GPU to themselves; the all-launch figure stays beside it
        th = c4["token_heads"] / per_step
        ach = PHASE_BYTES["bwd_intra"] * th / (statistics.mean(solo) / 1e3) / 1e9
        roof["all_launches"] = {"achieved": roof["achieved"], "frac": roof["frac"],
                                "launches": len(every)}
        roof.update(achieved=round(ach, 1), frac=round(ach / hbm, 4),
                    token_heads_per_launch=round(th),
                    traffic=round(NCU_TRAFFIC_PER_TOKEN_HEAD["config4"] * th),
                    launches=(f"{len(solo)} of {len(every)} timed launches: those that "
                              "started after the step's last state pass had ended"))
    ms = c4["ms"]
    cpu = None
    if world == 1:
        th_per_s, t_s, threads, n = cpu_baseline_chunk()
        cpu = cpu_config_line(th_per_s, t_s, threads, n, H4)
        c1["cpu_baseline"] = cpu_config_line(th_per_s, t_s, threads, n, H1)
        dec["cpu_baseline"] = cpu_decode()
        c0.update(cpu_config0(c0_out))
    line = {
        "metric": "gdn2 fwd+bwd tokens/s (BASELINE config 4)",
        "value": round(T4 / (ms / 1e3), 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded per 4,096-token block; config-0 recipe at config-4 shapes)",
        "config": {
            "workload": ("config4: chunk_gdn2 forward+backward on one GPU" if world == 1 else
                         f"config4: chunk_gdn2_cp forward+backward, sequence-parallel x{world}"),
            "batch": 1, "seq_len": T4, "heads": H4, "head_k": K, "head_v": V, "chunk": C,
            "tokens_per_rank": T4 // world,
            "parallelism": ("single GPU" if world == 1 else
                            f"sequence-parallel x{world}: NCCL all-gather of the span maps "
                            "once per direction"),
            "l2": "inputs (>10 GB per step) exceed L2; no flush",
        },
        "gpu_launches": c4["launches"],
        "e2e": {"value": round(T4 / (c4["e2e_ms"] / 1e3), 1), "unit": "tokens/s",
                "ms_per_step": round(c4["e2e_ms"], 3), "h2d_bytes_per_step": c4["h2d"],
                "d2h_bytes_per_step": c4["d2h"]},
        "roofline": roof,
        "phases": phases,
        "phases_rank": 0,
        "tensor_peak_tflops": tflops_peak,
        "tc_peak": tc_peak_line(T4 * H4, ms, tflops_peak, hbm),
        "sp_parity": parity,
        "heads": heads,
        "config1": c1,
        "config3": c3,
        "decode": dec,
        "config0": c0,
        "block_ops": blk,
        "clocks": clocks[0] if clocks else None,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--workload", choices=("config4", "step4", "block", "decode"),
                    default="config4",
                    help="config4 (headline, with every sub-record), or only the headline's "
                         "timed config-4 steps on one GPU (step4), or only the block "
                         "prologue / epilogue kernels (--steps timed launches each after "
                         "--warmup, one GPU), or only the config-2 decode step")
    ap.add_argument("--skip-model", action="store_true",
                    help="leave out the config-3 model step (24-layer decoder)")
    ap.add_argument("--profile", action="store_true",
                    help="small ncu case: config-1 phases at --batch, nothing else")
    ap.add_argument("--batch", type=int, default=2, help="batch of the --profile case")
    ap.add_argument("--seq", type=int, default=T1, help="sequence length of the --profile case")
    ap.add_argument("--heads", type=int, default=H1, help="heads of the --profile case")
    args = ap.parse_args(argv)
    if args.profile:
        run_profile_case(args, int(os.environ.get("LOCAL_RANK", "0")))
        return
    if args.workload == "step4":
        print(json.dumps({"workload": "step4", "step4": run_step4(args)}), flush=True)
        return
    if args.workload in ("block", "decode"):
        from qwendopamine_b200 import _native as N

        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        if args.workload == "block":
            rec = run_block_ops(dev, N.load(), N, iters=args.steps, warm=args.warmup)
        else:
            rec = run_decode(dev, N.load(), N, steps=args.steps, warm=args.warmup)
        print(json.dumps({"workload": args.workload, args.workload: rec}), flush=True)
        return
    if args.warmup < 3 and args.impl == "b200":
        args.warmup = 3
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    world, rank, local = dist_setup()
    try:
        run_b200(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()

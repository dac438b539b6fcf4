#!/usr/bin/env python
"""GDN-2 B200 benchmark (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload: chunkwise GDN-2 forward + backward, bf16
activations, fp32 decay / state / accumulation, B=8 T=4096 H=16 K=V=128,
chunk 64, scalar beta and log-decay broadcast through the channel-wise API,
seeded synthetic inputs (no dataset is involved).  A step is one forward and
one backward over the whole batch.  Under torchrun every rank runs its own
batch (data/batch sharding, no collective on the data path: weak scaling);
the reported time is the max over ranks.

* ``value``: tokens/s of the whole job with inputs resident in HBM; the step
  is the four kernel phases called through the C ABI, each bracketed by CUDA
  events on the launch stream, which also gives the live per-kernel roofline.
* ``e2e``: the same metric through the public API (``chunk_gdn2`` + autograd)
  as a training step sees it: every step copies its inputs from pinned host
  memory -- q, k, v, the upstream gradient dO, and the config's per-(token,
  head) beta and log-decay, broadcast channel-wise on the device -- runs the
  forward, forms the loss sum(o * dO) (whose gradient with respect to o is
  dO), runs the backward into device gradients and reads the loss back to the
  host.  The next step's copy runs on a second stream while the current step
  computes (a double-buffered loader); every copy is inside the timed region.
* ``decode``: BASELINE config 2 (B=256 H=16 K=V=128 fp32 state, in-place
  recurrent step, bf16 inputs), state read+write GB/s.
* ``block_ops``: the block's prologue / epilogue kernels at config-1 shapes
  (bf16): the causal conv + SiLU over one [8, 4096, 2048] projection, forward
  and backward, and the gated RMSNorm over o [8*4096*16, 128], forward and
  backward; algorithmic bytes (each tensor read or written once) per launch
  over the CUDA-event time, two alternating input sets (> L2).
* ``cpu_baseline``: the reference algorithm's CPU path (PyTorch restatement in
  oracle/gdn2_torch_port.py, fp32, autograd backward), all host threads, on a
  bounded slice of the same workload; rank 0 at N=1 only.

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

B, T, H, K, V, C = 8, 4096, 16, 128, 128, 64
DEC_B, DEC_STEPS, DEC_SETS = 256, 1024, 32
FALLBACK_HBM_GBS = 6650.0

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
# Algorithmic FLOPs per token-head (C = 64, K = V = 128), for context:
#   fwd_intra 6CK+2CV, fwd_state 6KV+2CV, bwd_state 6KV+2CV,
#   bwd_intra 6KV+6CV+12CK+4C^2
PHASE_FLOPS = {
    "fwd_intra": 6 * C * K + 2 * C * V,
    "fwd_state": 6 * K * V + 2 * C * V,
    "bwd_state": 6 * K * V + 2 * C * V,
    "bwd_intra": 6 * K * V + 6 * C * V + 12 * C * K + 4 * C * C,
}
# The metric's "% TC peak": the reference schedule's fwd+bwd FLOPs per
# token-head, 20CK + 14CV + 22KV + 4C^2 = 655,360, over the step time, against
# the measured bf16 peak and against the HBM-limited ceiling min(peak, AI x
# HBM GB/s) with AI = 655,360 / 6,900 minimum bytes per token-head.
STEP_FLOPS = 20 * C * K + 14 * C * V + 22 * K * V + 4 * C * C
STEP_MIN_BYTES = 6900
# DRAM traffic (read + write) of the dominant kernel, k_bwd_intra16, per
# token-head, from one ncu --set full capture at batch 2 (701.3 MB over
# 131,072 token-heads; traffic grows with token-heads, so it scales to a
# config-1 launch).  Summary under profiles/.
NCU_TRAFFIC_PER_TOKEN_HEAD = 5309.6


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops", 1643.0)), "measured"
    return FALLBACK_HBM_GBS, 1590.0, "fallback"


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
def make_config1(device, seed):
    """Config-1 inputs as in config 0's recipe: q, k ~ N(0,1) L2-normalised,
    v ~ N(0,1), beta = sigmoid(N(0,1)), g = logsigmoid(N(3,1)) per token and
    head, broadcast channel-wise; dO ~ N(0,1)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    bf = torch.bfloat16
    q = F.normalize(torch.randn(B, T, H, K, device=device, generator=gen), dim=-1).to(bf)
    k = F.normalize(torch.randn(B, T, H, K, device=device, generator=gen), dim=-1).to(bf)
    v = torch.randn(B, T, H, V, device=device, generator=gen).to(bf)
    beta = torch.sigmoid(torch.randn(B, T, H, device=device, generator=gen))
    gs = F.logsigmoid(torch.randn(B, T, H, device=device, generator=gen) + 3.0)
    g = gs[..., None].expand(B, T, H, K).contiguous()
    b = beta[..., None].expand(B, T, H, K).to(bf).contiguous()
    w = beta[..., None].expand(B, T, H, V).to(bf).contiguous()
    do = torch.randn(B, T, H, V, device=device, generator=gen).to(bf)
    return dict(q=q, k=k, v=v, g=g, b=b, w=w, do=do), dict(beta=beta.to(bf), g=gs)


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------
def run_b200(args, world, rank, local):
    from qwendopamine_b200 import _native as N
    from qwendopamine_b200 import chunk_gdn2

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    lib = N.load()
    x, x_scalar = make_config1(dev, 1234 + rank)
    tables = N.seq_tables(B, T, dev)
    prob = N.ChunkProblem(H, K, V, N.dtype_code(torch.bfloat16), 1, K ** -0.5, tables.struct())
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
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    barrier(world)
    torch.cuda.synchronize()
    evlist = [mk() for _ in range(args.steps)]
    for evs in evlist:
        step(evs)
    torch.cuda.synchronize()
    barrier(world)
    clocks = sampler.stop() if sampler else None
    total_ms = evlist[0][0].elapsed_time(evlist[-1][4])
    phase_ms = {ph: statistics.mean(e[i].elapsed_time(e[i + 1]) for e in evlist)
                for i, ph in enumerate(phases)}
    ms_step = max_over_ranks(total_ms / args.steps, world)
    tokens = B * T * world
    value = tokens / (ms_step / 1e3)

    # ---- end to end through the public API with host buffers ---------------
    # Host holds the config's own draws: q, k, v, dO [B,T,H,D] and the
    # per-(token, head) beta and log-decay [B,T,H]; the channel-wise b, w, g
    # the API takes are broadcast on the device.  Step i+1's inputs are copied
    # on a second stream into the other half of a double buffer while step i
    # computes; every copy is inside the timed region.
    host = {n: x[n].cpu().pin_memory() for n in ("q", "k", "v", "do")}
    host.update({n: t.cpu().pin_memory() for n, t in x_scalar.items()})
    bufs = [{n: torch.empty_like(t, device=dev) for n, t in host.items()} for _ in range(2)]
    loss_host = torch.empty((), dtype=torch.float32, pin_memory=True)
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = loss_host.numel() * loss_host.element_size()
    copy_stream = torch.cuda.Stream(dev)
    ev_copied = [torch.cuda.Event() for _ in range(2)]
    ev_consumed = [torch.cuda.Event() for _ in range(2)]
    used = [False, False]
    grads = []

    def issue_copy(i, after=None):
        j = i % 2
        with torch.cuda.stream(copy_stream):
            if after is not None:
                copy_stream.wait_event(after)
            if used[j]:
                copy_stream.wait_event(ev_consumed[j])
            for n, t in host.items():
                bufs[j][n].copy_(t, non_blocking=True)
            ev_copied[j].record(copy_stream)
        used[j] = True

    def compute(i):
        j = i % 2
        stream.wait_event(ev_copied[j])
        d = bufs[j]
        b_ = d["beta"][..., None].expand(B, T, H, K).contiguous()
        w_ = d["beta"][..., None].expand(B, T, H, V).contiguous()
        g_ = d["g"][..., None].expand(B, T, H, K).contiguous()
        leaves = [t.detach().requires_grad_() for t in (d["q"], d["k"], d["v"], g_, b_, w_)]
        out, _ = chunk_gdn2(*leaves, use_qk_l2norm_in_kernel=True)
        loss = (out * d["do"]).sum(dtype=torch.float32)
        grads[:] = torch.autograd.grad(loss, leaves)  # stay on the device
        loss_host.copy_(loss.detach(), non_blocking=True)
        ev_consumed[j].record(stream)

    def e2e_run(n, start=None):
        issue_copy(0, start)
        for i in range(n):
            if i + 1 < n:
                issue_copy(i + 1)
            compute(i)

    e2e_steps = max(1, min(args.steps, 5))
    e2e_run(min(args.warmup, 2))
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_run(e2e_steps, e0)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps, world)
    del host, bufs, grads

    # ---- decode (config 2) -------------------------------------------------
    dec = run_decode(dev, lib, N) if rank == 0 else None
    blk = run_block_ops(dev, lib, N) if rank == 0 else None

    if rank != 0:
        return
    hbm, tflops_peak, peak_kind = peaks()
    th = B * T * H  # token-heads per launch (one rank)
    phase_info = {}
    for ph in phases:
        t_s = phase_ms[ph] / 1e3
        phase_info[ph] = {
            "ms": round(phase_ms[ph], 4),
            "GBps": round(PHASE_BYTES[ph] * th / t_s / 1e9, 1),
            "TFLOPs": round(PHASE_FLOPS[ph] * th / t_s / 1e12, 2),
            "launches": args.steps,
        }
    dom = max(phases, key=lambda p: phase_ms[p])
    ach = PHASE_BYTES[dom] * th / (phase_ms[dom] / 1e3) / 1e9
    traffic = (round(NCU_TRAFFIC_PER_TOKEN_HEAD * th)
               if NCU_TRAFFIC_PER_TOKEN_HEAD and dom == "bwd_intra" else None)
    cpu = cpu_baseline() if world == 1 else None
    line = {
        "metric": "gdn2 fwd+bwd tokens/s (BASELINE config 1)",
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded; config-0 recipe at config-1 shapes)",
        "config": {
            "workload": "config1: chunk_gdn2 forward+backward",
            "batch_per_gpu": B, "seq_len": T, "heads": H, "head_k": K, "head_v": V,
            "chunk": C, "parallelism": f"batch-sharded x{world}, no data-path collective",
            "l2": "inputs (>1 GB per step) exceed L2; no flush",
        },
        "gpu_launches": 4 * args.steps,
        "e2e": {"value": round(B * T * world / (e2e_ms / 1e3), 1), "unit": "tokens/s",
                "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(ach, 1), "peak": hbm,
                     "unit": "GB/s", "frac": round(ach / hbm, 4), "traffic": traffic,
                     "peak_source": peak_kind,
                     "bytes_per_token_head": PHASE_BYTES[dom]},
        "phases": phase_info,
        "tensor_peak_tflops": tflops_peak,
        "tc_peak": tc_peak_line(th * world, ms_step, tflops_peak, hbm),
        "decode": dec,
        "block_ops": blk,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


def run_profile_case(args, local):
    """Small case for ncu captures: the config-1 step at batch ``args.batch``
    (inputs still larger than L2), ``args.warmup`` + ``args.steps`` steps of
    the four phases, no end-to-end, decode or CPU legs."""
    from qwendopamine_b200 import _native as N

    global B
    B = args.batch
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    lib = N.load()
    x, _ = make_config1(dev, 99)
    tables = N.seq_tables(B, T, dev)
    prob = N.ChunkProblem(H, K, V, N.dtype_code(torch.bfloat16), 1, K ** -0.5, tables.struct())
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
    print(json.dumps({"profile_case": {"batch": B, "T": T, "H": H, "K": K, "V": V,
                                       "launches_per_step": 4,
                                       "steps": args.warmup + args.steps}}))


SP_T, SP_H = 262144, 32


def run_config4(args, world, rank, local, mode):
    """B=1 T=262144 H=32 K=V=128 bf16 forward+backward.

    mode "sp": every rank owns T/world contiguous tokens (whole chunks); the
    span maps cross GPUs through one NCCL all-gather per direction
    (chunk_gdn2_cp).  mode "heads": every rank owns H/world heads of the whole
    sequence, no communication.  Total work is fixed: strong scaling.
    """
    from qwendopamine_b200 import chunk_gdn2
    from qwendopamine_b200.gdn2_ops.cp import chunk_gdn2_cp, gather_span_maps

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if mode == "sp":
        Tl, Hl = SP_T // world, SP_H
    else:
        Tl, Hl = SP_T, SP_H // world
    gen = torch.Generator(device=dev).manual_seed(77 + rank)
    bf = torch.bfloat16
    q = F.normalize(torch.randn(1, Tl, Hl, K, device=dev, generator=gen), dim=-1).to(bf)
    k = F.normalize(torch.randn(1, Tl, Hl, K, device=dev, generator=gen), dim=-1).to(bf)
    v = torch.randn(1, Tl, Hl, V, device=dev, generator=gen).to(bf)
    beta = torch.sigmoid(torch.randn(1, Tl, Hl, device=dev, generator=gen))
    gs = F.logsigmoid(torch.randn(1, Tl, Hl, device=dev, generator=gen) + 3.0)
    g = gs[..., None].expand(1, Tl, Hl, K).contiguous()
    b = beta[..., None].expand(1, Tl, Hl, K).to(bf).contiguous()
    w = beta[..., None].expand(1, Tl, Hl, V).to(bf).contiguous()
    do = torch.randn(1, Tl, Hl, V, device=dev, generator=gen).to(bf)
    leaves = [t.requires_grad_() for t in (q, k, v, g, b, w)]
    gather = (lambda t: gather_span_maps(t, None)) if world > 1 else (lambda t: t[None])

    def step():
        if mode == "sp":
            o, _ = chunk_gdn2_cp(*leaves, rank=rank, world=world, gather=gather)
        else:
            o, _ = chunk_gdn2(*leaves, use_qk_l2norm_in_kernel=True)
        torch.autograd.grad(o, leaves, do)

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
    if rank != 0:
        return
    launches = (8 if world > 1 else 6) if mode == "sp" else 4
    print(json.dumps({
        "metric": "gdn2 fwd+bwd tokens/s (BASELINE config 4)",
        "value": round(SP_T / (ms / 1e3), 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; config-0 recipe at config-4 shapes)",
        "config": {"workload": f"config4 {mode}", "batch": 1, "seq_len": SP_T, "heads": SP_H,
                   "head_k": K, "head_v": V, "chunk": C,
                   "parallelism": (f"sequence-parallel x{world} (NCCL all-gather of span maps)"
                                   if mode == "sp" else f"head-sharded x{world}, no collective")},
        "gpu_launches": launches * args.steps,
    }), flush=True)


def tc_peak_line(token_heads, ms, peak_tflops, hbm_gbs):
    """Whole-step tensor-core fraction as the metric names it."""
    tf = STEP_FLOPS * token_heads / (ms / 1e3) / 1e12
    ceiling = min(peak_tflops, STEP_FLOPS / STEP_MIN_BYTES * hbm_gbs / 1e3)
    return {"flops_per_token_head": STEP_FLOPS, "tflops": round(tf, 1),
            "frac_of_bf16_peak": round(tf / peak_tflops, 4),
            "hbm_ceiling_tflops": round(ceiling, 1), "frac_of_ceiling": round(tf / ceiling, 4)}


def run_decode(dev, lib, N, steps=DEC_STEPS, warm=16):
    """Config 2: one in-place recurrent step over B=256 sequences per call."""
    gen = torch.Generator(device=dev).manual_seed(7)
    bf = torch.bfloat16
    state = torch.randn(DEC_B, H, K, V, device=dev, generator=gen) * 0.02
    sets = []
    for _ in range(DEC_SETS):
        q = F.normalize(torch.randn(DEC_B, 1, H, K, device=dev, generator=gen), dim=-1).to(bf)
        k = F.normalize(torch.randn(DEC_B, 1, H, K, device=dev, generator=gen), dim=-1).to(bf)
        v = torch.randn(DEC_B, 1, H, V, device=dev, generator=gen).to(bf)
        beta = torch.sigmoid(torch.randn(DEC_B, 1, H, device=dev, generator=gen))
        gs = F.logsigmoid(torch.randn(DEC_B, 1, H, device=dev, generator=gen) + 3.0)
        sets.append(dict(q=q, k=k, v=v, g=gs[..., None].expand(DEC_B, 1, H, K).contiguous(),
                         b=beta[..., None].expand(DEC_B, 1, H, K).to(bf).contiguous(),
                         w=beta[..., None].expand(DEC_B, 1, H, V).to(bf).contiguous(),
                         o=torch.empty(DEC_B, 1, H, V, device=dev, dtype=bf)))
    prob = N.RecurrentProblem(DEC_B, 1, H, H, K, V, N.dtype_code(bf), 1, K ** -0.5, DEC_B,
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
    nbytes = 2 * DEC_B * H * K * V * 4
    hbm, _, kind = peaks()
    gbs = nbytes / (us / 1e6) / 1e9
    return {"workload": "config2: B=256 H=16 K=V=128 fp32 state, in-place step, bf16 inputs",
            "steps": steps, "us_per_step": round(us, 2), "GBps": round(gbs, 1),
            "frac": round(gbs / hbm, 4), "state_bytes_per_step": nbytes,
            "peak_source": kind, "gpu_launches": steps}


def run_block_ops(dev, lib, N, iters=20, warm=3):
    """Conv + SiLU and gated RMSNorm kernels at config-1 shapes (bf16)."""
    bf = torch.bfloat16
    gen = torch.Generator(device=dev).manual_seed(9)
    D, Wc, rows = H * K, 4, B * T * H
    st = N.stream_of(dev)
    stream = torch.cuda.current_stream(dev)
    hbm, _, kind = peaks()
    sets = [dict(x=torch.randn(B, T, D, device=dev, generator=gen).to(bf),
                 dy=torch.randn(B, T, D, device=dev, generator=gen).to(bf)) for _ in range(2)]
    w = torch.randn(D, Wc, device=dev, generator=gen) * 0.5
    y, dx = torch.empty_like(sets[0]["x"]), torch.empty_like(sets[0]["x"])
    cp = N.ConvProblem(B, T, D, Wc, N.dtype_code(bf), 1)
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
    tensor_bytes = B * T * D * 2
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
# CPU baseline (reference algorithm, PyTorch CPU restatement)
# ---------------------------------------------------------------------------
CPU_SAMPLE_HEADS = 4


def _cpu_sample_step(threads):
    """One fwd+bwd of the reference CPU path on a bounded slice of config 1:
    one sequence of T=4096 tokens and 4 of the 16 heads (fp32, autograd)."""
    from oracle import gdn2_torch_port as P

    torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(0)
    h = CPU_SAMPLE_HEADS
    q = F.normalize(torch.randn(1, T, h, K, generator=gen), dim=-1).requires_grad_()
    k = F.normalize(torch.randn(1, T, h, K, generator=gen), dim=-1).requires_grad_()
    v = torch.randn(1, T, h, V, generator=gen).requires_grad_()
    beta = torch.sigmoid(torch.randn(1, T, h, generator=gen))
    gs = F.logsigmoid(torch.randn(1, T, h, generator=gen) + 3.0)
    g = gs[..., None].expand(1, T, h, K).contiguous().requires_grad_()
    b = beta[..., None].expand(1, T, h, K).contiguous().requires_grad_()
    w = beta[..., None].expand(1, T, h, V).contiguous().requires_grad_()
    do = torch.randn(1, T, h, V, generator=gen)
    t0 = time.perf_counter()
    o, _ = P.chunk_fwd(q, k, v, g, b, w, chunk_size=C)
    torch.autograd.grad(o, (q, k, v, g, b, w), do)
    return time.perf_counter() - t0


def host_threads():
    """Cores this process may run on (the container's share, not the host's)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_baseline(steps=3, warm=True):
    threads = host_threads()
    if warm:
        _cpu_sample_step(threads)
    ts = [_cpu_sample_step(threads) for _ in range(steps)]
    t = min(ts)
    full_tokens = T * CPU_SAMPLE_HEADS / H  # config-1 tokens the slice is worth
    return {"value": round(full_tokens / t, 2), "unit": "tokens/s", "cores": threads,
            "kind": "port",
            "sample": (f"fwd+bwd of 1 sequence x T={T} x {CPU_SAMPLE_HEADS}/{H} heads, "
                       f"K=V={K}, fp32, oracle/gdn2_torch_port.chunk_fwd + autograd; "
                       f"{t:.2f} s per sample, best of {steps}; value scaled to config-1 "
                       "tokens (all 16 heads)")}


def run_reference(args, world, rank):
    if rank != 0:
        return
    for _ in range(args.warmup):
        _cpu_sample_step(host_threads())
    ts = [_cpu_sample_step(host_threads()) for _ in range(args.steps)]
    t = statistics.mean(ts)
    full_tokens = T * CPU_SAMPLE_HEADS / H
    value = full_tokens / t
    cores = host_threads()
    line = {
        "impl": "reference",
        "metric": "gdn2 fwd+bwd tokens/s (BASELINE config 1)",
        "value": round(value, 2),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t * 1e3, 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded; config-0 recipe at config-1 shapes)",
        "config": {"workload": "config1: chunk_gdn2 forward+backward", "batch_per_gpu": B,
                   "seq_len": T, "heads": H, "head_k": K, "head_v": V, "chunk": C},
        "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": cores,
                         "kind": "port",
                         "sample": (f"each step: fwd+bwd of 1 sequence x T={T} x "
                                    f"{CPU_SAMPLE_HEADS}/{H} heads, fp32, reference CPU "
                                    "algorithm (torch_chunk_gdn2 + autograd) restated in "
                                    "oracle/gdn2_torch_port.py; value scaled to config-1 "
                                    "tokens")},
        "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--workload", choices=("config1", "sp", "heads", "block", "decode"),
                    default="config1",
                    help="config1 (headline), config 4 sequence-parallel / head-sharded, "
                         "block: only the prologue / epilogue kernels (--steps timed launches "
                         "each after --warmup, one GPU), or decode: only the config-2 step")
    ap.add_argument("--profile", action="store_true",
                    help="small ncu case: config-1 phases at --batch, nothing else")
    ap.add_argument("--batch", type=int, default=2, help="batch of the --profile case")
    args = ap.parse_args(argv)
    if args.profile:
        run_profile_case(args, int(os.environ.get("LOCAL_RANK", "0")))
        return
    if args.workload == "block":
        from qwendopamine_b200 import _native as N

        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        blk = run_block_ops(dev, N.load(), N, iters=args.steps, warm=args.warmup)
        print(json.dumps({"workload": "block", "block_ops": blk}), flush=True)
        return
    if args.workload == "decode":
        from qwendopamine_b200 import _native as N

        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        dec = run_decode(dev, N.load(), N, steps=args.steps, warm=args.warmup)
        print(json.dumps({"workload": "decode", "decode": dec}), flush=True)
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
        if args.workload == "config1":
            run_b200(args, world, rank, local)
        else:
            run_config4(args, world, rank, local, args.workload)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()

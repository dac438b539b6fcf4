"""Helpers shared by the GDN-2 tests: seeded inputs and the relative-L2 metric.

Tolerances: rel-L2 <= 1e-4 for fp32 and
<= 2e-2 for bf16, always against the float64 oracle or the reference's
fp32 golden vectors.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2, torch.float16: 2e-2}


def rel(a, b) -> float:
    a = a.detach().double().cpu().numpy() if isinstance(a, torch.Tensor) else np.asarray(a, np.float64)
    b = b.detach().double().cpu().numpy() if isinstance(b, torch.Tensor) else np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def make_inputs(B, T, H, K, V, seed=0, decay="mild", h0=True, dtype=torch.float32,
                scalar_gates=False):
    """Seeded channel-wise inputs (CPU fp32 master copies).

    decay: "mild" -> g = -|U(0,1)| (reference tests), "baseline" ->
    logsigmoid(N(3,1)), or a float -> constant g.
    """
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, K, generator=gen)
    k = torch.randn(B, T, H, K, generator=gen)
    v = torch.randn(B, T, H, V, generator=gen)
    if scalar_gates:
        beta = torch.sigmoid(torch.randn(B, T, H, generator=gen))
        b = beta[..., None].expand(B, T, H, K).contiguous()
        w = beta[..., None].expand(B, T, H, V).contiguous()
    else:
        b = torch.sigmoid(torch.randn(B, T, H, K, generator=gen))
        w = torch.sigmoid(torch.randn(B, T, H, V, generator=gen))
    if decay == "mild":
        g = -torch.rand(B, T, H, K, generator=gen).abs()
    elif decay == "baseline":
        gs = F.logsigmoid(torch.randn(B, T, H, generator=gen) + 3.0)
        g = gs[..., None].expand(B, T, H, K).contiguous()
    else:
        g = torch.full((B, T, H, K), float(decay))
    s = torch.randn(B, H, K, V, generator=gen) * 0.1 if h0 else None
    # round the token tensors to the working dtype so the oracle sees the
    # exact values the kernels see
    q, k, v, b, w = (x.to(dtype).float() for x in (q, k, v, b, w))
    return dict(q=q, k=k, v=v, g=g, b=b, w=w, h0=s)


def to_dev(d, device, dtype):
    out = {}
    for n, x in d.items():
        if x is None:
            out[n] = None
        elif n in ("g", "h0", "dht"):
            out[n] = x.float().to(device)
        else:
            out[n] = x.to(device=device, dtype=dtype)
    return out


def np_(d, names):
    return [None if d[n] is None else d[n].double().numpy() for n in names]

"""PyTorch CPU restatement of the reference's GDN-2 CPU path -- TEST AND
BASELINE INFRASTRUCTURE ONLY.

The reference runs GDN-2 on CPU through ``torch_chunk_gdn2`` (training,
gdn2.py:243-369, backward by autograd) and ``torch_recurrent_gdn2`` (decode,
gdn2.py:100-184).  The reference checkout is not available on the GPU box, so
``bench.py`` times this restatement instead (``cpu_baseline.kind = "port"``):
same algorithm (absolute-gamma WY chunk form with ``solve_triangular``, fp32,
autograd backward; token loop for decode), same tensor shapes, all host
threads.  ``tests/test_oracle_port.py`` checks it against the golden fixtures
made from the reference itself.

Nothing in the product package imports this file.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def chunk_fwd(q, k, v, g, b, w, initial_state=None, chunk_size=64, l2norm=True):
    """fp32 chunkwise forward (absolute-gamma WY form); differentiable."""
    Bsz, T, H, K = q.shape
    V = v.shape[-1]
    q, k, v, g, b, w = (x.float() for x in (q, k, v, g, b, w))
    if l2norm:
        q = F.normalize(q, p=2, dim=-1, eps=1e-6)
        k = F.normalize(k, p=2, dim=-1, eps=1e-6)
    q = q * K ** -0.5
    q, k, v, g, b, w = (x.transpose(1, 2) for x in (q, k, v, g, b, w))  # [B,H,T,D]
    S = (q.new_zeros(Bsz, H, K, V) if initial_state is None else initial_state.float())
    outs = []
    for s in range(0, T, chunk_size):
        e = min(s + chunk_size, T)
        qc, kc, vc, gc, bc, wc = (x[:, :, s:e] for x in (q, k, v, g, b, w))
        gam = torch.exp(torch.cumsum(gc, dim=2))
        kbar = kc / gam.clamp_min(1e-12)
        ebar = gam * bc * kc
        n = e - s
        lower = torch.tril(ebar @ kbar.transpose(-1, -2), diagonal=-1)
        I_plus_T = torch.eye(n, dtype=q.dtype) + lower
        Y = torch.linalg.solve_triangular(I_plus_T, ebar, upper=False, unitriangular=True)
        U = torch.linalg.solve_triangular(I_plus_T, wc * vc, upper=False, unitriangular=True)
        delta = U - Y @ S
        qg = gam * qc
        scores = torch.tril(qg @ kbar.transpose(-1, -2))
        outs.append(qg @ S + scores @ delta)
        S = gam[:, :, -1:, :].transpose(-1, -2) * (S + kbar.transpose(-1, -2) @ delta)
    o = torch.cat(outs, dim=2).transpose(1, 2)
    return o, S


def recurrent_step(q, k, v, g, b, w, state, l2norm=True):
    """One token-serial step per sequence (decode), in place on ``state``."""
    K = q.shape[-1]
    q, k, v, g, b, w = (x.float() for x in (q, k, v, g, b, w))
    if l2norm:
        q = F.normalize(q, p=2, dim=-1, eps=1e-6)
        k = F.normalize(k, p=2, dim=-1, eps=1e-6)
    q = q * K ** -0.5
    outs = []
    for t in range(q.shape[1]):
        state.mul_(torch.exp(g[:, t]).unsqueeze(-1))
        r = torch.einsum("bhkv,bhk->bhv", state, b[:, t] * k[:, t])
        d = w[:, t] * v[:, t] - r
        state.add_(k[:, t].unsqueeze(-1) * d.unsqueeze(-2))
        outs.append(torch.einsum("bhkv,bhk->bhv", state, q[:, t]))
    return torch.stack(outs, dim=1), state

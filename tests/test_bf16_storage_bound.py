"""Why d_beta of 64-wide heads under decays of 6 nats per token has a looser
bound on the bf16 path (CPU only).

The chunkwise algorithm stores three tensors in the token dtype between its
kernels, as the reference does: the decayed keys Kd (``kg``,
gdn2_ops/chunk_gdn2.py:1139), the per-chunk state gradient dh (returned in the
token dtype by ``chunk_gated_delta_rule_bwd_dhu``, chunk_gdn2.py:2255) and the
new-value gradient dVN (``dv``).  Under a decay of -6 per token the d_beta of
the sequence's last token carries almost all of the tensor's norm, and it is
one scalar per head, z_{T-1} . (dS_T^T k_T), times a vector; on the test case
that scalar nearly cancels for one head.  A float64 run of the chunk form with
ONLY those three roundings (everything else exact) already leaves d_beta at
1.9e-2 rel-L2 at K = 64 (5e-3 at K = 128) while every other gradient stays
below 3.5e-3, so the 3e-2 bound of the bf16 GPU test
(test_gpu_chunk.py::test_extreme_decay_16bit_forward_backward) is set by the
storage precision, not by a kernel defect; the fp32 path reaches 7e-6 there.
"""

import torch

from gdn2_testutil import make_inputs, np_, rel
from oracle import gdn2_oracle as O

NAMES = ("q", "k", "v", "g", "b", "w")


def _bf16(x):
    return x.to(torch.bfloat16).to(torch.float64)


class _RoundGrad(torch.autograd.Function):
    """Identity whose backward rounds the incoming gradient to bf16 (a
    gradient that the backward stores in the token dtype)."""

    @staticmethod
    def forward(ctx, x):
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        return _bf16(g)


def _chunk_head(q, k, v, g, b, w, h0, scale, round_kd, round_dh, round_dvn, C=64):
    """Relative-decay chunk form of one head in float64 (gdn2.py:243-369 up to
    the decay factoring): VN = A Z - A E h,  o = Qg h + Aqk VN,
    h' = e^{G_last} h + Kd^T VN."""
    T, K = q.shape
    qn = q / q.norm(dim=-1, keepdim=True)
    kn = k / k.norm(dim=-1, keepdim=True)
    h, outs = h0, []
    for c0 in range(0, T, C):
        c1 = min(T, c0 + C)
        n = c1 - c0
        G = torch.cumsum(g[c0:c1], 0)
        qc, kc, bc = qn[c0:c1], kn[c0:c1], b[c0:c1]
        Z = v[c0:c1] * w[c0:c1]
        Kd = kc * torch.exp(G[-1] - G)
        if round_kd:
            Kd = Kd + (_bf16(Kd) - Kd).detach()
        causal = torch.tril(torch.ones(n, n, dtype=torch.bool))[..., None]
        ex = torch.exp(torch.where(causal, G[:, None, :] - G[None, :, :],
                                   torch.full((n, n, K), -1e4, dtype=G.dtype)))
        Akk = torch.einsum("rc,ic,ric->ri", bc * kc, kc, ex).tril(-1)
        Aqk = torch.einsum("rc,ic,ric->ri", scale * qc, kc, ex).tril(0)
        A = torch.linalg.inv(torch.eye(n, dtype=G.dtype) + Akk)
        VN = A @ Z - (A @ (bc * kc * torch.exp(G))) @ h
        if round_dvn:
            VN = _RoundGrad.apply(VN)
        outs.append((scale * qc * torch.exp(G)) @ h + Aqk @ VN)
        h = torch.exp(G[-1])[:, None] * h + Kd.T @ VN
        if round_dh:
            h = _RoundGrad.apply(h)
    return torch.cat(outs, 0), h


def _grads(d, do, dht, **rounding):
    leaves = {n: d[n].double().clone().requires_grad_() for n in (*NAMES, "h0")}
    K = d["q"].shape[-1]
    loss = 0.0
    for hh in range(d["q"].shape[2]):
        x = {n: leaves[n][0, :, hh] for n in NAMES}
        o, ht = _chunk_head(*(x[n] for n in NAMES), leaves["h0"][0, hh], K ** -0.5, **rounding)
        loss = loss + (o * do[0, :, hh].double()).sum() + (ht * dht[0, hh].double()).sum()
    loss.backward()
    return {n: leaves[n].grad.numpy() for n in NAMES}


def _case(K):
    d = make_inputs(1, 150, 2, K, K, seed=11, decay=-6.0, dtype=torch.bfloat16)
    gen = torch.Generator().manual_seed(13)
    do = torch.randn(1, 150, 2, K, generator=gen).bfloat16().float()
    dht = torch.randn(1, 2, K, K, generator=gen)
    ref = O.recurrent_bwd(*np_(d, NAMES), do.numpy(), d["h0"].numpy(), dht.numpy(),
                          norm_mode="fla")
    return d, do, dht, dict(zip(NAMES, ref))


def test_exact_chunk_form_matches_oracle():
    d, do, dht, ref = _case(64)
    gr = _grads(d, do, dht, round_kd=False, round_dh=False, round_dvn=False)
    for n in NAMES:
        assert rel(gr[n], ref[n]) < 1e-6, n


def test_token_dtype_storage_alone_sets_the_d_beta_bound():
    for K, lo, hi in ((64, 1.5e-2, 2.5e-2), (128, 3e-3, 8e-3)):
        d, do, dht, ref = _case(K)
        gr = _grads(d, do, dht, round_kd=True, round_dh=True, round_dvn=True)
        assert lo < rel(gr["b"], ref["b"]) < hi, K
        for n in ("q", "k", "v", "w"):
            assert rel(gr[n], ref[n]) < 4e-3, (K, n)

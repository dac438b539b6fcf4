"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run once in a container where the reference checkout is importable:

    PYTHONPATH=<reference>/src python tests/golden/make_golden.py <reference>/src

It imports the reference's own pure-PyTorch GDN-2 functions
(``qwendopamine.models.gdn2.gdn2.torch_recurrent_gdn2`` and
``torch_chunk_gdn2``, gdn2.py:100-369), runs them on seeded inputs, and stores
inputs, outputs, final states and autograd gradients as ``.npz`` files next to
this script.  Nothing at test time imports the reference: the GPU box has no
copy of it, and the fixtures travel instead.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))


def _ref():
    if len(sys.argv) > 1:
        sys.path.insert(0, sys.argv[1])
    from qwendopamine.models.gdn2.gdn2 import torch_chunk_gdn2, torch_recurrent_gdn2

    return torch_recurrent_gdn2, torch_chunk_gdn2


def _np(t):
    return t.detach().to(torch.float32).cpu().numpy()


def _grads(fn, tensors, do, dht, **kw):
    q, k, v, g, b, w, h0 = tensors
    o, ht = fn(q=q, k=k, v=v, g=g, b=b, w=w, initial_state=h0,
               output_final_state=True, **kw)
    loss = (o * do).sum() + (ht * dht).sum()
    gr = torch.autograd.grad(loss, tensors)
    return o, ht, gr


def small_case(rec, chk):
    """Reference-test recipe (test_gdn2.py:116-124) with a nonzero init state."""
    out = {}
    torch.manual_seed(42)
    B, T, H, K, V = 2, 41, 4, 16, 16
    q = torch.randn(B, T, H, K)
    k = torch.randn(B, T, H, K)
    v = torch.randn(B, T, H, V)
    g = -torch.rand(B, T, H, K).abs()
    b = torch.sigmoid(torch.randn(B, T, H, K))
    w = torch.sigmoid(torch.randn(B, T, H, V))
    h0 = torch.randn(B, H, K, V) * 0.1
    do = torch.randn(B, T, H, V)
    dht = torch.randn(B, H, K, V)
    tensors = [x.clone().requires_grad_() for x in (q, k, v, g, b, w, h0)]
    o, ht, gr = _grads(rec, tensors, do, dht)
    for n, x in zip(("q", "k", "v", "g", "b", "w", "h0", "do", "dht"),
                    (q, k, v, g, b, w, h0, do, dht)):
        out[n] = _np(x)
    out["o_rec"], out["ht_rec"] = _np(o), _np(ht)
    for n, x in zip(("dq", "dk", "dv", "dg", "db", "dw", "dh0"), gr):
        out[n + "_rec"] = _np(x)
    for cs in (8, 33, 64):
        oc, hc = chk(q=q, k=k, v=v, g=g, b=b, w=w, initial_state=h0,
                     output_final_state=True, chunk_size=cs)
        out[f"o_chunk{cs}"], out[f"ht_chunk{cs}"] = _np(oc), _np(hc)
    np.savez_compressed(os.path.join(HERE, "ref_small.npz"), **out)


def config0_case(rec, chk):
    """B=1 T=512 H=4 K=V=64, fp32, zero init, seed 0.

    Scalar beta and scalar log-decay per token per head are broadcast through
    the channel-wise API: g -> [..,K], b = beta -> [..,K], w = beta -> [..,V].
    Draw order q, k, v, beta, g.
    """
    torch.manual_seed(0)
    B, T, H, K, V = 1, 512, 4, 64, 64
    q = F.normalize(torch.randn(B, T, H, K), dim=-1)
    k = F.normalize(torch.randn(B, T, H, K), dim=-1)
    v = torch.randn(B, T, H, V)
    beta = torch.sigmoid(torch.randn(B, T, H))
    gs = F.logsigmoid(torch.randn(B, T, H) + 3.0)
    g = gs[..., None].expand(B, T, H, K).contiguous()
    b = beta[..., None].expand(B, T, H, K).contiguous()
    w = beta[..., None].expand(B, T, H, V).contiguous()
    o_c, h_c = chk(q=q, k=k, v=v, g=g, b=b, w=w, output_final_state=True,
                   chunk_size=64)
    o_r, h_r = rec(q=q, k=k, v=v, g=g, b=b, w=w, output_final_state=True)
    # Inputs are regenerated at test time from the same seed (torch's CPU
    # generator is deterministic for a given torch version); a fingerprint of
    # each input is stored so a drift in the generator is caught.
    fp = {f"fp_{n}": np.array([_np(x).sum(), (_np(x) ** 2).sum(), *_np(x).ravel()[:4]])
          for n, x in (("q", q), ("k", k), ("v", v), ("beta", beta), ("g", gs))}
    np.savez_compressed(
        os.path.join(HERE, "config0.npz"),
        o_chunk=_np(o_c), ht_chunk=_np(h_c), o_rec=_np(o_r), ht_rec=_np(h_r), **fp,
    )


def strong_decay_case(rec, chk):
    """Per-token log-decay -2 on every channel: the reference chunk oracle's
    absolute-gamma form underflows here, the recurrent form stays exact."""
    torch.manual_seed(5)
    B, T, H, K, V = 1, 130, 2, 32, 32
    q = torch.randn(B, T, H, K)
    k = torch.randn(B, T, H, K)
    v = torch.randn(B, T, H, V)
    g = torch.full((B, T, H, K), -2.0)
    b = torch.sigmoid(torch.randn(B, T, H, K))
    w = torch.sigmoid(torch.randn(B, T, H, V))
    h0 = torch.randn(B, H, K, V) * 0.1
    o_r, h_r = rec(q=q, k=k, v=v, g=g, b=b, w=w, initial_state=h0,
                   output_final_state=True)
    o_c, h_c = chk(q=q, k=k, v=v, g=g, b=b, w=w, initial_state=h0,
                   output_final_state=True, chunk_size=64)
    np.savez_compressed(
        os.path.join(HERE, "strong_decay.npz"),
        q=_np(q), k=_np(k), v=_np(v), g=_np(g), b=_np(b), w=_np(w), h0=_np(h0),
        o_rec=_np(o_r), ht_rec=_np(h_r), o_chunk=_np(o_c), ht_chunk=_np(h_c),
    )


def decode_case(rec):
    """Config-2 recipe at a reduced batch: T=1 steps on an N(0,0.02) state,
    bf16-representable inputs, three consecutive steps chained; the state
    after the third step is stored."""
    torch.manual_seed(11)
    B, H, K, V = 2, 2, 128, 128
    h = torch.randn(B, H, K, V) * 0.02
    out = {"h0": _np(h)}
    for step in range(3):
        q = F.normalize(torch.randn(B, 1, H, K), dim=-1).bfloat16().float()
        k = F.normalize(torch.randn(B, 1, H, K), dim=-1).bfloat16().float()
        v = torch.randn(B, 1, H, V).bfloat16().float()
        beta = torch.sigmoid(torch.randn(B, 1, H)).bfloat16().float()
        gs = F.logsigmoid(torch.randn(B, 1, H) + 3.0)
        g = gs[..., None].expand(B, 1, H, K).contiguous()
        b = beta[..., None].expand(B, 1, H, K).contiguous()
        w = beta[..., None].expand(B, 1, H, V).contiguous()
        o, h = rec(q=q, k=k, v=v, g=g, b=b, w=w, initial_state=h,
                   output_final_state=True)
        for n, x in zip(("q", "k", "v", "g", "b", "w", "o"),
                        (q, k, v, g, b, w, o)):
            out[f"{n}{step}"] = _np(x)
    out["ht"] = _np(h)
    np.savez_compressed(os.path.join(HERE, "decode.npz"), **out)


def main():
    rec, chk = _ref()
    torch.set_num_threads(8)
    small_case(rec, chk)
    config0_case(rec, chk)
    strong_decay_case(rec, chk)
    decode_case(rec)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()

"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run once in a container where the reference checkout is importable:

    PYTHONPATH=<reference>/src python tests/golden/make_golden.py <reference>/src

It imports the reference's own pure-PyTorch GDN-2 functions
(``qwendopamine.models.gdn2.gdn2.torch_recurrent_gdn2`` and
``torch_chunk_gdn2``, gdn2.py:100-369), its block pieces and its whole
``GatedDeltaNet2`` module, runs them on seeded inputs, and stores inputs,
outputs, final states, caches, state_dicts and autograd gradients as ``.npz``
files next to this script.  Nothing at test time imports the reference: the GPU box has no
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


def block_ops_case():
    """The reference's ShortConvolution and RMSNormGated (gdn2.py:372-452):
    fp32 with autograd gradients, a one-token decode step through the cache,
    and bf16 forwards (the reference evaluates both in the input dtype)."""
    from qwendopamine.models.gdn2.gdn2 import RMSNormGated, ShortConvolution

    out = {}
    torch.manual_seed(11)
    B, T, D = 2, 37, 48
    for tag, W, bias, act in (("a", 4, True, "silu"), ("b", 3, False, None)):
        m = ShortConvolution(D, kernel_size=W, bias=bias, activation=act)
        with torch.no_grad():
            m.conv1d.weight.normal_(0.0, 0.5)
            if bias:
                m.conv1d.bias.normal_(0.0, 0.5)
        x = torch.randn(B, T, D, requires_grad=True)
        y, cache = m(x, output_final_state=True)
        dy = torch.randn_like(y)
        params = [x, m.conv1d.weight] + ([m.conv1d.bias] if bias else [])
        gr = torch.autograd.grad((y * dy).sum(), params)
        out[f"conv_{tag}_x"] = _np(x)
        out[f"conv_{tag}_w"] = _np(m.conv1d.weight)
        if bias:
            out[f"conv_{tag}_bias"] = _np(m.conv1d.bias)
            out[f"conv_{tag}_dbias"] = _np(gr[2])
        out[f"conv_{tag}_y"] = _np(y)
        out[f"conv_{tag}_cache"] = _np(cache)
        out[f"conv_{tag}_dy"] = _np(dy)
        out[f"conv_{tag}_dx"] = _np(gr[0])
        out[f"conv_{tag}_dw"] = _np(gr[1])
        if tag == "a":
            # one decode step with a cache: the cache is prepended
            c0 = torch.randn(B, D, W - 1)
            xt = torch.randn(B, 1, D)
            with torch.no_grad():
                yt, c1 = m(xt, cache=c0, output_final_state=True)
            out["conv_dec_cache"], out["conv_dec_x"] = _np(c0), _np(xt)
            out["conv_dec_y"], out["conv_dec_new_cache"] = _np(yt), _np(c1)
            # bf16 forward
            mb = ShortConvolution(D, kernel_size=W, bias=bias, activation=act).bfloat16()
            with torch.no_grad():
                mb.conv1d.weight.copy_(m.conv1d.weight)
                mb.conv1d.bias.copy_(m.conv1d.bias)
                yb, _ = mb(x.detach().bfloat16())
            out["conv_bf16_w"] = _np(mb.conv1d.weight)
            out["conv_bf16_bias"] = _np(mb.conv1d.bias)
            out["conv_bf16_y"] = _np(yb)

    N = 32
    norm = RMSNormGated(N, eps=1e-5)
    with torch.no_grad():
        norm.weight.normal_(1.0, 0.3)
    x = torch.randn(2, 9, 3, N, requires_grad=True)
    z = torch.randn(2, 9, 3, N, requires_grad=True)
    y = norm(x, z)
    dy = torch.randn_like(y)
    gx, gz, gw = torch.autograd.grad((y * dy).sum(), (x, z, norm.weight))
    out.update(norm_x=_np(x), norm_z=_np(z), norm_w=_np(norm.weight), norm_y=_np(y),
               norm_dy=_np(dy), norm_dx=_np(gx), norm_dz=_np(gz), norm_dw=_np(gw))
    with torch.no_grad():
        xb, zb = x.detach().bfloat16(), z.detach().bfloat16()
        out["norm_bf16_y"] = _np(norm.bfloat16()(xb, zb))           # bf16 weight
        out["norm_bf16_w"] = _np(norm.weight)
        norm32 = RMSNormGated(N, eps=1e-5)
        norm32.weight.copy_(torch.from_numpy(out["norm_w"]))
        out["norm_bf16w32_y"] = _np(norm32(xb, zb))                # fp32 weight: fp32 result
    np.savez_compressed(os.path.join(HERE, "block_ops.npz"), **out)


def module_case():
    """The reference's whole ``GatedDeltaNet2`` module (gdn2.py:488-1004),
    fp32, on its exact token-serial backend (``torch-recurrent``): for each
    case the seeded initial state_dict, a training-mode forward with the cache
    returned (output, recurrent state, the three conv states), the gradients
    of sum(out * dy) for every parameter, and (unpadded cases) one eval-mode
    decode step through that cache.

    The padded case packs a single sequence: with one sequence per batch the
    reference's pure-PyTorch core (which does not take ``cu_seqlens``) and its
    GPU core (which does) agree, and the B200 module follows the GPU core.
    """
    from qwendopamine.models.gdn2.gdn2 import GatedDeltaNet2

    sys.path.insert(0, os.path.dirname(HERE))
    from module_cases import MODULE_CASES

    out = {}
    for name, (kw, seed, Bs, Ts, pad) in MODULE_CASES.items():
        torch.manual_seed(seed)
        m = GatedDeltaNet2(layer_idx=0, backend="torch-recurrent", **kw)
        for n, p in m.state_dict().items():
            out[f"{name}.sd.{n}"] = _np(p)
        m.train()
        gen = torch.Generator().manual_seed(100 + seed)
        x = torch.randn(Bs, Ts, kw["hidden_size"], generator=gen)
        dy = torch.randn(Bs, Ts, kw["hidden_size"], generator=gen)
        out[f"{name}.x"], out[f"{name}.dy"] = _np(x), _np(dy)
        if pad:
            mask = torch.ones(Bs, Ts, dtype=torch.long)
            mask[0, :pad] = 0
            out[f"{name}.mask"] = mask.numpy()
            y, _, _ = m(x, attention_mask=mask)
        else:
            cache = {}
            y, _, cache = m(x, past_key_values=cache, use_cache=True)
            out[f"{name}.rec"] = _np(cache["recurrent_state"])
            for tag, c in zip("qkv", cache["conv_state"]):
                out[f"{name}.conv_{tag}"] = _np(c)
        out[f"{name}.out"] = _np(y)
        params = dict(m.named_parameters())
        gr = torch.autograd.grad((y * dy).sum(), list(params.values()))
        for n, g_ in zip(params, gr):
            out[f"{name}.grad.{n}"] = _np(g_)
        if not pad:
            # one decode step through the cache (eval: the recurrent mode)
            m.eval()
            x1 = torch.randn(Bs, 1, kw["hidden_size"], generator=gen)
            with torch.no_grad():
                y1, _, cache = m(x1, past_key_values=cache, use_cache=True)
            out[f"{name}.x1"], out[f"{name}.out1"] = _np(x1), _np(y1)
            out[f"{name}.rec1"] = _np(cache["recurrent_state"])
            for tag, c in zip("qkv", cache["conv_state"]):
                out[f"{name}.conv1_{tag}"] = _np(c)
    np.savez_compressed(os.path.join(HERE, "module.npz"), **out)


def main():
    rec, chk = _ref()
    torch.set_num_threads(8)
    small_case(rec, chk)
    config0_case(rec, chk)
    strong_decay_case(rec, chk)
    decode_case(rec)
    block_ops_case()
    module_case()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()

"""Sequence-parallel GDN-2 kernels on one GPU.

P ranks are emulated in one process through the C ABI: every span runs the
intra kernel and the pre-scan, the span maps are stacked (what the NCCL
all-gather produces), each span folds its predecessors with gdn2_cp_merge and
runs its state pass; the backward mirrors it.  Outputs, the final state and
all gradients must match the float64 oracle on the whole sequence.
"""

import numpy as np
import pytest
import torch

from gdn2_testutil import make_inputs, np_, rel, to_dev
from oracle import gdn2_oracle as O
from qwendopamine_b200 import _native as N

pytestmark = pytest.mark.gpu
NAMES = ("q", "k", "v", "g", "b", "w")


def _spans(T, P):
    nch = (T + 63) // 64
    per = nch // P
    cuts = [0] + [min(T, 64 * per * (r + 1)) for r in range(P - 1)] + [T]
    return [(cuts[r], cuts[r + 1]) for r in range(P)]


def _emulate(d, P, dtype, dev, do, dht, prescan_ws=False):
    lib = N.load()
    B, T, H, K = d["q"].shape
    V = d["v"].shape[-1]
    x = to_dev(d, dev, dtype)
    st = N.stream_of(dev)
    ranks = []
    for (a, e) in _spans(T, P):
        loc = {n: x[n][:, a:e].contiguous() for n in NAMES}
        tab = N.seq_tables(B, e - a, dev)
        prob = N.ChunkProblem(H, K, V, N.dtype_code(dtype), 1, K ** -0.5, tab.struct())
        sb = lib.gdn2_chunk_saved_bytes(prob)
        saved = torch.empty(sb, dtype=torch.uint8, device=dev)
        N.check(lib.gdn2_chunk_fwd_intra(prob, *(N.ptr(loc[n]) for n in NAMES), N.ptr(saved), sb,
                                         st), "intra")
        hm = torch.empty(B, H, K, V + K, device=dev)
        N.check(lib.gdn2_cp_fwd_prescan(prob, N.ptr(saved), sb, N.ptr(hm), None, 0, st), "pre")
        ranks.append(dict(a=a, e=e, loc=loc, tab=tab, prob=prob, sb=sb, saved=saved, hm=hm))
    hm_all = torch.stack([r["hm"] for r in ranks])
    outs, hts = [], []
    for i, r in enumerate(ranks):
        h0 = torch.empty(B, H, K, V, device=dev)
        N.check(lib.gdn2_cp_merge(r["prob"], N.ptr(hm_all), None, i, P, 1, N.ptr(x["h0"]),
                                  N.ptr(h0), st), "merge")
        o = torch.empty_like(r["loc"]["v"])
        ht = torch.empty(B, H, K, V, device=dev)
        N.check(lib.gdn2_chunk_fwd_state(r["prob"], N.ptr(h0), N.ptr(o), N.ptr(ht),
                                         N.ptr(r["saved"]), r["sb"], st), "state")
        outs.append(o)
        hts.append(ht)
    # backward
    dod = do.to(dev, dtype)
    dhtd = dht.to(dev)
    for i, r in enumerate(ranks):
        r["do"] = dod[:, r["a"]:r["e"]].contiguous()
        r["dhm"] = torch.empty(B, H, K, V, device=dev)
        pb = lib.gdn2_cp_workspace_bytes(r["prob"]) if prescan_ws else 0
        pws = torch.empty(max(pb, 1), dtype=torch.uint8, device=dev)
        N.check(lib.gdn2_cp_bwd_prescan(r["prob"], N.ptr(r["saved"]), r["sb"], N.ptr(r["do"]),
                                        N.ptr(dhtd) if i == P - 1 else None, N.ptr(r["dhm"]),
                                        N.ptr(pws) if pb else None, pb, st), "bwd pre")
    dhm_all = torch.stack([r["dhm"] for r in ranks])
    grads = {n: [] for n in (*NAMES, "h0")}
    for i, r in enumerate(ranks):
        if i == P - 1:
            dh_end = dhtd
        else:
            dh_end = torch.empty(B, H, K, V, device=dev)
            N.check(lib.gdn2_cp_merge(r["prob"], N.ptr(hm_all), N.ptr(dhm_all), i, P, 0, None,
                                      N.ptr(dh_end), st), "merge bwd")
        wb = lib.gdn2_chunk_bwd_workspace_bytes(r["prob"])
        ws = torch.empty(wb, dtype=torch.uint8, device=dev)
        gr = {n: torch.empty_like(r["loc"][n]) for n in NAMES}
        dh0 = torch.empty(B, H, K, V, device=dev)
        N.check(lib.gdn2_chunk_bwd(r["prob"], *(N.ptr(r["loc"][n]) for n in NAMES),
                                   N.ptr(r["saved"]), r["sb"], N.ptr(r["do"]), N.ptr(dh_end),
                                   *(N.ptr(gr[n]) for n in NAMES), N.ptr(dh0), N.ptr(ws), wb, st),
                "bwd")
        for n in NAMES:
            grads[n].append(gr[n])
        if i == 0:
            grads["h0"].append(dh0)
    torch.cuda.synchronize(dev)
    o = torch.cat(outs, 1)
    g = {n: torch.cat(v, 1) for n, v in grads.items() if n != "h0"}
    g["h0"] = grads["h0"][0]
    return o, hts[-1], g


@pytest.mark.parametrize("P,T", [(2, 256), (4, 300), (8, 1030), (3, 64 * 3)])
def test_sequence_parallel_matches_full_sequence_fp32(cuda_device, P, T):
    B, H, K, V = 2, 2, 64, 64
    d = make_inputs(B, T, H, K, V, seed=P * T)
    gen = torch.Generator().manual_seed(P)
    do = torch.randn(B, T, H, V, generator=gen)
    dht = torch.randn(B, H, K, V, generator=gen)
    o, ht, g = _emulate(d, P, torch.float32, cuda_device, do, dht)
    args = np_(d, NAMES)
    ro, rh = O.recurrent_fwd(*args, d["h0"].numpy(), norm_mode="fla")
    assert rel(o, ro) < 1e-4 and rel(ht, rh) < 1e-4
    ref = O.recurrent_bwd(*args, do.numpy(), d["h0"].numpy(), dht.numpy(), norm_mode="fla")
    for n, r in zip((*NAMES, "h0"), ref):
        assert rel(g[n], r) < 1e-4, n


@pytest.mark.parametrize("prescan_ws", [False, True])
def test_sequence_parallel_config4_recipe_bf16(cuda_device, prescan_ws):
    """Config-4 recipe (scalar beta / decay broadcast, bf16) on 8 spans of a
    shortened sequence with H=32 heads; the backward pre-scan as the
    register-state pass and, given a workspace, as the tensor-core state
    pass."""
    P, B, T, H, K, V = 8, 1, 8 * 128, 32, 128, 128
    d = make_inputs(B, T, H, K, V, seed=4, decay="baseline", dtype=torch.bfloat16,
                    scalar_gates=True, h0=False)
    d["h0"] = torch.zeros(B, H, K, V)
    gen = torch.Generator().manual_seed(8)
    do = torch.randn(B, T, H, V, generator=gen).bfloat16().float()
    dht = torch.randn(B, H, K, V, generator=gen) if prescan_ws else torch.zeros(B, H, K, V)
    o, ht, g = _emulate(d, P, torch.bfloat16, cuda_device, do, dht, prescan_ws=prescan_ws)
    args = np_(d, NAMES)
    ro, rh = O.recurrent_fwd(*args, None, norm_mode="fla")
    assert rel(o, ro) < 2e-2 and rel(ht, rh) < 2e-2
    ref = O.recurrent_bwd(*args, do.numpy(), None, dht.numpy() if prescan_ws else None,
                          norm_mode="fla")
    for n, r in zip(NAMES, ref):
        assert rel(g[n], r) < 2e-2, n


def test_cp_autograd_function_single_rank_equals_chunk(cuda_device):
    from qwendopamine_b200 import chunk_gdn2
    from qwendopamine_b200.gdn2_ops.cp import chunk_gdn2_cp

    d = make_inputs(1, 200, 2, 64, 64, seed=2)
    x = to_dev(d, cuda_device, torch.float32)
    l1 = {n: x[n].clone().requires_grad_() for n in (*NAMES, "h0")}
    l2 = {n: x[n].clone().requires_grad_() for n in (*NAMES, "h0")}
    o1, h1 = chunk_gdn2_cp(*(l1[n] for n in NAMES), rank=0, world=1,
                           gather=lambda t: t[None], initial_state=l1["h0"])
    o2, h2 = chunk_gdn2(*(l2[n] for n in NAMES), initial_state=l2["h0"], output_final_state=True,
                        use_qk_l2norm_in_kernel=True)
    assert rel(o1, o2) < 1e-6 and rel(h1, h2) < 1e-6
    gen = torch.Generator(device=cuda_device).manual_seed(0)
    do = torch.randn(o1.shape, device=cuda_device, generator=gen)
    dh = torch.randn(h1.shape, device=cuda_device, generator=gen)
    ((o1 * do).sum() + (h1 * dh).sum()).backward()
    ((o2 * do).sum() + (h2 * dh).sum()).backward()
    for n in (*NAMES, "h0"):
        assert rel(l1[n].grad, l2[n].grad) < 1e-6, n


def test_sequence_parallel_subspans_emulated_in_one_process(cuda_device):
    """Four ranks of chunk_gdn2_cp in one process, bf16, each rank's span of
    128 chunks cut into four sub-spans joined by the fp32 span-map folds, a
    slow decay so every span's state reaches the next ones, a loss on the
    outputs and on the last rank's end state: outputs, end state and all six
    gradients against chunk_gdn2 on the whole sequence.  The all-gathers are
    emulated in two passes (a span's map and its span-start gradient depend
    on that span alone, so a first pass records them)."""
    from qwendopamine_b200 import chunk_gdn2
    from qwendopamine_b200.gdn2_ops.cp import CPChunkGDN2Function, _sub_spans

    P, B, T, H, K, V = 4, 1, 4 * 8192, 2, 128, 128
    Tr = T // P
    assert _sub_spans(B, Tr, H, torch.bfloat16) == 4
    d = make_inputs(B, T, H, K, V, seed=21, decay=-0.00025, dtype=torch.bfloat16, h0=False)
    d["b"] = (d["b"] * 0.01).bfloat16().float()  # weak erasure: the state outlives a span
    x = to_dev(d, cuda_device, torch.bfloat16)
    gen = torch.Generator(device=cuda_device).manual_seed(5)
    do = torch.randn(B, T, H, V, device=cuda_device, generator=gen).bfloat16()
    dht = torch.randn(B, H, K, V, device=cuda_device, generator=gen)

    # whole sequence on one GPU
    full = {n: x[n].clone().requires_grad_() for n in NAMES}
    o_ref, ht_ref = chunk_gdn2(*(full[n] for n in NAMES), output_final_state=True,
                               use_qk_l2norm_in_kernel=True)
    ((o_ref.float() * do.float()).sum() + (ht_ref * dht).sum()).backward()

    # the spans are coupled: span 1 from a zero state differs from the truth
    with torch.no_grad():
        o_alone, _ = chunk_gdn2(*(x[n][:, Tr:2 * Tr] for n in NAMES), use_qk_l2norm_in_kernel=True)
    assert rel(o_alone, o_ref[:, Tr:2 * Tr]) > 5e-2

    rec = {"f": [None] * P, "b": [None] * P}

    def make_gather(r):
        def gather(t):
            key = "f" if t.shape[-1] == V + K else "b"
            rec[key][r] = t.detach().clone()
            return torch.stack([z if z is not None else torch.zeros_like(t) for z in rec[key]])
        return gather

    def run():
        outs, hts, leaves = [], [], []
        for r in range(P):
            loc = {n: x[n][:, r * Tr:(r + 1) * Tr].detach().clone().requires_grad_() for n in NAMES}
            o, ht = CPChunkGDN2Function.apply(*(loc[n] for n in NAMES), None, K ** -0.5, True, r,
                                              P, make_gather(r))
            outs.append(o)
            hts.append(ht)
            leaves.append(loc)
        grads = [None] * P
        for r in reversed(range(P)):  # later ranks' span-start gradients first
            loss = (outs[r].float() * do[:, r * Tr:(r + 1) * Tr].float()).sum()
            if r == P - 1:
                loss = loss + (hts[r] * dht).sum()
            grads[r] = torch.autograd.grad(loss, [leaves[r][n] for n in NAMES])
        return outs, hts, grads

    run()  # records every span's map and span-start gradient
    outs, hts, grads = run()
    torch.cuda.synchronize(cuda_device)
    assert rel(torch.cat(outs, 1), o_ref) < 2e-2
    assert rel(hts[-1], ht_ref) < 2e-2
    for i, n in enumerate(NAMES):
        assert rel(torch.cat([g[i] for g in grads], 1), full[n].grad) < 2e-2, n


def test_chunk_gdn2_few_heads_long_sequence_takes_subspans(cuda_device):
    """chunk_gdn2 with few sequence-heads over a long sequence (B=1, H=2,
    T=32,768) runs the single-GPU sub-span path (eight sub-spans of 64
    chunks: pre-scan, one gdn2_cp_unfold launch per direction, state passes
    on the pieces); on spans that carry state into each other its outputs,
    final state and all gradients, the initial state's included, match the
    plain chunk path."""
    from qwendopamine_b200 import chunk_gdn2
    from qwendopamine_b200.gdn2_ops.chunk_gdn2 import ChunkGDN2Function
    from qwendopamine_b200.gdn2_ops.cp import sub_spans_single

    B, T, H, K, V = 1, 32768, 2, 128, 128
    assert sub_spans_single(B, T, H, K, V, torch.bfloat16) == 8
    d = make_inputs(B, T, H, K, V, seed=31, decay=-0.0005, dtype=torch.bfloat16, h0=True)
    d["b"] = (d["b"] * 0.01).bfloat16().float()  # weak erasure: the state outlives a piece
    x = to_dev(d, cuda_device, torch.bfloat16)
    gen = torch.Generator(device=cuda_device).manual_seed(6)
    do = torch.randn(B, T, H, V, device=cuda_device, generator=gen).bfloat16()
    dht = torch.randn(B, H, K, V, device=cuda_device, generator=gen)

    l1 = {n: x[n].clone().requires_grad_() for n in (*NAMES, "h0")}
    o1, h1 = chunk_gdn2(*(l1[n] for n in NAMES), initial_state=l1["h0"], output_final_state=True,
                        use_qk_l2norm_in_kernel=True)
    ((o1.float() * do.float()).sum() + (h1 * dht).sum()).backward()

    l2 = {n: x[n].clone().requires_grad_() for n in (*NAMES, "h0")}
    tables = N.seq_tables(B, T, cuda_device)
    o2, h2 = ChunkGDN2Function.apply(*(l2[n] for n in NAMES), K ** -0.5, l2["h0"], True, True,
                                     tables, torch.float32, None, None, None)
    ((o2.float() * do.float()).sum() + (h2 * dht).sum()).backward()
    torch.cuda.synchronize(cuda_device)
    assert rel(o1, o2) < 2e-2 and rel(h1, h2) < 2e-2
    for n in (*NAMES, "h0"):
        assert rel(l1[n].grad, l2[n].grad) < 2e-2, n

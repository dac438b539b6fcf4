"""The PyTorch CPU port used for the CPU baseline reproduces the reference's
own outputs and autograd gradients (golden fixtures)."""

import os

import numpy as np
import torch

from gdn2_testutil import rel
from oracle import gdn2_torch_port as P

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_port_chunk_forward_and_autograd_match_reference():
    d = np.load(os.path.join(GOLD, "ref_small.npz"))
    names = ("q", "k", "v", "g", "b", "w", "h0")
    t = {n: torch.from_numpy(d[n]).requires_grad_() for n in names}
    o, ht = P.chunk_fwd(*(t[n] for n in names[:-1]), t["h0"], chunk_size=64)
    assert rel(o, d["o_chunk64"]) < 1e-5 and rel(ht, d["ht_chunk64"]) < 1e-5
    ((o * torch.from_numpy(d["do"])).sum() + (ht * torch.from_numpy(d["dht"])).sum()).backward()
    for n in names:
        assert rel(t[n].grad, d[f"d{n}_rec"]) < 1e-4, n


def test_port_decode_matches_reference_chain():
    d = np.load(os.path.join(GOLD, "decode.npz"))
    h = torch.from_numpy(d["h0"]).clone()
    for s in range(3):
        o, h = P.recurrent_step(*(torch.from_numpy(d[f"{n}{s}"]) for n in
                                  ("q", "k", "v", "g", "b", "w")), h)
        assert rel(o, d[f"o{s}"]) < 1e-5
    assert rel(h, d["ht"]) < 1e-6

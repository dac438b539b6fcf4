"""The overlapped path (state passes on a second stream beside the
intra-chunk kernels of neighbouring pieces of the sequence) against the
one-stream chunk path and the float64 oracle.

With the state passes at the one-stream path's width (the value-half pass
for these head counts) the pieces run the same kernels on the same chunks
and hand the fp32 state (forward) and state gradient (backward) from piece
to piece, so every output and gradient must equal the one-stream path's bit
for bit.  At the widths the overlapped path picks by default (full-width
state passes beside the intra kernels) the state products are summed in
another order, so that configuration is checked against the float64 oracle.
"""

import pytest
import torch

from gdn2_testutil import TOL, make_inputs, np_, rel, to_dev
from oracle import gdn2_oracle as O
from qwendopamine_b200 import _native as N
from qwendopamine_b200 import chunk_gdn2
from qwendopamine_b200.gdn2_ops.chunk_gdn2 import ChunkGDN2Function
from qwendopamine_b200.gdn2_ops.overlap import OverlapChunkGDN2Function, overlap_pieces

pytestmark = pytest.mark.gpu
NAMES = ("q", "k", "v", "g", "b", "w")


@pytest.fixture
def one_stream_widths(monkeypatch):
    """State passes at the width the one-stream path uses (value halves)."""
    from qwendopamine_b200.gdn2_ops import overlap as OV

    monkeypatch.setattr(OV, "FULL_WIDTH", {"fwd": False, "bwd": False})


def _leaves(x):
    return [x[n].clone().requires_grad_() for n in NAMES]


def _run_plain(x, h0, do, dht, gate=None):
    lv = _leaves(x)
    B, T, H, K = x["q"].shape
    tables = N.seq_tables(B, T, x["q"].device)
    h = h0.clone().requires_grad_() if h0 is not None else None
    A, dtb = (gate or (None, None))
    A = A.clone().requires_grad_() if A is not None else None
    dtb = dtb.clone().requires_grad_() if dtb is not None else None
    o, ht = ChunkGDN2Function.apply(*lv, K ** -0.5, h, True, True, tables, torch.float32, A, dtb,
                                    None)
    extra = [t for t in (h, A, dtb) if t is not None]
    grads = torch.autograd.grad((o, ht), lv + extra, (do, dht))
    return o, ht, grads


def _run_overlap(x, h0, do, dht, pieces, gate=None):
    lv = _leaves(x)
    K = x["q"].shape[-1]
    h = h0.clone().requires_grad_() if h0 is not None else None
    A, dtb = (gate or (None, None))
    A = A.clone().requires_grad_() if A is not None else None
    dtb = dtb.clone().requires_grad_() if dtb is not None else None
    o, ht = OverlapChunkGDN2Function.apply(*lv, K ** -0.5, h, True, True, pieces, A, dtb, None)
    extra = [t for t in (h, A, dtb) if t is not None]
    grads = torch.autograd.grad((o, ht), lv + extra, (do, dht))
    return o, ht, grads


def _inputs(dev, T, H, seed, gate=False):
    d = make_inputs(1, T, H, 128, 128, seed=seed, decay="mild", dtype=torch.bfloat16)
    x = to_dev(d, dev, torch.bfloat16)
    gen = torch.Generator().manual_seed(seed + 1)
    do = torch.randn(1, T, H, 128, generator=gen).to(dev, torch.bfloat16)
    dht = (torch.randn(1, H, 128, 128, generator=gen) * 0.1).to(dev)
    g = None
    if gate:
        A = (torch.rand(H, generator=gen) * 0.5).to(dev)
        dtb = (torch.randn(H * 128, generator=gen) * 0.3).to(dev)
        x["g"] = (torch.randn(1, T, H, 128, generator=gen) - 2.0).to(dev)
        g = (A, dtb)
    return d, x, do, dht, g


@pytest.mark.parametrize("T,H,pieces,gate", [(64 * 70 + 17, 12, 3, False),
                                              (64 * 96, 24, 4, True),
                                              (64 * 9 + 1, 8, 2, False)])
def test_overlap_equals_one_stream_path(cuda_device, one_stream_widths, T, H, pieces, gate):
    d, x, do, dht, g = _inputs(cuda_device, T, H, seed=T + H, gate=gate)
    ref = _run_plain(x, x["h0"], do, dht, g)
    got = _run_overlap(x, x["h0"], do, dht, pieces, g)
    torch.cuda.synchronize()
    assert torch.equal(got[0], ref[0]), "o differs"
    assert torch.equal(got[1], ref[1]), "final state differs"
    for n, a, r in zip(["dq", "dk", "dv", "dg", "db", "dw", "dh0"], got[2], ref[2]):
        assert torch.equal(a, r), f"{n} differs (rel {rel(a, r):.3e})"
    if gate:
        # dA_log / d dt_bias are sums over every chunk, added with float
        # atomics, whose order changes with the launches: fp32 rounding only
        for n, a, r in zip(["dA_log", "ddt_bias"], got[2][7:], ref[2][7:]):
            assert rel(a, r) < 1e-5, f"{n}: rel {rel(a, r):.3e}"


@pytest.mark.parametrize("fwd_full,bwd_full", [(True, True), (False, False), (False, True)])
def test_overlap_matches_oracle(cuda_device, monkeypatch, fwd_full, bwd_full):
    """Two heads of an overlapped run against the float64 token-serial
    recurrence and its reverse pass, with the state passes at full width, in
    value halves, and mixed (value-half forward, full-width backward: what
    the cost model picks for 16 heads)."""
    from qwendopamine_b200.gdn2_ops import overlap as OV

    monkeypatch.setattr(OV, "FULL_WIDTH", {"fwd": fwd_full, "bwd": bwd_full})
    _check_oracle(cuda_device, 64 * 40 + 5, 10, 4, seed=7, hs=slice(3, 5))


def test_overlap_cost_model_plan_matches_oracle(cuda_device, monkeypatch):
    """The widths the cost model picks for 32 heads over three pieces: the
    first two forward state passes at full width beside the intra kernels,
    the third in value halves after them, the backward's first pass in
    value halves and the others at full width."""
    from qwendopamine_b200.gdn2_ops import overlap as OV

    monkeypatch.setattr(OV, "FULL_WIDTH", {"fwd": None, "bwd": None})
    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    if sms == 148:
        assert OV.forward_plan([32] * 3, 32, sms) == 2
        assert OV.full_width("bwd", 96, 32, sms)
    _check_oracle(cuda_device, 64 * 96, 32, 3, seed=11, hs=slice(30, 32))


def _check_oracle(dev, T, H, pieces, seed, hs):
    d, x, do, dht, _ = _inputs(dev, T, H, seed=seed)
    o, ht, grads = _run_overlap(x, x["h0"], do, dht, pieces)
    torch.cuda.synchronize()
    sub = {n: d[n][:, :, hs] for n in NAMES}
    args = np_(sub, NAMES)
    h0 = d["h0"][:, hs].double().numpy()
    do_ = do[:, :, hs].double().cpu().numpy()
    dht_ = dht[:, hs].double().cpu().numpy()
    ro, rh = O.recurrent_fwd(*args, h0, norm_mode="fla")
    rg = O.recurrent_bwd(*args, do_, h0, dht_, norm_mode="fla")
    tol = TOL[torch.bfloat16]
    assert rel(o[:, :, hs], ro) < tol
    assert rel(ht[:, hs], rh) < tol
    for n, a, r in zip(("dq", "dk", "dv", "dg", "db", "dw", "dh0"), grads, rg):
        a = a[:, hs] if n == "dh0" else a[:, :, hs]
        assert rel(a, r) < tol, n


def test_chunk_gdn2_routes_long_sequences_through_overlap(cuda_device, one_stream_widths):
    """chunk_gdn2 sends one 32,768-token sequence with 32 heads through the
    overlapped path (two pieces) and gives the one-stream path's results."""
    T, H = 32768, 32
    assert overlap_pieces(1, T, H, 128, 128, torch.bfloat16, cuda_device) == 2
    d, x, do, dht, _ = _inputs(cuda_device, T, H, seed=3)
    ref = _run_plain(x, x["h0"], do, dht)
    lv = _leaves(x)
    h = x["h0"].clone().requires_grad_()
    o, ht = chunk_gdn2(*lv, initial_state=h, output_final_state=True,
                       use_qk_l2norm_in_kernel=True)
    grads = torch.autograd.grad((o, ht), lv + [h], (do, dht))
    torch.cuda.synchronize()
    assert torch.equal(o, ref[0]) and torch.equal(ht, ref[1])
    for a, r in zip(grads, ref[2]):
        assert torch.equal(a, r)

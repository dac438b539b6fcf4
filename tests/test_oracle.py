"""Pin the CPU oracle to the reference's own outputs (tests/golden/*.npz).

The fixtures were produced by importing the reference's pure-PyTorch GDN-2
functions (see tests/golden/make_golden.py); these tests need no GPU.
"""

import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import gdn2_oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - np.asarray(b, np.float64))
                 / max(np.linalg.norm(np.asarray(b, np.float64)), 1e-30))


@pytest.fixture(scope="module")
def small():
    return np.load(os.path.join(GOLD, "ref_small.npz"))


def test_recurrent_forward_matches_reference(small):
    d = small
    o, ht = O.recurrent_fwd(d["q"], d["k"], d["v"], d["g"], d["b"], d["w"], d["h0"])
    assert rel(o, d["o_rec"]) < 1e-6
    assert rel(ht, d["ht_rec"]) < 1e-6


def test_recurrent_backward_matches_reference_autograd(small):
    d = small
    grads = O.recurrent_bwd(d["q"], d["k"], d["v"], d["g"], d["b"], d["w"], d["do"], d["h0"],
                            d["dht"])
    for name, x in zip(("dq", "dk", "dv", "dg", "db", "dw", "dh0"), grads):
        assert rel(x, d[name + "_rec"]) < 1e-6, name


@pytest.mark.parametrize("cs", [8, 33, 64])
def test_absolute_chunk_form_matches_reference_chunk(small, cs):
    d = small
    o, ht = O.chunk_fwd_absolute(d["q"], d["k"], d["v"], d["g"], d["b"], d["w"], d["h0"],
                                 chunk_size=cs)
    assert rel(o, d[f"o_chunk{cs}"]) < 1e-5
    assert rel(ht, d[f"ht_chunk{cs}"]) < 1e-5


@pytest.mark.parametrize("cs", [8, 33, 64])
def test_relative_chunk_form_matches_recurrence(small, cs):
    d = small
    o, ht, _ = O.chunk_fwd_relative(d["q"], d["k"], d["v"], d["g"], d["b"], d["w"], d["h0"],
                                    chunk_size=cs, norm_mode="torch")
    assert rel(o, d["o_rec"]) < 1e-6
    assert rel(ht, d["ht_rec"]) < 1e-6


def config0_inputs():
    """BASELINE config 0 inputs, regenerated from seed 0 (make_golden.py)."""
    torch.manual_seed(0)
    B, T, H, K, V = 1, 512, 4, 64, 64
    q = F.normalize(torch.randn(B, T, H, K), dim=-1)
    k = F.normalize(torch.randn(B, T, H, K), dim=-1)
    v = torch.randn(B, T, H, V)
    beta = torch.sigmoid(torch.randn(B, T, H))
    gs = F.logsigmoid(torch.randn(B, T, H) + 3.0)
    return q, k, v, beta, gs


def test_config0_inputs_regenerate_bit_exactly():
    d = np.load(os.path.join(GOLD, "config0.npz"))
    for name, x in zip(("q", "k", "v", "beta", "g"), config0_inputs()):
        x = x.numpy()
        fp = np.array([x.sum(), (x ** 2).sum(), *x.ravel()[:4]])
        np.testing.assert_array_equal(fp[2:], d[f"fp_{name}"][2:])
        np.testing.assert_allclose(fp[:2], d[f"fp_{name}"][:2], rtol=1e-6)


def test_config0_oracle_matches_reference():
    d = np.load(os.path.join(GOLD, "config0.npz"))
    q, k, v, beta, gs = (x.numpy() for x in config0_inputs())
    K = q.shape[-1]
    g = np.repeat(gs[..., None], K, -1)
    b = np.repeat(beta[..., None], K, -1)
    w = np.repeat(beta[..., None], v.shape[-1], -1)
    o, ht = O.recurrent_fwd(q, k, v, g, b, w)
    assert rel(o, d["o_rec"]) < 1e-6
    assert rel(ht, d["ht_rec"]) < 1e-6
    assert rel(o, d["o_chunk"]) < 1e-5


def test_strong_decay_reference_chunk_underflows_but_relative_form_is_exact():
    d = np.load(os.path.join(GOLD, "strong_decay.npz"))
    args = [d[n] for n in ("q", "k", "v", "g", "b", "w", "h0")]
    o, ht, _ = O.chunk_fwd_relative(*args, norm_mode="torch")
    assert rel(o, d["o_rec"]) < 1e-6
    # the reference's absolute-gamma chunk oracle is far off here
    assert rel(d["o_chunk"], d["o_rec"]) > 0.1
    oa, _ = O.chunk_fwd_absolute(*args)
    assert rel(oa, d["o_chunk"]) < 1e-4


def test_decode_chain_matches_reference():
    d = np.load(os.path.join(GOLD, "decode.npz"))
    h = d["h0"]
    for s in range(3):
        o, h = O.recurrent_fwd(*(d[f"{n}{s}"] for n in ("q", "k", "v", "g", "b", "w")), h)
        assert rel(o, d[f"o{s}"]) < 1e-5
    assert rel(h, d["ht"]) < 1e-6


def test_span_transition_composes_to_full_sequence(small):
    d = small
    sl = lambda x, a, b: x[:1, a:b]
    names = ("q", "k", "v", "g", "b", "w")
    full_o, full_h = O.recurrent_fwd(*(d[n][:1] for n in names), d["h0"][:1])
    h = d["h0"][:1].astype(np.float64)
    for a, b in ((0, 13), (13, 30), (30, 41)):
        M, he = O.span_transition(*(sl(d[n], a, b) for n in names), norm_mode="torch")
        h = np.einsum("bhij,bhjv->bhiv", M, h) + he
    assert rel(h, full_h) < 1e-9


def test_pieces_chained_by_state_and_state_gradient_give_the_whole_sequence(small):
    """The identity the overlapped path (pieces of one sequence, each its own
    problem) relies on: forward passes chained through their end states give
    the whole sequence's outputs and final state, and backward passes walked
    in reverse, each started from the start-state gradient of the piece after
    it, give the whole sequence's gradients."""
    d = small
    names = ("q", "k", "v", "g", "b", "w")
    x = {n: d[n][:1].astype(np.float64) for n in names}
    h0, do, dht = d["h0"][:1], d["do"][:1], d["dht"][:1]
    full_o, full_h = O.recurrent_fwd(*(x[n] for n in names), h0)
    full_g = O.recurrent_bwd(*(x[n] for n in names), do, h0, dht)
    cuts = [0, 13, 30, d["q"].shape[1]]
    pieces = list(zip(cuts[:-1], cuts[1:]))
    outs, starts, h = [], [], h0
    for a, b in pieces:
        starts.append(h)
        o, h = O.recurrent_fwd(*(x[n][:, a:b] for n in names), h)
        outs.append(o)
    assert rel(np.concatenate(outs, axis=1), full_o) < 1e-12
    assert rel(h, full_h) < 1e-12
    grads, d_end = [None] * len(pieces), dht
    for i in reversed(range(len(pieces))):
        a, b = pieces[i]
        grads[i] = O.recurrent_bwd(*(x[n][:, a:b] for n in names), do[:, a:b], starts[i], d_end)
        d_end = grads[i][6]
    for j, n in enumerate(("dq", "dk", "dv", "dg", "db", "dw")):
        assert rel(np.concatenate([g[j] for g in grads], axis=1), full_g[j]) < 1e-12, n
    assert rel(d_end, full_g[6]) < 1e-12


def test_varlen_oracle_keeps_sequences_independent(small):
    d = small
    names = ("q", "k", "v", "g", "b", "w")
    cat = [np.concatenate([d[n][0], d[n][1]], 0)[None] for n in names]
    T = d["q"].shape[1]
    o, hT = O.recurrent_fwd_varlen(*cat, [0, T, 2 * T], d["h0"])
    o_ref, h_ref = O.recurrent_fwd(*(d[n] for n in names), d["h0"])
    assert rel(o[0, :T], o_ref[0]) < 1e-9 and rel(o[0, T:], o_ref[1]) < 1e-9
    assert rel(hT, h_ref) < 1e-9


def test_normalize_modes_and_backward_are_consistent():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((5, 16))
    dy = rng.standard_normal((5, 16))
    for mode in ("torch", "fla"):
        y, den = O._normalize(x, mode=mode)
        dx = O._normalize_bwd(y, den, dy, mode=mode)
        eps = 1e-6
        num = np.zeros_like(x)
        for i in range(x.shape[0]):
            for j in range(x.shape[1]):
                xp, xm = x.copy(), x.copy()
                xp[i, j] += eps
                xm[i, j] -= eps
                num[i, j] = ((O._normalize(xp, mode=mode)[0] - O._normalize(xm, mode=mode)[0])
                             * dy).sum() / (2 * eps)
        assert rel(dx, num) < 1e-6

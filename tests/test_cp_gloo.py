"""Multi-process tests of the sequence-parallel exchange on CPU (gloo, 2 ranks).

The GPU kernels are not needed here: each rank computes its span map with the
oracle, the product's ``gather_span_maps`` exchanges them over gloo, and the
fold recurrences documented for ``gdn2_cp_merge`` are checked against the
whole-sequence oracle -- forward (initial states) and backward (end-state
gradients).  A second test makes one rank fail before the exchange and checks
that the survivor gets an error from the short process-group timeout instead
of hanging.
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    gen = torch.Generator().manual_seed(0)
    B, T, H, K, V = 1, 96, 2, 8, 8
    q = torch.randn(B, T, H, K, generator=gen)
    k = torch.randn(B, T, H, K, generator=gen)
    v = torch.randn(B, T, H, V, generator=gen)
    g = -torch.rand(B, T, H, K, generator=gen)
    b = torch.sigmoid(torch.randn(B, T, H, K, generator=gen))
    w = torch.sigmoid(torch.randn(B, T, H, V, generator=gen))
    h0 = torch.randn(B, H, K, V, generator=gen) * 0.1
    do = torch.randn(B, T, H, V, generator=gen)
    return [x.double().numpy() for x in (q, k, v, g, b, w, h0, do)]


def _end_state_grads(world, B, H, K, V):
    """A distinct seeded gradient for every rank's end state S_r."""
    rng = np.random.default_rng(11)
    return [rng.standard_normal((B, H, K, V)) for _ in range(world)]


def _worker_exchange(rank, world, port, out_q):
    import sys

    sys.path.insert(0, ROOT)
    from oracle import gdn2_oracle as O
    from qwendopamine_b200.gdn2_ops.cp import gather_span_maps

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        q, k, v, g, b, w, h0, do = _inputs()
        T = q.shape[1]
        span = T // world
        a, e = rank * span, (rank + 1) * span
        sl = lambda x: x[:, a:e]
        M, he = O.span_transition(*(sl(x) for x in (q, k, v, g, b, w)), norm_mode="torch")
        K, V = q.shape[-1], v.shape[-1]
        hm = np.concatenate([he, M], axis=-1)[0]               # [H, K, V+K]
        hm_all = gather_span_maps(torch.from_numpy(hm), None).numpy()
        # forward fold: x = h0; x = M_j x + h_e_j for j < rank
        x = h0[0]
        for j in range(rank):
            x = np.einsum("hkm,hmv->hkv", hm_all[j][..., V:], x) + hm_all[j][..., :V]
        # this rank's initial state must be the whole-sequence state at `a`
        _, ref_state = O.recurrent_fwd(*(x_[:, :a] for x_ in (q, k, v, g, b, w)), h0,
                                       norm_mode="torch")
        fwd_err = float(np.abs(x - ref_state[0]).max()) if a > 0 else float(np.abs(x - h0[0]).max())
        # backward, with a loss on every rank's end state S_j as well as on
        # the outputs (dht_j the gradient that reaches S_j directly): the
        # span-start gradient of the local outputs and of dht_r ...
        dhts = _end_state_grads(world, q.shape[0], q.shape[2], K, V)
        *_, dh_start = O.recurrent_bwd(*(sl(x_) for x_ in (q, k, v, g, b, w)), sl(do), x[None],
                                       dhts[rank], norm_mode="torch")
        dh_all = gather_span_maps(torch.from_numpy(dh_start[0]), None).numpy()
        # ... folded from the later ranks, plus this rank's own dht_r, is the
        # total gradient of S_r
        y = np.zeros_like(dh_start[0])
        for j in range(world - 1, rank, -1):
            y = np.einsum("hmk,hmv->hkv", hm_all[j][..., V:], y) + dh_all[j]
        y = y + dhts[rank][0]
        # reference: walk the later spans backwards from the final state,
        # adding each span end's own gradient
        ref = dhts[world - 1]
        for j in range(world - 1, rank, -1):
            a_j, e_j = j * span, (j + 1) * span
            *_, ref = O.recurrent_bwd(*(x_[:, a_j:e_j] for x_ in (q, k, v, g, b, w)),
                                      do[:, a_j:e_j], np.zeros_like(ref), ref, norm_mode="torch")
            ref = ref + dhts[j - 1]
        bwd_err = float(np.abs(y - ref[0]).max())
        order_ok = bool(np.allclose(hm_all[rank], hm))
        out_q.put((rank, fwd_err, bwd_err, order_ok))
    finally:
        dist.destroy_process_group()


def _worker_fail(rank, world, port, out_q):
    import sys

    sys.path.insert(0, ROOT)
    from qwendopamine_b200.gdn2_ops.cp import gather_span_maps

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        out_q.put((rank, "raised"))
        raise SystemExit(3)  # this rank dies before the exchange
    try:
        gather_span_maps(torch.zeros(4), None)
        out_q.put((rank, "no-error"))
    except Exception as exc:  # the timeout surfaces as an error, not a hang
        out_q.put((rank, f"error:{type(exc).__name__}"))


def _worker_conv_halo(rank, world, port, out_q):
    """Sequence-parallel short-convolution halo over gloo: each rank's prefix
    is its predecessor's last W-1 rows; the prefix gradient returns to that
    predecessor.  The oracle convolution of each span with its received
    prefix must equal the whole sequence's rows of that span, and the
    gradients routed back must complete each span's dx."""
    import sys

    sys.path.insert(0, ROOT)
    from oracle import block_oracle as BO
    from qwendopamine_b200.gdn2_ops.cp import ConvHaloFunction, gather_span_maps

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        gen = torch.Generator().manual_seed(5)
        B, T, D, W = 2, 7 * world, 8, 4
        x = torch.randn(B, T, D, generator=gen, dtype=torch.float64)
        wt = torch.randn(D, W, generator=gen, dtype=torch.float64)
        dy = torch.randn(B, T, D, generator=gen, dtype=torch.float64)
        span = T // world
        a, e = rank * span, (rank + 1) * span
        xs = x[:, a:e].clone().requires_grad_()
        prefix = ConvHaloFunction.apply(xs[:, -(W - 1):], rank, world,
                                        lambda t: gather_span_maps(t, None))
        want = x[:, a - (W - 1):a] if rank > 0 else torch.zeros(B, W - 1, D, dtype=x.dtype)
        prefix_ok = bool(torch.equal(prefix.detach(), want))
        y = BO.conv_fwd(xs.detach().numpy(), wt.numpy(), prefix=prefix.detach().numpy())
        y_full = BO.conv_fwd(x.numpy(), wt.numpy())[:, a:e]
        fwd_err = float(np.abs(y - y_full).max())
        # backward: this span's local dx and prefix gradient from the oracle,
        # the prefix gradient routed to the previous rank through the halo
        dx, _, _, dpre = BO.conv_bwd(xs.detach().numpy(), wt.numpy(), dy[:, a:e].numpy(),
                                     prefix=prefix.detach().numpy())
        prefix.backward(torch.from_numpy(dpre))
        dx_total = dx + xs.grad.numpy()
        dx_full = BO.conv_bwd(x.numpy(), wt.numpy(), dy.numpy())[0][:, a:e]
        bwd_err = float(np.abs(dx_total - dx_full).max())
        out_q.put((rank, prefix_ok, fwd_err, bwd_err))
    finally:
        dist.destroy_process_group()


def _run(fn, world, timeout):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    for _ in range(world):
        results.append(q.get(timeout=timeout))
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return sorted(results)


@pytest.mark.parametrize("world", [2, 3])
def test_span_map_exchange_and_fold_over_gloo(world):
    """Forward folds give every rank the whole sequence's state at its span
    start; backward folds, with a loss on the outputs and on every rank's end
    state, give every rank the whole loss's gradient of its end state."""
    res = _run(_worker_exchange, world, timeout=120)
    assert [r[0] for r in res] == list(range(world))
    for rank, fwd_err, bwd_err, order_ok in res:
        assert order_ok, rank
        assert fwd_err < 1e-10, (rank, fwd_err)
        assert bwd_err < 1e-10, (rank, bwd_err)


def test_dead_rank_surfaces_as_error_not_hang():
    res = _run(_worker_fail, 2, timeout=120)
    assert res[1] == (1, "raised")
    assert res[0][0] == 0 and res[0][1].startswith("error:")


def test_conv_halo_exchange_over_gloo():
    res = _run(_worker_conv_halo, 3, timeout=120)
    assert [r[0] for r in res] == [0, 1, 2]
    for rank, prefix_ok, fwd_err, bwd_err in res:
        assert prefix_ok, rank
        assert fwd_err < 1e-12, (rank, fwd_err)
        assert bwd_err < 1e-12, (rank, bwd_err)



def test_sub_span_folds_match_the_whole_span():
    """The sequence-parallel path cuts a rank's span into sub-spans; the
    folds that join them (qwendopamine_b200.gdn2_ops.cp) must reproduce the
    whole span: composed maps = the span's map, unfolded initial states = the
    recurrence's state at each cut, composed / unfolded gradients = the
    reverse pass's.  Float64 oracle maps on the CPU."""
    import sys

    sys.path.insert(0, ROOT)
    from oracle import gdn2_oracle as O
    from qwendopamine_b200.gdn2_ops import cp

    q, k, v, g, b, w, h0, do = _inputs()
    B, T, H, K = q.shape
    V = v.shape[-1]
    cuts = [0, 40, 64, T]  # three sub-spans
    args = (q, k, v, g, b, w)
    sub = [tuple(x[:, a:e] for x in args) for a, e in zip(cuts[:-1], cuts[1:])]
    maps = [O.span_transition(*s, norm_mode="torch") for s in sub]
    hm_sub = torch.from_numpy(np.stack([np.concatenate([he, M], -1) for M, he in maps], 1))
    M_all, he_all = O.span_transition(*args, norm_mode="torch")
    comp = cp._compose_maps(hm_sub.float()).double().numpy()
    assert np.abs(comp[..., :V] - he_all).max() < 1e-5
    assert np.abs(comp[..., V:] - M_all).max() < 1e-5
    # initial state of every sub-span
    states = cp._unfold_states(torch.from_numpy(h0).float(), hm_sub.float()).view(B, 3, H, K, V)
    for j, a in enumerate(cuts[:-1]):
        ref = h0 if a == 0 else O.recurrent_fwd(*(x[:, :a] for x in args), h0, norm_mode="torch")[1]
        assert np.abs(states[:, j].double().numpy() - ref).max() < 1e-5, j
    # gradients: each sub-span's start gradient from its own outputs (zero end
    # gradient), composed with a final-state gradient, vs the whole span's
    dht = np.random.default_rng(1).standard_normal((B, H, K, V))
    dhm = []
    for (a, e), s in zip(zip(cuts[:-1], cuts[1:]), sub):
        dhm.append(O.recurrent_bwd(*s, do[:, a:e], None, None, norm_mode="torch")[-1])
    dhm_sub = torch.from_numpy(np.stack(dhm, 1)).float()
    start = cp._compose_grads(dhm_sub, hm_sub.float(), torch.from_numpy(dht).float())
    ref_start = O.recurrent_bwd(*args, do, None, dht, norm_mode="torch")[-1]
    assert np.abs(start.double().numpy() - ref_start).max() < 1e-4
    ends = cp._unfold_grads(torch.from_numpy(dht).float(), dhm_sub, hm_sub.float())
    ends = ends.view(B, 3, H, K, V)
    for j, e in enumerate(cuts[1:]):
        ref_end = (dht if e == T else
                   O.recurrent_bwd(*(x[:, e:] for x in args), do[:, e:], None, dht,
                                   norm_mode="torch")[-1])
        assert np.abs(ends[:, j].double().numpy() - ref_end).max() < 1e-4, j

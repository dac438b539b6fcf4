"""Forward state pass on tcgen05 / TMEM / TMA (bf16, K = V = 128).

The chunkwise forward routes bf16 problems with K = V = 128 through
k_fwd_state_tc.  These cases check its outputs, final states and per-chunk
checkpoints against the float64 oracle (rel-L2 <= 2e-2, the bf16 tolerance),
on ragged and empty packed sequences and on a 64-chunk sequence that cycles
the two-slot copy ring many times, and check that no bounded wait ran out.
"""

import numpy as np
import pytest
import torch

from gdn2_testutil import TOL, make_inputs, np_, rel, to_dev
from oracle import gdn2_oracle as O

pytestmark = pytest.mark.gpu
NAMES = ("q", "k", "v", "g", "b", "w")
BF = torch.bfloat16


def _fault_word():
    from qwendopamine_b200 import _native as N

    return N.fault_status(clear=True)


def test_tc_state_varlen_ragged_and_empty(cuda_device):
    from qwendopamine_b200 import chunk_gdn2

    _fault_word()
    cu = [0, 1, 64, 129, 129, 300, 364, 500]
    N = len(cu) - 1
    H = 3
    d = make_inputs(1, cu[-1], H, 128, 128, seed=41, dtype=BF, h0=False)
    gen = torch.Generator().manual_seed(8)
    h0 = torch.randn(N, H, 128, 128, generator=gen) * 0.1
    x = to_dev(d, cuda_device, BF)
    o, ht = chunk_gdn2(x["q"], x["k"], x["v"], x["g"], x["b"], x["w"],
                       initial_state=h0.to(cuda_device), output_final_state=True,
                       use_qk_l2norm_in_kernel=True,
                       cu_seqlens=torch.tensor(cu, device=cuda_device))
    ro, rh = O.recurrent_fwd_varlen(*np_(d, NAMES), cu, h0.numpy(), norm_mode="fla")
    assert rel(o, ro) < TOL[BF]
    assert rel(ht, rh) < TOL[BF]
    # the empty sequence passes its initial state through unchanged
    assert torch.equal(ht[3].cpu(), h0[3])
    assert _fault_word() == 0


def test_tc_state_long_sequence_and_checkpoints(cuda_device):
    from qwendopamine_b200 import chunk_gdn2

    _fault_word()
    B, T, H = 1, 4096, 2
    d = make_inputs(B, T, H, 128, 128, seed=42, dtype=BF, decay="baseline")
    x = to_dev(d, cuda_device, BF)
    with torch.inference_mode():
        o, ht, h = chunk_gdn2(x["q"], x["k"], x["v"], x["g"], x["b"], x["w"],
                              initial_state=x["h0"], output_final_state=True,
                              use_qk_l2norm_in_kernel=True, return_intermediate_states=True)
    ro, rh = O.recurrent_fwd(*np_(d, NAMES), d["h0"].numpy(), norm_mode="fla")
    assert rel(o, ro) < TOL[BF]
    assert rel(ht, rh) < TOL[BF]
    # checkpoint j is the state entering chunk j: the recurrence's state after
    # 64*j tokens (j = 0: the initial state)
    hs = h.float().cpu().numpy()  # [B, NT, H, K, V]
    for j in (0, 1, 17, 63):
        if j == 0:
            ref = d["h0"].numpy()
        else:
            _, ref = O.recurrent_fwd(*(a[:, :64 * j] for a in np_(d, NAMES)),
                                     d["h0"].numpy(), norm_mode="fla")
        assert rel(hs[:, j], ref) < TOL[BF], j
    assert _fault_word() == 0


@pytest.mark.parametrize("B,T,H", [(8, 256, 16), (1, 65, 1), (20, 64, 9)])
def test_tc_state_batched_shapes(cuda_device, B, T, H):
    _fault_word()
    d = make_inputs(B, T, H, 128, 128, seed=B * 7 + T + H, dtype=BF)
    from qwendopamine_b200 import chunk_gdn2

    x = to_dev(d, cuda_device, BF)
    o, ht = chunk_gdn2(x["q"], x["k"], x["v"], x["g"], x["b"], x["w"], initial_state=x["h0"],
                       output_final_state=True, use_qk_l2norm_in_kernel=True)
    ro, rh = O.recurrent_fwd(*np_(d, NAMES), d["h0"].numpy(), norm_mode="fla")
    assert rel(o, ro) < TOL[BF]
    assert rel(ht, rh) < TOL[BF]
    assert _fault_word() == 0


def test_tc_state_backward_varlen_ragged_and_empty(cuda_device):
    """Backward state pass on tcgen05: packed sequences with partial last
    chunks (whose dO rows past the end belong to the next sequence), an empty
    and a single-token sequence; gradients per sequence against the oracle."""
    from qwendopamine_b200 import chunk_gdn2

    _fault_word()
    cu = [0, 1, 64, 129, 129, 300, 364, 500]
    N, H, K = len(cu) - 1, 2, 128
    d = make_inputs(1, cu[-1], H, K, K, seed=43, dtype=BF, h0=False)
    gen = torch.Generator().manual_seed(9)
    h0 = torch.randn(N, H, K, K, generator=gen) * 0.1
    do = torch.randn(1, cu[-1], H, K, generator=gen).bfloat16().float()
    dht = torch.randn(N, H, K, K, generator=gen)
    x = to_dev(d, cuda_device, BF)
    leaves = {n: x[n].clone().requires_grad_() for n in NAMES}
    h0d = h0.to(cuda_device).requires_grad_()
    o, ht = chunk_gdn2(*(leaves[n] for n in NAMES), initial_state=h0d, output_final_state=True,
                       use_qk_l2norm_in_kernel=True,
                       cu_seqlens=torch.tensor(cu, device=cuda_device))
    ((o.float() * do.to(cuda_device)).sum() + (ht * dht.to(cuda_device)).sum()).backward()
    for s in range(N):
        a_, e_ = cu[s], cu[s + 1]
        if e_ == a_:
            assert torch.equal(h0d.grad[s].cpu(), dht[s]), "empty sequence: dh0 = dht"
            continue
        sl = [t[:, a_:e_].double().numpy() for t in (d[n] for n in NAMES)]
        ref = O.recurrent_bwd(*sl, do[:, a_:e_].numpy(), h0[s:s + 1].numpy(),
                              dht[s:s + 1].numpy(), norm_mode="fla")
        for n, r in zip(NAMES, ref):
            assert rel(leaves[n].grad[:, a_:e_], r) < TOL[BF], (s, n)
        assert rel(h0d.grad[s:s + 1], ref[6]) < TOL[BF], (s, "h0")
    assert _fault_word() == 0


def test_tc_state_bounded_wait_runs_out_cleanly(cuda_device):
    """The device-side failure path, made to happen without a fault: the
    test hook runs the tcgen05 forward state pass with one chunk's tiles never
    requested and a 50 us limit on every wait.  The wait for that chunk runs
    out, the CTA drains its copies and products in flight, frees its tensor
    memory and sets bit 0 of the fault word; the launch itself succeeds.  The
    same context then runs a normal forward + backward that matches the
    oracle with a clean fault word."""
    from qwendopamine_b200 import _native as N
    from qwendopamine_b200 import chunk_gdn2

    lib = N.load()
    _fault_word()
    B, T, H = 1, 8 * 64, 2
    d = make_inputs(B, T, H, 128, 128, seed=43, dtype=BF, decay="baseline", h0=False)
    x = to_dev(d, cuda_device, BF)
    tables = N.seq_tables(B, T, cuda_device)
    prob = N.ChunkProblem(H, 128, 128, N.dtype_code(BF), 1, 128 ** -0.5, tables.struct())
    sb = lib.gdn2_chunk_saved_bytes(prob)
    saved = torch.empty(sb, dtype=torch.uint8, device=cuda_device)
    o = torch.zeros_like(x["v"])
    st = N.stream_of(cuda_device)
    N.check(lib.gdn2_chunk_fwd_intra(prob, *(N.ptr(x[n]) for n in NAMES), N.ptr(saved), sb, st),
            "gdn2_chunk_fwd_intra")
    rc = lib.gdn2_test_fwd_state_wait_timeout(prob, N.ptr(o), N.ptr(saved), sb, 3, 50_000, st)
    N.check(rc, "gdn2_test_fwd_state_wait_timeout")
    assert _fault_word() & 1 == 1
    # the context is intact: a normal pass on it is correct and raises no bit
    leaves = {n: x[n].clone().requires_grad_() for n in NAMES}
    o, _ = chunk_gdn2(*(leaves[n] for n in NAMES), use_qk_l2norm_in_kernel=True)
    do = torch.randn(B, T, H, 128, generator=torch.Generator().manual_seed(9)).bfloat16()
    o.backward(do.to(cuda_device))
    ro, _ = O.recurrent_fwd(*np_(d, NAMES), None, norm_mode="fla")
    assert rel(o, ro) < TOL[BF]
    ref = O.recurrent_bwd(*np_(d, NAMES), do.float().numpy(), None, None, norm_mode="fla")
    for n, r in zip(NAMES, ref):
        assert rel(leaves[n].grad, r) < TOL[BF], n
    assert _fault_word() == 0


def test_tc_state_wait_timeout_hook_argument_checks(cuda_device):
    from qwendopamine_b200 import _native as N

    lib = N.load()
    tables = N.seq_tables(1, 128, cuda_device)
    buf = torch.empty(1 << 20, dtype=torch.uint8, device=cuda_device)
    st = N.stream_of(cuda_device)
    # fp32 problems never take the tcgen05 pass
    p32 = N.ChunkProblem(1, 128, 128, N.dtype_code(torch.float32), 1, 0.1, tables.struct())
    big = torch.empty(lib.gdn2_chunk_saved_bytes(p32), dtype=torch.uint8, device=cuda_device)
    assert lib.gdn2_test_fwd_state_wait_timeout(p32, N.ptr(buf), N.ptr(big), big.numel(), 0,
                                                1000, st) == N.ERR_UNSUPPORTED
    pbf = N.ChunkProblem(1, 128, 128, N.dtype_code(BF), 1, 0.1, tables.struct())
    assert lib.gdn2_test_fwd_state_wait_timeout(pbf, N.ptr(buf), N.ptr(big), big.numel(), 0,
                                                0, st) == N.ERR_INVALID
    assert _fault_word() == 0

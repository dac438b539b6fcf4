"""Parity of the B200 recurrent (decode) kernel, through the C ABI, with the
reference's golden decode chain and the float64 oracle."""

import os

import numpy as np
import pytest
import torch

from gdn2_testutil import make_inputs, np_, rel, to_dev
from oracle import gdn2_oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
NAMES = ("q", "k", "v", "g", "b", "w")


def test_decode_chain_matches_reference_golden(cuda_device):
    """Config-2 recipe (bf16 inputs, fp32 N(0,0.02) state), three chained steps."""
    from qwendopamine_b200 import fused_recurrent_gdn2

    gd = np.load(os.path.join(GOLD, "decode.npz"))
    h = torch.from_numpy(gd["h0"]).to(cuda_device)
    for s in range(3):
        x = {n: torch.from_numpy(gd[f"{n}{s}"]).to(cuda_device) for n in NAMES}
        for n in ("q", "k", "v", "b", "w"):
            x[n] = x[n].bfloat16()
        o, h = fused_recurrent_gdn2(**x, initial_state=h, output_final_state=True,
                                    use_qk_l2norm_in_kernel=True)
        assert o.dtype == torch.bfloat16
        assert rel(o, gd[f"o{s}"]) < 2e-2
    assert rel(h, gd["ht"]) < 1e-4


@pytest.mark.parametrize("T,K,V", [(1, 128, 128), (37, 64, 64), (5, 16, 16), (20, 48, 80),
                                   (3, 100, 6)])
def test_multi_token_fp32(cuda_device, T, K, V):
    from qwendopamine_b200 import fused_recurrent_gdn2

    d = make_inputs(3, T, 2, K, V, seed=T * K)
    x = to_dev(d, cuda_device, torch.float32)
    o, ht = fused_recurrent_gdn2(*(x[n] for n in NAMES), initial_state=x["h0"],
                                 output_final_state=True, use_qk_l2norm_in_kernel=True)
    ro, rh = O.recurrent_fwd(*np_(d, NAMES), d["h0"].numpy(), norm_mode="fla")
    assert rel(o, ro) < 1e-4
    assert rel(ht, rh) < 1e-4


def test_inplace_state_pool_with_indices(cuda_device):
    from qwendopamine_b200 import fused_recurrent_gdn2_fwd

    d = make_inputs(4, 1, 2, 64, 64, seed=2, h0=False)
    gen = torch.Generator().manual_seed(7)
    pool = torch.randn(7, 2, 64, 64, generator=gen) * 0.05
    idx = torch.tensor([5, 0, -1, 3], dtype=torch.int32)
    x = to_dev(d, cuda_device, torch.float32)
    pool_d = pool.to(cuda_device)
    o, fs = fused_recurrent_gdn2_fwd(*(x[n] for n in NAMES), initial_state=pool_d,
                                     inplace_final_state=True,
                                     ssm_state_indices=idx.to(cuda_device),
                                     use_qk_l2norm_in_kernel=True)
    assert fs.data_ptr() == pool_d.data_ptr()
    for n, slot in enumerate(idx.tolist()):
        if slot < 0:
            continue
        sl = [a[n:n + 1] for a in np_(d, NAMES)]
        ro, rh = O.recurrent_fwd(*sl, pool[slot:slot + 1].numpy(), norm_mode="fla")
        assert rel(o[n:n + 1], ro) < 1e-4
        assert rel(pool_d[slot], rh[0]) < 1e-4
    untouched = [s for s in range(7) if s not in idx.tolist()]
    assert torch.equal(pool_d[untouched].cpu(), pool[untouched])


def test_inplace_dense_state(cuda_device):
    from qwendopamine_b200 import fused_recurrent_gdn2_fwd

    d = make_inputs(2, 4, 2, 32, 32, seed=4)
    x = to_dev(d, cuda_device, torch.float32)
    st = x["h0"].clone()
    fused_recurrent_gdn2_fwd(*(x[n] for n in NAMES), initial_state=st, inplace_final_state=True,
                             use_qk_l2norm_in_kernel=True)
    _, rh = O.recurrent_fwd(*np_(d, NAMES), d["h0"].numpy(), norm_mode="fla")
    assert rel(st, rh) < 1e-4


def test_varlen_decode(cuda_device):
    from qwendopamine_b200 import fused_recurrent_gdn2

    cu = [0, 3, 3, 10, 11]
    d = make_inputs(1, cu[-1], 2, 32, 32, seed=11, h0=False)
    h0 = torch.randn(4, 2, 32, 32, generator=torch.Generator().manual_seed(1)) * 0.1
    x = to_dev(d, cuda_device, torch.float32)
    o, ht = fused_recurrent_gdn2(*(x[n] for n in NAMES), initial_state=h0.to(cuda_device),
                                 output_final_state=True, use_qk_l2norm_in_kernel=True,
                                 cu_seqlens=torch.tensor(cu, device=cuda_device))
    ro, rh = O.recurrent_fwd_varlen(*np_(d, NAMES), cu, h0.numpy(), norm_mode="fla")
    assert rel(o, ro) < 1e-4
    assert rel(ht, rh) < 1e-4


def test_grouped_value_heads(cuda_device):
    """q, k with H heads shared by HV = 2H value heads (fused_recurrent_gdn2.py:155)."""
    from qwendopamine_b200 import fused_recurrent_gdn2

    B, T, H, HV, K, V = 2, 6, 2, 4, 32, 32
    d = make_inputs(B, T, HV, K, V, seed=17)
    qk_small = make_inputs(B, T, H, K, V, seed=18)
    d["q"], d["k"] = qk_small["q"], qk_small["k"]
    x = to_dev(d, cuda_device, torch.float32)
    o, ht = fused_recurrent_gdn2(*(x[n] for n in NAMES), initial_state=x["h0"],
                                 output_final_state=True, use_qk_l2norm_in_kernel=True)
    rep = {n: (d[n].repeat_interleave(HV // H, dim=2) if n in ("q", "k") else d[n])
           for n in NAMES}
    ro, rh = O.recurrent_fwd(*(rep[n].double().numpy() for n in NAMES), d["h0"].numpy(),
                             norm_mode="fla")
    assert rel(o, ro) < 1e-4
    assert rel(ht, rh) < 1e-4


def test_recurrent_and_chunk_agree(cuda_device):
    from qwendopamine_b200 import chunk_gdn2, fused_recurrent_gdn2

    d = make_inputs(2, 50, 2, 64, 64, seed=19)
    x = to_dev(d, cuda_device, torch.float32)
    o1, h1 = fused_recurrent_gdn2(*(x[n] for n in NAMES), initial_state=x["h0"],
                                  output_final_state=True, use_qk_l2norm_in_kernel=True)
    o2, h2 = chunk_gdn2(*(x[n] for n in NAMES), initial_state=x["h0"], output_final_state=True,
                        use_qk_l2norm_in_kernel=True)
    assert rel(o1, o2) < 1e-4 and rel(h1, h2) < 1e-4


def _fault_word():
    from qwendopamine_b200 import _native as N

    return N.fault_status(clear=True)


@pytest.mark.parametrize("K", [128, 64])
def test_stream_decode_many_units_bf16(cuda_device, K):
    """Full-state streaming kernel (K = V): 600 (sequence, head) units, more
    than one per SM, so the two-buffer copy ring cycles; bf16 tokens."""
    from qwendopamine_b200 import fused_recurrent_gdn2

    _fault_word()
    d = make_inputs(300, 1, 2, K, K, seed=K + 1, dtype=torch.bfloat16)
    x = to_dev(d, cuda_device, torch.bfloat16)
    o, ht = fused_recurrent_gdn2(*(x[n] for n in NAMES), initial_state=x["h0"],
                                 output_final_state=True, use_qk_l2norm_in_kernel=True)
    ro, rh = O.recurrent_fwd(*np_(d, NAMES), d["h0"].numpy(), norm_mode="fla")
    assert rel(o, ro) < 2e-2
    assert rel(ht, rh) < 1e-4
    assert _fault_word() == 0


def test_stream_state_pool_varlen_gva_no_h0(cuda_device):
    """Streaming kernel with a state pool (skipped slots, in place), packed
    sequences (one empty), grouped value heads, and a call without state."""
    from qwendopamine_b200 import fused_recurrent_gdn2, fused_recurrent_gdn2_fwd

    _fault_word()
    K = 128
    # pool + indices, in place
    d = make_inputs(5, 1, 2, K, K, seed=21, h0=False, dtype=torch.bfloat16)
    gen = torch.Generator().manual_seed(22)
    pool = torch.randn(9, 2, K, K, generator=gen) * 0.05
    idx = torch.tensor([7, -1, 0, 4, -1], dtype=torch.int32)
    x = to_dev(d, cuda_device, torch.bfloat16)
    pool_d = pool.to(cuda_device)
    o, _ = fused_recurrent_gdn2_fwd(*(x[n] for n in NAMES), initial_state=pool_d,
                                    inplace_final_state=True,
                                    ssm_state_indices=idx.to(cuda_device),
                                    use_qk_l2norm_in_kernel=True)
    for n, slot in enumerate(idx.tolist()):
        if slot < 0:
            continue
        sl = [a[n:n + 1] for a in np_(d, NAMES)]
        ro, rh = O.recurrent_fwd(*sl, pool[slot:slot + 1].numpy(), norm_mode="fla")
        assert rel(o[n:n + 1], ro) < 2e-2
        assert rel(pool_d[slot], rh[0]) < 1e-4
    untouched = [s for s in range(9) if s not in idx.tolist()]
    assert torch.equal(pool_d[untouched].cpu(), pool[untouched])
    # packed sequences with an empty one
    cu = [0, 2, 2, 7, 8]
    dv = make_inputs(1, cu[-1], 2, K, K, seed=23, h0=False)
    h0 = torch.randn(4, 2, K, K, generator=gen) * 0.1
    xv = to_dev(dv, cuda_device, torch.float32)
    o, ht = fused_recurrent_gdn2(*(xv[n] for n in NAMES), initial_state=h0.to(cuda_device),
                                 output_final_state=True, use_qk_l2norm_in_kernel=True,
                                 cu_seqlens=torch.tensor(cu, device=cuda_device))
    ro, rh = O.recurrent_fwd_varlen(*np_(dv, NAMES), cu, h0.numpy(), norm_mode="fla")
    assert rel(o, ro) < 1e-4 and rel(ht, rh) < 1e-4
    # grouped value heads (HV = 2H) and no initial state
    B, T, H, HV = 3, 4, 2, 4
    dg = make_inputs(B, T, HV, K, K, seed=24, h0=False)
    qk = make_inputs(B, T, H, K, K, seed=25)
    dg["q"], dg["k"] = qk["q"], qk["k"]
    xg = to_dev(dg, cuda_device, torch.float32)
    o, ht = fused_recurrent_gdn2(*(xg[n] for n in NAMES), initial_state=None,
                                 output_final_state=True, use_qk_l2norm_in_kernel=True)
    rep = {n: (dg[n].repeat_interleave(HV // H, dim=2) if n in ("q", "k") else dg[n])
           for n in NAMES}
    ro, rh = O.recurrent_fwd(*(rep[n].double().numpy() for n in NAMES), None, norm_mode="fla")
    assert rel(o, ro) < 1e-4 and rel(ht, rh) < 1e-4
    assert _fault_word() == 0


@pytest.mark.parametrize("K", [128, 32])
def test_speculative_decoding_slots(cuda_device, K):
    """2-D ssm_state_indices with num_accepted_tokens (reference
    fused_recurrent_gdn2.py:217-226, 311-324): sequence n starts from slot
    indices[n, accepted[n]-1] and the state after its token t lands in slot
    indices[n, t]; negative slots are skipped; other slots stay untouched."""
    from qwendopamine_b200 import fused_recurrent_gdn2_fwd

    _fault_word()
    cu = [0, 3, 4, 8]
    idx = torch.tensor([[2, 7, 5, -1], [9, -1, -1, -1], [0, 4, 11, 6]], dtype=torch.int32)
    acc = torch.tensor([2, 1, 3], dtype=torch.int32)
    H = 2
    d = make_inputs(1, cu[-1], H, K, K, seed=31 + K, h0=False)
    gen = torch.Generator().manual_seed(32)
    pool = torch.randn(12, H, K, K, generator=gen) * 0.05
    x = to_dev(d, cuda_device, torch.float32)
    pool_d = pool.to(cuda_device)
    o, fs = fused_recurrent_gdn2_fwd(*(x[n] for n in NAMES), initial_state=pool_d,
                                     inplace_final_state=True,
                                     cu_seqlens=torch.tensor(cu, device=cuda_device),
                                     ssm_state_indices=idx.to(cuda_device),
                                     num_accepted_tokens=acc.to(cuda_device),
                                     use_qk_l2norm_in_kernel=True)
    assert fs.data_ptr() == pool_d.data_ptr()
    expect = pool.clone()
    written = set()
    for n in range(3):
        a_, e_ = cu[n], cu[n + 1]
        sl = [t[:, a_:e_] for t in np_(d, NAMES)]
        s0 = pool[int(idx[n, acc[n] - 1])][None].numpy()
        ro, _, states = O.recurrent_fwd(*sl, s0, norm_mode="fla", return_states=True)
        assert rel(o[:, a_:e_], ro) < 1e-4, n
        for t in range(e_ - a_):
            slot = int(idx[n, t])
            if slot >= 0:
                expect[slot] = torch.from_numpy(states[t + 1][0]).float()
                written.add(slot)
    for slot in range(12):
        if slot in written:
            assert rel(pool_d[slot], expect[slot]) < 1e-4, slot
        else:
            assert torch.equal(pool_d[slot].cpu(), pool[slot]), slot
    assert _fault_word() == 0


@pytest.mark.parametrize("K", [128, 32])
@pytest.mark.parametrize("lower_bound", [None, -2.0])
def test_gate_in_kernel_decode(cuda_device, K, lower_bound):
    """Gate fused in the decode kernels (fused_recurrent_gdn2.py:257-272):
    -exp(A_log[h]) softplus(g + dt_bias[h]) or lower_bound sigmoid(exp(A_log[h])
    (g + dt_bias[h])), h the key head of each value head (grouped heads here)."""
    from qwendopamine_b200 import fused_recurrent_gdn2

    _fault_word()
    B, T, H, HV = 3, 2, 2, 4
    d = make_inputs(B, T, HV, K, K, seed=41 + K)
    qk = make_inputs(B, T, H, K, K, seed=42 + K)
    d["q"], d["k"] = qk["q"], qk["k"]
    gen = torch.Generator().manual_seed(43)
    raw = torch.randn(B, T, HV, K, generator=gen) * 2
    A_log = torch.rand(H, generator=gen) * 2 - 1
    dt_bias = torch.randn(H * K, generator=gen)
    x = to_dev(d, cuda_device, torch.float32)
    o, ht = fused_recurrent_gdn2(x["q"], x["k"], x["v"], raw.to(cuda_device), x["b"], x["w"],
                                 A_log=A_log.to(cuda_device), dt_bias=dt_bias.to(cuda_device),
                                 initial_state=x["h0"], output_final_state=True,
                                 use_qk_l2norm_in_kernel=True, use_gate_in_kernel=True,
                                 lower_bound=lower_bound)
    hk = torch.arange(HV) // (HV // H)  # key head of each value head
    xx = raw.double() + dt_bias.double().view(H, K)[hk]
    a = A_log.double().exp()[hk].view(HV, 1)
    if lower_bound is None:
        geff = -a * torch.nn.functional.softplus(xx)
    else:
        geff = lower_bound * torch.sigmoid(a * xx)
    rep = {n: (d[n].repeat_interleave(HV // H, dim=2) if n in ("q", "k") else d[n])
           for n in NAMES}
    rep["g"] = geff
    ro, rh = O.recurrent_fwd(*(rep[n].double().numpy() for n in NAMES), d["h0"].numpy(),
                             norm_mode="fla")
    assert rel(o, ro) < 1e-4
    assert rel(ht, rh) < 1e-4
    assert _fault_word() == 0

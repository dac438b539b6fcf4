"""Head sizes above 128 (K, V <= 256, as the reference's chunk_gdn2 accepts,
chunk_gdn2.py:1380-1382; V = 2 * head_dim under expand_v = 2, gdn2.py:568-571).

The chunkwise forward / backward take the slab-walking kernels of
chunk_wide.cu, decode takes the 256-row recurrent kernel; every result is
checked against the float64 oracle: rel-L2 <= 1e-4 for fp32, <= 2e-2 for
bf16 -- outputs, final states, all six input gradients and dh0.
"""

import pytest
import torch

from gdn2_testutil import TOL, make_inputs, np_, rel, to_dev
from oracle import gdn2_oracle as O

pytestmark = pytest.mark.gpu
NAMES = ("q", "k", "v", "g", "b", "w")
SHAPES = [(256, 256), (128, 256), (256, 128), (200, 136)]


def _fwd_bwd(d, dev, dtype, do, dht, **kw):
    from qwendopamine_b200 import chunk_gdn2

    x = to_dev(d, dev, dtype)
    leaves = {n: x[n].clone().requires_grad_() for n in NAMES}
    h0 = x["h0"].clone().requires_grad_() if x["h0"] is not None else None
    o, ht = chunk_gdn2(*(leaves[n] for n in NAMES), initial_state=h0, output_final_state=True,
                       use_qk_l2norm_in_kernel=True, **kw)
    ((o.float() * do.to(dev)).sum() + (ht * dht.to(dev)).sum()).backward()
    g = {n: leaves[n].grad for n in NAMES}
    g["h0"] = h0.grad if h0 is not None else None
    return o, ht, g


@pytest.mark.parametrize("KV", SHAPES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_wide_heads_forward_backward(cuda_device, KV, dtype):
    K, V = KV
    B, T, H = 2, 150, 2   # a partial last chunk
    d = make_inputs(B, T, H, K, V, seed=K + V, dtype=dtype)
    gen = torch.Generator().manual_seed(K * V)
    do = torch.randn(B, T, H, V, generator=gen).to(dtype).float()
    dht = torch.randn(B, H, K, V, generator=gen)
    o, ht, g = _fwd_bwd(d, cuda_device, dtype, do, dht)
    ro, rh = O.recurrent_fwd(*np_(d, NAMES), d["h0"].numpy(), norm_mode="fla")
    tol = TOL[dtype]
    assert rel(o, ro) < tol and rel(ht, rh) < tol
    ref = O.recurrent_bwd(*np_(d, NAMES), do.numpy(), d["h0"].numpy(), dht.numpy(),
                          norm_mode="fla")
    for n, r in zip((*NAMES, "h0"), ref):
        assert rel(g[n], r) < tol, n


def test_wide_heads_varlen_strong_decay_fp32(cuda_device):
    """Packed sequences (an empty one, a one-token one) and decays strong
    enough that the score blocks' exact forms matter."""
    cu = [0, 70, 70, 71, 200]
    K, V = 256, 192
    d = make_inputs(1, cu[-1], 2, K, V, seed=5, decay=-3.0, h0=False)
    gen = torch.Generator().manual_seed(6)
    h0 = torch.randn(4, 2, K, V, generator=gen) * 0.1
    do = torch.randn(1, cu[-1], 2, V, generator=gen)
    d["h0"] = h0
    o, ht, g = _fwd_bwd(d, cuda_device, torch.float32, do, torch.zeros(4, 2, K, V),
                        cu_seqlens=torch.tensor(cu, device=cuda_device))
    for s in range(4):
        a, e = cu[s], cu[s + 1]
        sl = [d[n][:, a:e].double().numpy() for n in NAMES]
        ro, rh = O.recurrent_fwd(*sl, h0[s:s + 1].numpy(), norm_mode="fla")
        assert rel(ht[s:s + 1], rh) < 1e-4, s
        if e > a:
            assert rel(o[:, a:e], ro) < 1e-4, s
            ref = O.recurrent_bwd(*sl, do[:, a:e].numpy(), h0[s:s + 1].numpy(), None,
                                  norm_mode="fla")
            for n, r in zip(NAMES, ref):
                assert rel(g[n][:, a:e], r) < 1e-4, (s, n)
            assert rel(g["h0"][s:s + 1], ref[6]) < 1e-4, s


@pytest.mark.parametrize("KV", [(256, 256), (128, 256)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_wide_heads_decode(cuda_device, KV, dtype):
    from qwendopamine_b200 import fused_recurrent_gdn2

    K, V = KV
    d = make_inputs(3, 4, 2, K, V, seed=K * 3 + V, dtype=dtype)
    x = to_dev(d, cuda_device, dtype)
    o, ht = fused_recurrent_gdn2(*(x[n] for n in NAMES), initial_state=x["h0"],
                                 output_final_state=True, use_qk_l2norm_in_kernel=True)
    ro, rh = O.recurrent_fwd(*np_(d, NAMES), d["h0"].numpy(), norm_mode="fla")
    assert rel(o, ro) < TOL[dtype] and rel(ht, rh) < 1e-4


def test_wide_heads_prescan_matches_span_map(cuda_device):
    """The context-parallel pre-scan ([h_e | M] over V + K columns) at K = V =
    256 against the oracle's span transition."""
    from qwendopamine_b200 import _native as N

    lib = N.load()
    K = V = 256
    d = make_inputs(1, 130, 2, K, V, seed=9, h0=False)
    x = to_dev(d, cuda_device, torch.float32)
    tab = N.seq_tables(1, 130, cuda_device)
    prob = N.ChunkProblem(2, K, V, N.dtype_code(torch.float32), 1, K ** -0.5, tab.struct())
    sb = lib.gdn2_chunk_saved_bytes(prob)
    saved = torch.empty(sb, dtype=torch.uint8, device=cuda_device)
    st = N.stream_of(cuda_device)
    N.check(lib.gdn2_chunk_fwd_intra(prob, *(N.ptr(x[n]) for n in NAMES), N.ptr(saved), sb, st),
            "intra")
    hm = torch.empty(1, 2, K, V + K, device=cuda_device)
    N.check(lib.gdn2_cp_fwd_prescan(prob, N.ptr(saved), sb, N.ptr(hm), None, 0, st), "prescan")
    M, he = O.span_transition(*np_(d, NAMES), norm_mode="fla")
    assert rel(hm[..., :V], he) < 1e-4
    assert rel(hm[..., V:], M) < 1e-4


def test_module_expand_v2_head_dim_128(cuda_device, monkeypatch):
    """The module with expand_v = 2 and head_dim = 128 (V = 256): forward and
    backward run, and its core call matches the oracle on the exact tensors
    the module feeds it (the gate is formed by torch ops at this size)."""
    import qwendopamine_b200.gdn2 as M
    from qwendopamine_b200 import GatedDeltaNet2

    seen = {}
    real = M.chunk_gdn2

    def spy(**kw):
        out = real(**kw)
        seen.update(kw)
        seen["o"] = out[0]
        return out

    monkeypatch.setattr(M, "chunk_gdn2", spy)
    torch.manual_seed(0)
    layer = GatedDeltaNet2(hidden_size=256, num_heads=2, head_dim=128, expand_v=2.0).to(
        cuda_device).train()
    assert layer.head_v_dim == 256
    x = torch.randn(2, 100, 256, device=cuda_device, requires_grad=True)
    out, _, _ = layer(x)
    out.square().mean().backward()
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in layer.parameters())
    g = seen["g"].detach().double()
    H, K = g.shape[-2:]
    xg = g + seen["dt_bias"].detach().double().view(H, K)
    logdecay = (-seen["A_log"].detach().double().exp().view(H, 1) *
                torch.nn.functional.softplus(xg)).cpu().numpy()
    args = [seen[n].detach().double().cpu().numpy() for n in ("q", "k", "v", "g", "b", "w")]
    args[3] = logdecay
    ro, _ = O.recurrent_fwd(*args, norm_mode="fla")
    assert rel(seen["o"], ro) < 1e-4

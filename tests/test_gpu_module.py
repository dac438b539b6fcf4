"""The drop-in ``GatedDeltaNet2`` module on the GPU: its core calls run the
B200 kernels and agree with the oracle on the exact tensors the module feeds
them; decode with a cache continues a prefill exactly; padding is masked."""

import pytest
import torch

from gdn2_testutil import rel
from oracle import gdn2_oracle as O

pytestmark = pytest.mark.gpu


def _layer(dev, dtype=torch.float32, **kw):
    from qwendopamine_b200 import GatedDeltaNet2

    torch.manual_seed(0)
    kw.setdefault("hidden_size", 256)
    kw.setdefault("num_heads", 2)
    kw.setdefault("head_dim", 64)
    return GatedDeltaNet2(**kw).to(device=dev, dtype=dtype)


def _log_decay(kw):
    """The log-decay the core applies: the module hands the kernels the raw
    gate projection with use_gate_in_kernel (fp32 decays), so form
    -exp(A_log) * softplus(g + dt_bias) here (float64), and its derivative."""
    g = kw["g"].detach().double()
    if not kw.get("use_gate_in_kernel"):
        return g.cpu().numpy(), None
    H, K = g.shape[-2:]
    x = g + kw["dt_bias"].detach().double().view(H, K)
    a = kw["A_log"].detach().double().exp().view(H, 1)
    return (-a * torch.nn.functional.softplus(x)).cpu().numpy(), (-a * torch.sigmoid(x)).cpu().numpy()


def test_module_core_matches_oracle_on_its_own_inputs(cuda_device, monkeypatch):
    import qwendopamine_b200.gdn2 as M

    seen = {}
    real = M.chunk_gdn2

    def spy(**kw):
        out = real(**kw)
        seen.update(kw)
        seen["o"], seen["ht"] = out
        return out

    monkeypatch.setattr(M, "chunk_gdn2", spy)
    layer = _layer(cuda_device).train()
    x = torch.randn(2, 100, 256, device=cuda_device)
    out, attn, _ = layer(x)
    assert out.shape == (2, 100, 256) and attn is None
    args = [seen[n].detach().double().cpu().numpy() for n in ("q", "k", "v", "g", "b", "w")]
    args[3] = _log_decay(seen)[0]
    ro, _ = O.recurrent_fwd(*args, norm_mode="fla")
    assert rel(seen["o"], ro) < 1e-4


def test_module_backward_reaches_every_parameter(cuda_device):
    layer = _layer(cuda_device, torch.bfloat16).train()
    x = torch.randn(2, 70, 256, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    out, _, _ = layer(x)
    out.float().sum().backward()
    assert x.grad is not None and torch.isfinite(x.grad.float()).all()
    for name, p in layer.named_parameters():
        assert p.grad is not None, name
        assert torch.isfinite(p.grad.float()).all(), name


def test_module_gradients_match_oracle_core(cuda_device, monkeypatch):
    """Gradients of the core inputs inside the module equal the oracle's."""
    import qwendopamine_b200.gdn2 as M

    grabbed = {}
    real = M.chunk_gdn2

    def spy(**kw):
        for n in ("q", "k", "v", "g", "b", "w"):
            kw[n].retain_grad()
            grabbed[n] = kw[n]
        grabbed["kw"] = kw
        o, ht = real(**kw)
        o.retain_grad()
        grabbed["o"] = o
        return o, ht

    monkeypatch.setattr(M, "chunk_gdn2", spy)
    layer = _layer(cuda_device).train()
    x = torch.randn(1, 90, 256, device=cuda_device)
    out, _, _ = layer(x)
    (out * torch.randn_like(out)).sum().backward()
    args = [grabbed[n].detach().double().cpu().numpy() for n in ("q", "k", "v", "g", "b", "w")]
    args[3], dgate = _log_decay(grabbed["kw"])
    ref = list(O.recurrent_bwd(*args, grabbed["o"].grad.double().cpu().numpy(), norm_mode="fla"))
    if dgate is not None:  # chain rule through the gate to the raw projection
        ref[3] = ref[3] * dgate
    for n, r in zip(("q", "k", "v", "g", "b", "w"), ref):
        assert rel(grabbed[n].grad, r) < 1e-4, n


def test_prefill_then_decode_matches_full_sequence(cuda_device):
    layer = _layer(cuda_device).eval()
    x = torch.randn(2, 40, 256, device=cuda_device)
    with torch.no_grad():
        full, _, _ = layer(x)
        cache = {}
        pre, _, _ = layer(x[:, :30], past_key_values=cache, use_cache=True)
        steps = [layer(x[:, t:t + 1], past_key_values=cache, use_cache=True)[0]
                 for t in range(30, 40)]
    inc = torch.cat([pre, *steps], dim=1)
    assert rel(inc, full) < 1e-4
    assert cache["recurrent_state"].dtype == torch.float32
    assert cache["recurrent_state"].shape == (2, 2, 64, 64)


def test_chunk_mode_equals_recurrent_mode(cuda_device):
    layer = _layer(cuda_device)
    x = torch.randn(2, 64, 256, device=cuda_device)
    with torch.no_grad():
        layer.train()
        a, _, _ = layer(x)  # chunk kernels
        layer.eval()
        b, _, _ = layer(x)  # seq_len <= 64 in eval -> recurrent kernel
    assert rel(a, b) < 1e-4


def test_padding_tokens_are_zeroed(cuda_device):
    layer = _layer(cuda_device).train()
    x = torch.randn(2, 6, 256, device=cuda_device)
    mask = torch.tensor([[1, 1, 1, 1, 1, 1], [1, 1, 1, 0, 0, 0]], device=cuda_device)
    out, _, _ = layer(x, attention_mask=mask)
    assert torch.all(out[1, 3:] == 0)
    # The packed layout puts sequence 0 first, so its tokens see exactly what
    # they would alone.  (Sequence 1 does not: like the reference, the short
    # convolution ignores cu_seqlens and reads sequence 0's last tokens; the
    # recurrence itself restarts at every sequence boundary.)
    ref, _, _ = layer(x[:1])
    assert rel(out[0], ref[0]) < 1e-4
    unmasked, _, _ = layer(x)
    assert not torch.allclose(out, unmasked)


def test_bf16_forward_is_finite(cuda_device):
    layer = _layer(cuda_device, torch.bfloat16).train()
    x = torch.randn(2, 8, 256, device=cuda_device, dtype=torch.bfloat16)
    out, _, _ = layer(x)
    assert out.dtype == torch.bfloat16 and torch.isfinite(out.float()).all()


def test_dynamic_cache_decode(cuda_device):
    from transformers.cache_utils import DynamicCache

    layer = _layer(cuda_device, layer_idx=0).eval()
    x = torch.randn(1, 1, 256, device=cuda_device)
    with torch.no_grad():
        out, _, cache = layer(x, past_key_values=DynamicCache(), use_cache=True)
    assert out.shape == (1, 1, 256) and cache is not None

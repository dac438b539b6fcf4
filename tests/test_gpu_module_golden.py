"""The whole drop-in module against the reference module's own outputs.

tests/golden/module.npz holds, for three seeded cases, what the reference's
``GatedDeltaNet2`` (gdn2.py:488-1004, fp32, exact token-serial core) produced:
its initial state_dict, the training-mode output with the returned cache
(recurrent state and the three conv states), the gradients of
sum(out * dy) for every parameter, and one eval-mode decode step through
that cache.  The B200 module is loaded with that state_dict and must agree
within the fp32 contract (rel-L2 <= 1e-4) everywhere: the gate formation in
the kernel, grouped value heads (GVA), ``allow_neg_eigval``, ``expand_v``,
the conv bias, the gated RMSNorm with g_proj, o_proj and the unpad / repad
of a padding mask are all inside the comparison.
"""

import numpy as np
import pytest
import torch

from gdn2_testutil import rel
from module_cases import GOLDEN, MODULE_CASES

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _load(name, dev):
    from qwendopamine_b200 import GatedDeltaNet2

    g = np.load(GOLDEN)
    kw = MODULE_CASES[name][0]
    m = GatedDeltaNet2(layer_idx=0, **kw)
    sd = {n[len(name) + 4:]: torch.from_numpy(g[n]) for n in g.files
          if n.startswith(f"{name}.sd.")}
    m.load_state_dict(sd, strict=True)
    return m.to(dev), g


@pytest.mark.parametrize("name", sorted(MODULE_CASES))
def test_module_matches_reference_module(cuda_device, name):
    m, g = _load(name, cuda_device)
    pad = MODULE_CASES[name][4]
    f = lambda key: torch.from_numpy(g[f"{name}.{key}"]).to(cuda_device)
    x, dy = f("x"), f("dy")
    m.train()
    if pad:
        mask = torch.from_numpy(g[f"{name}.mask"]).to(cuda_device)
        y, _, _ = m(x, attention_mask=mask)
    else:
        cache = {}
        y, _, cache = m(x, past_key_values=cache, use_cache=True)
        assert rel(cache["recurrent_state"], g[f"{name}.rec"]) <= TOL, "recurrent_state"
        for tag, c in zip("qkv", cache["conv_state"]):
            assert rel(c, g[f"{name}.conv_{tag}"]) <= TOL, f"conv_state {tag}"
    assert rel(y, g[f"{name}.out"]) <= TOL, "out"
    if pad:  # padded rows are exact zeros, as the reference's repad leaves them
        assert torch.count_nonzero(y[0, :pad]) == 0
    params = dict(m.named_parameters())
    grads = torch.autograd.grad((y * dy).sum(), list(params.values()))
    for n, gr in zip(params, grads):
        assert rel(gr, g[f"{name}.grad.{n}"]) <= TOL, f"grad {n}"
    if not pad:
        m.eval()
        with torch.no_grad():
            y1, _, cache = m(f("x1"), past_key_values=cache, use_cache=True)
        assert rel(y1, g[f"{name}.out1"]) <= TOL, "decode out"
        assert rel(cache["recurrent_state"], g[f"{name}.rec1"]) <= TOL, "decode state"
        for tag, c in zip("qkv", cache["conv_state"]):
            assert rel(c, g[f"{name}.conv1_{tag}"]) <= TOL, f"decode conv_state {tag}"

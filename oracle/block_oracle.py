"""CPU oracle for the GDN-2 block prologue / epilogue -- TEST INFRASTRUCTURE ONLY.

Only ``tests/`` and ``bench.py``'s CPU legs may import this module; the
product path (``qwendopamine_b200``) never calls it.

It restates, in numpy, two pure-PyTorch pieces of the reference's
``src/qwendopamine/models/gdn2/gdn2.py``:

* :func:`conv_fwd` / :func:`conv_bwd` -- ``ShortConvolution.forward``
  (gdn2.py:396-430): causal depthwise ``F.conv1d`` with ``padding = W - 1``
  truncated to the first T outputs, or, for one token with a cache, the cache
  prepended; then SiLU.  The backward is derived by hand (the reference gets
  it from autograd).  ``prefix`` generalises the cache: the W - 1 rows that
  precede x (zero when absent).
* :func:`gated_norm_fwd` / :func:`gated_norm_bwd` -- ``RMSNormGated.forward``
  (gdn2.py:446-452) in float64, and :func:`gated_norm_fwd_rounded`, the same
  steps with every intermediate rounded to bfloat16 as the reference computes
  them for bf16 inputs (it runs in the input dtype, not fp32).

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own
``ShortConvolution`` and ``RMSNormGated`` on seeded inputs (fp32 with autograd,
and bf16 forward) and stores them in ``tests/golden/block_ops.npz``;
``tests/test_block_oracle.py`` checks these functions against that fixture.
"""

from __future__ import annotations

import numpy as np


def _sig(x):
    return 1.0 / (1.0 + np.exp(-x))


def _cat_prefix(x, W, prefix):
    B, T, D = x.shape
    pad = np.zeros((B, W - 1, D)) if prefix is None else np.asarray(prefix, np.float64)
    return np.concatenate([pad, x], axis=1)


def conv_fwd(x, weight, bias=None, prefix=None, activation="silu"):
    """y[b, t, d] = act(bias[d] + sum_j weight[d, j] * xc[b, t + j, d]) with
    xc = [prefix; x] (W - 1 zero rows without a prefix).  x [B, T, D],
    weight [D, W] (or the conv1d shape [D, 1, W])."""
    x = np.asarray(x, np.float64)
    w = np.asarray(weight, np.float64).reshape(x.shape[-1], -1)
    W = w.shape[1]
    T = x.shape[1]
    xc = _cat_prefix(x, W, prefix)
    c = sum(w[:, j] * xc[:, j:j + T, :] for j in range(W))
    if bias is not None:
        c = c + np.asarray(bias, np.float64)
    return c * _sig(c) if activation == "silu" else c


def conv_bwd(x, weight, dy, bias=None, prefix=None, activation="silu"):
    """Returns (dx, dweight [D, W], dbias [D], dprefix [B, W-1, D])."""
    x = np.asarray(x, np.float64)
    dy = np.asarray(dy, np.float64)
    w = np.asarray(weight, np.float64).reshape(x.shape[-1], -1)
    W = w.shape[1]
    T = x.shape[1]
    xc = _cat_prefix(x, W, prefix)
    c = sum(w[:, j] * xc[:, j:j + T, :] for j in range(W))
    if bias is not None:
        c = c + np.asarray(bias, np.float64)
    if activation == "silu":
        s = _sig(c)
        dc = dy * s * (1.0 + c * (1.0 - s))
    else:
        dc = dy
    dxc = np.zeros_like(xc)
    dw = np.zeros_like(w)
    for j in range(W):
        dxc[:, j:j + T, :] += w[:, j] * dc
        dw[:, j] = (dc * xc[:, j:j + T, :]).sum(axis=(0, 1))
    return dxc[:, W - 1:], dw, dc.sum(axis=(0, 1)), dxc[:, :W - 1]


def gated_norm_fwd(x, z, weight, eps=1e-5):
    x = np.asarray(x, np.float64)
    z = np.asarray(z, np.float64)
    r = 1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    return x * r * np.asarray(weight, np.float64) * (z * _sig(z))


def gated_norm_bwd(x, z, weight, dy, eps=1e-5):
    """Returns (dx, dz, dweight)."""
    x = np.asarray(x, np.float64)
    z = np.asarray(z, np.float64)
    dy = np.asarray(dy, np.float64)
    w = np.asarray(weight, np.float64)
    r = 1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    n = x * r
    sg = _sig(z)
    s = z * sg
    dn = dy * w * s
    dx = r * (dn - n * (dn * n).mean(-1, keepdims=True))
    dz = dy * n * w * sg * (1.0 + z * (1.0 - sg))
    dw = (dy * n * s).reshape(-1, x.shape[-1]).sum(0)
    return dx, dz, dw


def bf16_round(a):
    """Round float32 values to the nearest bfloat16 (ties to even), as float32."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def gated_norm_fwd_rounded(x, z, weight, eps=1e-5, weight_fp32=False):
    """The reference's bf16 evaluation order (gdn2.py:449-452): x.pow(2),
    .mean(-1), + eps, rsqrt, x * r, * weight, silu(z), the product -- each
    step computed in float32 and rounded once to bfloat16, as torch's CUDA
    kernels do (the product with an fp32 weight stays float32, and so does
    the result).  torch's CPU bfloat16 rsqrt is not this: on its scalar tail
    path it rounds the square root and then the reciprocal, so a CPU run of
    the reference can differ in r by one bfloat16 step."""
    R = bf16_round
    x = R(np.asarray(x, np.float32))
    z = R(np.asarray(z, np.float32))
    w = np.asarray(weight, np.float32)
    w = w if weight_fp32 else R(w)
    var = R((R(x * x).astype(np.float32).sum(-1, keepdims=True, dtype=np.float32)
             * np.float32(1.0 / x.shape[-1])).astype(np.float32))
    ve = R(var + np.float32(eps)).astype(np.float64)
    r = R((1.0 / np.sqrt(ve)).astype(np.float32))
    n = R(x * r)
    n = n * w if weight_fp32 else R(n * w)
    s = R((z / (np.float32(1.0) + np.exp(-z))).astype(np.float32))
    y = (n * s).astype(np.float32)
    return y if weight_fp32 else R(y)

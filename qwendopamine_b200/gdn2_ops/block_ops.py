"""Prologue and epilogue of the GDN-2 block on B200.

* :func:`short_conv` -- causal depthwise convolution + SiLU of the q / k / v
  projections (the reference's ``ShortConvolution``, gdn2.py:372-430), with an
  optional prefix of the ``W - 1`` preceding tokens (a decode cache, or the
  previous span's last tokens under sequence parallelism) and the decode-cache
  update.
* :func:`gated_rms_norm` -- SiLU-gated RMSNorm (``RMSNormGated``,
  gdn2.py:433-452), evaluated in the input dtype as the reference does, or in
  fp32 where the reference runs under ``torch.autocast``.

Both run ``libgdn2_b200.so`` kernels through the C ABI
(``gdn2_conv_fwd`` / ``gdn2_conv_bwd``, ``gdn2_gated_norm_fwd`` /
``gdn2_gated_norm_bwd``); there is no PyTorch fallback.
"""

from __future__ import annotations

import torch

from .. import _native as N

__all__ = ["ShortConvFunction", "GatedRMSNormFunction", "short_conv", "gated_rms_norm"]


def _dense16(t):
    """Contiguous and starting on a 16-byte boundary (the kernels move rows
    with vector loads)."""
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("GDN-2 block kernels need CUDA tensors -- the B200 build has no "
                               "CPU path")


def _conv_problem(x, W, activation, prefix):
    B, T, D = x.shape
    p = N.ConvProblem(B, T, D, W, N.dtype_code(x.dtype), activation)
    if prefix is not None:
        p.prefix_sb, p.prefix_sw, p.prefix_sd = prefix.stride()
    return p


class ShortConvFunction(torch.autograd.Function):
    """y = act(conv(x)) with a [B, W-1, D] prefix (any strides) or zero padding.

    ``weight`` is the ``nn.Conv1d`` weight ``[D, 1, W]`` and ``bias`` ``[D]``
    or None; both enter the kernel rounded to ``x``'s dtype, as ``F.conv1d``
    sees them.  Returns ``y`` and, when ``want_state``, the last ``W - 1`` rows
    of ``[prefix; x]`` as ``[B, D, W-1]`` (the reference's cache layout).
    """

    @staticmethod
    def forward(ctx, x, weight, bias, prefix, activation, want_state):
        _require_cuda(x, weight, bias, prefix)
        lib = N.load()
        x = _dense16(x)
        D, W = weight.shape[0], weight.shape[-1]
        w32 = weight.detach().reshape(D, W).to(x.dtype).float().contiguous()
        b32 = bias.detach().to(x.dtype).float().contiguous() if bias is not None else None
        if prefix is not None:
            prefix = prefix.to(x.dtype)
        prob = _conv_problem(x, W, activation, prefix)
        y = torch.empty_like(x)
        state = (x.new_empty(x.shape[0], D, W - 1) if want_state and W > 1 else None)
        st = N.stream_of(x.device)
        N.check(lib.gdn2_conv_fwd(prob, N.ptr(x), N.ptr(w32), N.ptr(b32), N.ptr(prefix), N.ptr(y),
                                  N.ptr(state), st), "gdn2_conv_fwd")
        ctx.save_for_backward(x, w32, b32, prefix)
        ctx.meta = (activation, weight.dtype, weight.shape, bias is not None,
                    bias.dtype if bias is not None else None)
        if state is not None:
            ctx.mark_non_differentiable(state)
        return y, state

    @staticmethod
    def backward(ctx, dy, dstate):
        x, w32, b32, prefix = ctx.saved_tensors
        activation, wdt, wshape, has_bias, bdt = ctx.meta
        lib = N.load()
        dy = _dense16(dy.to(x.dtype))
        D, W = w32.shape
        prob = _conv_problem(x, W, activation, prefix)
        ws = torch.empty(max(lib.gdn2_conv_bwd_workspace_bytes(prob), 1), dtype=torch.uint8,
                         device=x.device)
        dx = torch.empty_like(x)
        dw = torch.empty(D, W, dtype=torch.float32, device=x.device)
        db = torch.empty(D, dtype=torch.float32, device=x.device) if has_bias else None
        dpre = None
        if prefix is not None and ctx.needs_input_grad[3]:
            dpre = torch.empty(x.shape[0], W - 1, D, dtype=torch.float32, device=x.device)
        st = N.stream_of(x.device)
        N.check(lib.gdn2_conv_bwd(prob, N.ptr(x), N.ptr(w32), N.ptr(b32), N.ptr(prefix), N.ptr(dy),
                                  N.ptr(dx), N.ptr(dw), N.ptr(db), N.ptr(dpre), N.ptr(ws),
                                  ws.numel(), st), "gdn2_conv_bwd")
        # the reference's weight gradient is produced in the token dtype
        dw = dw.to(x.dtype).to(wdt).view(wshape)
        if db is not None:
            db = db.to(x.dtype).to(bdt)
        if dpre is not None:
            dpre = dpre.to(prefix.dtype)
        return dx, dw, db, dpre, None, None


def short_conv(x, weight, bias=None, activation="silu", prefix=None, output_final_state=False):
    """Causal depthwise convolution of ``x`` [B, T, D] (+ SiLU when
    ``activation == "silu"``).  Returns ``(y, new_state)``; ``new_state`` is
    the ``[B, D, W-1]`` cache after the last token when ``output_final_state``."""
    act = 1 if activation == "silu" else 0
    y, state = ShortConvFunction.apply(x, weight, bias, prefix, act, bool(output_final_state))
    return y, state


def _norm_problem(x, weight_dtype, eps, fp32_math):
    n = x.shape[-1]
    return N.NormProblem(x.numel() // n if n else 0, n, N.dtype_code(x.dtype),
                         N.dtype_code(weight_dtype), float(eps), int(fp32_math))


class GatedRMSNormFunction(torch.autograd.Function):
    """y = x * rsqrt(mean(x^2) + eps) * weight * silu(z) over the last dim."""

    @staticmethod
    def forward(ctx, x, z, weight, eps, fp32_math):
        _require_cuda(x, z, weight)
        lib = N.load()
        if z.dtype != x.dtype:
            raise NotImplementedError(
                f"gated_rms_norm: x ({x.dtype}) and z ({z.dtype}) must share a dtype")
        x, z = _dense16(x), _dense16(z)
        # a weight in another dtype enters as fp32 (exact); the result type
        # is then fp32, as torch's promotion makes it
        w = weight.detach()
        if fp32_math or w.dtype != x.dtype:
            w = w.float()
        w = _dense16(w)
        prob = _norm_problem(x, w.dtype, eps, fp32_math)
        out_dtype = torch.float32 if fp32_math else torch.promote_types(x.dtype, weight.dtype)
        y = torch.empty(x.shape, dtype=out_dtype, device=x.device)
        N.check(lib.gdn2_gated_norm_fwd(prob, N.ptr(x), N.ptr(z), N.ptr(w), N.ptr(y),
                                        N.stream_of(x.device)), "gdn2_gated_norm_fwd")
        ctx.save_for_backward(x, z, w)
        ctx.meta = (eps, fp32_math, weight.dtype, out_dtype)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, z, w = ctx.saved_tensors
        eps, fp32_math, wdt, out_dtype = ctx.meta
        lib = N.load()
        dy = _dense16(dy.to(out_dtype))
        prob = _norm_problem(x, w.dtype, eps, fp32_math)
        ws = torch.empty(max(lib.gdn2_gated_norm_bwd_workspace_bytes(prob), 1), dtype=torch.uint8,
                         device=x.device)
        dx = torch.empty_like(x)
        dz = torch.empty_like(z)
        dw = torch.empty(x.shape[-1], dtype=torch.float32, device=x.device)
        N.check(lib.gdn2_gated_norm_bwd(prob, N.ptr(x), N.ptr(z), N.ptr(w), N.ptr(dy), N.ptr(dx),
                                        N.ptr(dz), N.ptr(dw), N.ptr(ws), ws.numel(),
                                        N.stream_of(x.device)), "gdn2_gated_norm_bwd")
        return dx, dz, dw.to(wdt), None, None


def gated_rms_norm(x, z, weight, eps=1e-5, fp32_math=None):
    """SiLU-gated RMSNorm of ``x`` gated by ``z`` (both ``[..., N]``).

    ``fp32_math`` defaults to whether CUDA autocast is active: under autocast
    the reference's ``pow`` / ``rsqrt`` run in fp32 and its result is fp32."""
    if fp32_math is None:
        fp32_math = torch.is_autocast_enabled("cuda") and x.dtype != torch.float32
    return GatedRMSNormFunction.apply(x, z, weight, eps, bool(fp32_math))

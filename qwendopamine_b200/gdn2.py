r"""``GatedDeltaNet2`` -- the GDN-2 token mixer, B200 build.

Drop-in for ``qwendopamine.models.gdn2.gdn2.GatedDeltaNet2``
(gdn2.py:491-1004): the constructor, the duck-typed config handling, every
parameter name / shape / initialisation, the ``forward(hidden_states,
attention_mask, past_key_values, use_cache, ...)`` signature, the returned
``(out, None, past_key_values)`` triple and the cache layout (fp32
``recurrent_state [N, H, K, V]`` plus three conv states) are unchanged, so
state_dicts, block registries and HF caches work as before.

What differs: the core recurrence always runs on the hand-written B200
kernels (:mod:`qwendopamine_b200.gdn2_ops`).  ``backend`` accepts the
reference's names; ``"auto"``, ``"cuda"``, ``"triton"`` and ``"fla"`` all
select the CUDA kernels.  The pure-PyTorch backends (``"torch"``,
``"torch-chunk"``, ``"torch-recurrent"``, ``"compiled"``) are not part of this
build and raise, as does any input that is not on a CUDA device: kernel
errors propagate instead of silently falling back (the reference's
``_warn_fallback_once`` path, gdn2.py:917-927).

Recurrence: ``S_t = (I - k_t (b_t*k_t)^T) Diag(e^{g_t}) S_{t-1} + k_t (w_t*v_t)^T``.
"""

from __future__ import annotations

import math
from typing import Any, Literal

import torch
import torch.nn.functional as F
from torch import nn

try:  # the HF cache classes are optional at import time
    from transformers.cache_utils import Cache
except ImportError:  # pragma: no cover
    class Cache:  # type: ignore[no-redef]
        pass

try:
    from transformers.cache_utils import LinearAttentionCacheLayerMixin
except ImportError:  # pragma: no cover
    LinearAttentionCacheLayerMixin = type(None)  # type: ignore[misc, assignment]

from .gdn2_ops.block_ops import gated_rms_norm, short_conv
from .gdn2_ops.chunk_gdn2 import chunk_gdn2
from .gdn2_ops.fused_recurrent_gdn2 import fused_recurrent_gdn2

# The reference's backend names (gdn2.py:58-66) plus "cuda".
GDN2_BACKENDS = (
    "auto",
    "torch",
    "torch-chunk",
    "torch-recurrent",
    "compiled",
    "triton",
    "fla",
    "cuda",
)
_CUDA_BACKENDS = ("auto", "cuda", "triton", "fla")


def resolve_gdn2_backend(requested: str, *, training: bool, seq_len: int) -> str:
    """Resolve the execution backend (reference gdn2.py:69-97).

    Every accelerated name resolves to ``"cuda"``; the pure-PyTorch names are
    returned unchanged and rejected by :class:`GatedDeltaNet2` at call time.
    """
    if requested not in GDN2_BACKENDS:
        raise ValueError(
            f"Invalid GDN-2 backend '{requested}'. Valid backends: {list(GDN2_BACKENDS)}")
    return "cuda" if requested in _CUDA_BACKENDS else requested


class ShortConvolution(nn.Module):
    """Causal depthwise 1-D convolution with optional SiLU (reference
    gdn2.py:372-430), computed by ``gdn2_conv_fwd`` / ``gdn2_conv_bwd``.
    With a cache and a single new token, the cached ``kernel_size - 1``
    inputs are prepended instead of zero padding; a longer input ignores the
    cache, as the reference does."""

    def __init__(self, hidden_size: int, kernel_size: int = 4, bias: bool = False,
                 activation: str | None = "silu") -> None:
        super().__init__()
        self.hidden_size = hidden_size
        self.kernel_size = kernel_size
        self.activation = activation
        self.conv1d = nn.Conv1d(hidden_size, hidden_size, kernel_size, groups=hidden_size,
                                bias=bias, padding=kernel_size - 1)

    def forward(self, x: torch.Tensor, cache: torch.Tensor | None = None,
                output_final_state: bool = False, cu_seqlens: torch.Tensor | None = None
                ) -> tuple[torch.Tensor, torch.Tensor | None]:
        if not x.is_cuda:
            raise RuntimeError("ShortConvolution (B200 build) runs on CUDA devices only")
        batch, t, d = x.shape
        keep = self.kernel_size - 1
        weight, bias = self.conv1d.weight, self.conv1d.bias
        if torch.is_autocast_enabled("cuda"):
            x = x.to(torch.get_autocast_dtype("cuda"))  # F.conv1d's autocast cast
        elif weight.dtype != x.dtype:
            raise RuntimeError(f"Input type ({x.dtype}) and weight type ({weight.dtype}) "
                               "should be the same")
        if cache is None and output_final_state and t == 1:
            cache = x.new_zeros(batch, d, keep)
        if cache is not None and t == 1:
            return short_conv(x, weight, bias, self.activation, prefix=cache.transpose(1, 2),
                              output_final_state=output_final_state)
        new_cache = x.transpose(1, 2)[:, :, -keep:] if output_final_state else None
        y, _ = short_conv(x, weight, bias, self.activation)
        return y, new_cache


class RMSNormGated(nn.Module):
    """SiLU-gated RMSNorm computed in the input dtype (reference
    gdn2.py:433-452; deliberately not the fp32-promoting variant)."""

    def __init__(self, hidden_size: int, eps: float = 1e-5) -> None:
        super().__init__()
        self.hidden_size = hidden_size
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size))

    def forward(self, x: torch.Tensor, z: torch.Tensor) -> torch.Tensor:
        # one kernel (gdn2_gated_norm_fwd / _bwd); under CUDA autocast the
        # reference's pow / rsqrt run in fp32 and so does the kernel
        return gated_rms_norm(x, z, self.weight, self.eps)


def _unpad_info(mask: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, int]:
    """Indices of real tokens, int32 cu_seqlens and the longest sequence."""
    lens = mask.sum(dim=-1, dtype=torch.int32)
    idx = torch.nonzero(mask.flatten(), as_tuple=False).flatten()
    cu = F.pad(torch.cumsum(lens, dim=0, dtype=torch.int32), (1, 0))
    return idx, cu, int(lens.max().item())


def _repad(x: torch.Tensor, idx: torch.Tensor, batch: int, seqlen: int) -> torch.Tensor:
    full = x.new_zeros(batch * seqlen, *x.shape[1:])
    full[idx] = x
    return full.view(batch, seqlen, *x.shape[1:])


def _heads(x: torch.Tensor, d: int) -> torch.Tensor:
    return x.view(*x.shape[:-1], x.shape[-1] // d, d)


class GatedDeltaNet2(nn.Module):
    """Gated DeltaNet 2 (GDN-2) token-mixing layer, B200 kernels."""

    def __init__(
        self,
        hidden_size_or_config: int | Any = 2048,
        hidden_size: int | None = None,
        num_heads: int | None = None,
        head_dim: int | None = None,
        layer_idx: int | None = None,
        mode: Literal["chunk", "fused_recurrent"] = "chunk",
        expand_v: float = 1.0,
        num_v_heads: int | None = None,
        use_short_conv: bool = True,
        allow_neg_eigval: bool = False,
        conv_size: int = 4,
        conv_bias: bool = False,
        norm_eps: float = 1e-5,
        chunk_size: int = 64,
        backend: str = "auto",
        compile_backend: bool = False,
        fp32_decay: bool = True,
        **kwargs: Any,
    ) -> None:
        super().__init__()
        cfg = hidden_size_or_config
        if hasattr(cfg, "hidden_size") or hasattr(cfg, "n_embd"):
            # duck-typed config, same attribute fallbacks as gdn2.py:515-540
            def pick(*names, default):
                for n in names:
                    if hasattr(cfg, n):
                        return getattr(cfg, n)
                return default

            hidden_size = pick("hidden_size", "n_embd", default=2048)
            num_heads = pick("num_heads", "n_head", default=16)
            head_dim = pick("head_dim", "head_size", default=128)
            num_v_heads = pick("num_v_heads", "n_query_groups", default=num_v_heads or num_heads)
            conv_size = pick("conv_size", "conv_kernel_size", default=conv_size)
            norm_eps = pick("norm_eps", "rms_norm_eps", default=norm_eps)
            allow_neg_eigval = pick("allow_neg_eigval", default=allow_neg_eigval)
            expand_v = pick("expand_v", default=expand_v)
            chunk_size = pick("chunk_size", "train_chunk_size", default=chunk_size)
            backend = pick("backend", default=backend)
            compile_backend = pick("compile_backend", default=compile_backend)
            fp32_decay = pick("fp32_decay", default=fp32_decay)
        elif hidden_size is None:
            hidden_size = int(cfg)

        if backend not in GDN2_BACKENDS:
            raise ValueError(
                f"Invalid GDN-2 backend '{backend}'. Valid backends: {list(GDN2_BACKENDS)}")

        self.hidden_size = hidden_size
        self.num_heads = 16 if num_heads is None else num_heads
        self.head_dim = 128 if head_dim is None else head_dim
        self.num_v_heads = self.num_heads if num_v_heads is None else num_v_heads
        if self.num_v_heads > self.num_heads and self.num_v_heads % self.num_heads != 0:
            raise ValueError(
                f"num_v_heads={self.num_v_heads} must be divisible by num_heads={self.num_heads}.")
        self.layer_idx = layer_idx
        self.mode = mode
        self.use_short_conv = use_short_conv
        self.allow_neg_eigval = allow_neg_eigval
        self.conv_size = conv_size
        self.conv_bias = conv_bias
        self.norm_eps = norm_eps
        self.expand_v = expand_v
        self.chunk_size = chunk_size
        self.backend = backend
        self.compile_backend = compile_backend
        self.fp32_decay = fp32_decay

        self.head_k_dim = self.head_dim
        self.head_v_dim = int(self.head_dim * self.expand_v)
        self.key_dim = int(self.num_heads * self.head_k_dim)
        self.value_dim = int(self.num_v_heads * self.head_v_dim)

        hs, kd, vd, hv = self.hidden_size, self.key_dim, self.value_dim, self.head_v_dim
        self.q_proj = nn.Linear(hs, kd, bias=False)
        self.k_proj = nn.Linear(hs, kd, bias=False)
        self.v_proj = nn.Linear(hs, vd, bias=False)
        if self.use_short_conv:
            self.q_conv1d = ShortConvolution(kd, kernel_size=conv_size, bias=conv_bias)
            self.k_conv1d = ShortConvolution(kd, kernel_size=conv_size, bias=conv_bias)
            self.v_conv1d = ShortConvolution(vd, kernel_size=conv_size, bias=conv_bias)
        self.f_proj = nn.Sequential(nn.Linear(hs, hv, bias=False), nn.Linear(hv, kd, bias=False))
        self.b_proj = nn.Linear(hs, kd, bias=False)
        self.w_proj = nn.Linear(hs, vd, bias=False)

        # decay parameters: A ~ U(1, 16); dt log-uniform in [1e-3, 1e-1]
        self.A_log = nn.Parameter(torch.empty(self.num_heads, dtype=torch.float32).uniform_(1, 16)
                                  .log())
        self.A_log._no_weight_decay = True  # type: ignore[attr-defined]
        lo, hi = math.log(0.001), math.log(0.1)
        dt = torch.exp(torch.rand(kd, dtype=torch.float32) * (hi - lo) + lo).clamp(min=1e-4)
        self.dt_bias = nn.Parameter(dt + torch.log(-torch.expm1(-dt)))  # softplus^-1(dt)
        self.dt_bias._no_weight_decay = True  # type: ignore[attr-defined]

        self.g_proj = nn.Sequential(nn.Linear(hs, hv, bias=False), nn.Linear(hv, vd, bias=True))
        self.o_norm = RMSNormGated(hv, eps=norm_eps)
        self.o_proj = nn.Linear(vd, hs, bias=False)
        self.apply(self._initialize_weights)

    def _initialize_weights(self, module: nn.Module) -> None:
        if getattr(module, "_is_hf_initialized", False):
            return
        if isinstance(module, nn.Linear):
            nn.init.xavier_uniform_(module.weight, gain=2 ** -2.5)
            if module.bias is not None:
                nn.init.zeros_(module.bias)
        elif isinstance(module, nn.Conv1d):
            nn.init.kaiming_uniform_(module.weight, a=math.sqrt(5))
            if module.bias is not None:
                nn.init.zeros_(module.bias)
        elif isinstance(module, RMSNormGated):
            nn.init.ones_(module.weight)
        module._is_hf_initialized = True  # type: ignore[attr-defined]

    # ---- cache glue (reference gdn2.py:655-778) ----------------------------
    def _get_cache(self, past_key_values):
        if past_key_values is None:
            return None, None
        if isinstance(past_key_values, dict):
            return past_key_values.get("recurrent_state"), past_key_values.get("conv_state")
        if isinstance(past_key_values, Cache):
            layers = getattr(past_key_values, "layers", [])
            if self.layer_idx is None or self.layer_idx >= len(layers):
                return None, None
            layer = layers[self.layer_idx]
            rec = getattr(layer, "recurrent_states", None)
            if rec is None:
                rec = getattr(layer, "recurrent_state", None)
            elif isinstance(rec, dict):
                rec = rec.get(0)
            elif isinstance(rec, (list, tuple)):
                rec = rec[0] if rec else None
            elif not isinstance(rec, torch.Tensor):
                rec = None
            conv = getattr(layer, "conv_states", None)
            if conv is None:
                conv = getattr(layer, "conv_state", None)
            elif isinstance(conv, dict):
                conv = (conv.get(0), conv.get(1), conv.get(2))
            elif isinstance(conv, (list, tuple)) and len(conv) == 3:
                conv = tuple(conv)
            else:
                conv = None
            return rec, conv
        return None, None

    def _update_cache(self, past_key_values, recurrent_state, conv_state) -> None:
        if past_key_values is None:
            return
        if isinstance(past_key_values, dict):
            if recurrent_state is not None:
                past_key_values["recurrent_state"] = recurrent_state
            if conv_state is not None:
                past_key_values["conv_state"] = conv_state
            return
        if self.layer_idx is None or not isinstance(past_key_values, Cache):
            return
        layers = getattr(past_key_values, "layers", [])
        if self.layer_idx >= len(layers):
            return
        layer = layers[self.layer_idx]
        recurrent_layer = (isinstance(layer, LinearAttentionCacheLayerMixin)
                           or hasattr(layer, "update_recurrent_state")
                           or hasattr(layer, "recurrent_states"))
        if recurrent_state is not None:
            if recurrent_layer and hasattr(past_key_values, "update_recurrent_state"):
                past_key_values.update_recurrent_state(recurrent_state, self.layer_idx)
            else:
                rec = getattr(layer, "recurrent_states", None)
                if isinstance(rec, dict):
                    rec[0] = recurrent_state
                elif hasattr(layer, "recurrent_state"):
                    layer.recurrent_state = recurrent_state
        if conv_state is not None:
            if recurrent_layer and hasattr(past_key_values, "update_conv_state"):
                past_key_values.update_conv_state(conv_state, self.layer_idx)
            else:
                conv = getattr(layer, "conv_states", None)
                if isinstance(conv, dict):
                    conv[0], conv[1], conv[2] = conv_state
                elif hasattr(layer, "conv_state"):
                    layer.conv_state = conv_state

    # ---- forward -----------------------------------------------------------
    def forward(
        self,
        hidden_states: torch.Tensor,
        attention_mask: torch.Tensor | None = None,
        past_key_values: Cache | dict[str, Any] | None = None,
        use_cache: bool | None = False,
        output_attentions: bool | None = False,
        **kwargs: Any,
    ) -> tuple[torch.Tensor, torch.Tensor | None, Cache | dict[str, Any] | None]:
        batch, seq_len, _ = hidden_states.shape
        mode = "fused_recurrent" if (seq_len <= 64 and not self.training) else self.mode
        backend = resolve_gdn2_backend(self.backend, training=self.training, seq_len=seq_len)
        if backend != "cuda":
            raise RuntimeError(
                f"GDN-2 backend '{backend}' (pure PyTorch) is not part of the B200 build; "
                "use backend='auto' or 'cuda'.")
        if not hidden_states.is_cuda:
            raise RuntimeError(
                "GatedDeltaNet2 (B200 build) runs on CUDA devices only; there is no CPU "
                "fallback.")

        recurrent_state, conv_states = self._get_cache(past_key_values)
        cq, ck, cv = conv_states if conv_states is not None else (None, None, None)
        cu_seqlens = kwargs.get("cu_seqlens")

        padded = (attention_mask is not None and seq_len > 1 and past_key_values is None
                  and bool((attention_mask == 0).any()))
        indices = None
        if padded:
            indices, cu_seqlens, _ = _unpad_info(attention_mask)
            hidden_states = hidden_states.reshape(-1, *hidden_states.shape[2:])[indices][None]

        want_cache = bool(use_cache)
        x = hidden_states
        if self.use_short_conv:
            q, cq = self.q_conv1d(self.q_proj(x), cache=cq, output_final_state=want_cache,
                                  cu_seqlens=cu_seqlens)
            k, ck = self.k_conv1d(self.k_proj(x), cache=ck, output_final_state=want_cache,
                                  cu_seqlens=cu_seqlens)
            v, cv = self.v_conv1d(self.v_proj(x), cache=cv, output_final_state=want_cache,
                                  cu_seqlens=cu_seqlens)
        else:
            q, k, v = F.silu(self.q_proj(x)), F.silu(self.k_proj(x)), F.silu(self.v_proj(x))

        # With fp32 decays the kernels apply the gate themselves
        # (use_gate_in_kernel: -exp(A_log) * softplus(f + dt_bias) on the raw
        # projection, the reference's gdn2.py:840-845 formula); otherwise g is
        # formed here and rounded to the token dtype as the reference does.
        gate_in_kernel = self.fp32_decay
        if gate_in_kernel:
            g = self.f_proj(x).float()
        else:
            decay = self.A_log.float().exp().repeat_interleave(self.head_k_dim)
            g = (-decay * F.softplus(self.f_proj(x).float() + self.dt_bias)).to(x.dtype)
        A_log, dt_bias = self.A_log, self.dt_bias
        b = self.b_proj(x).sigmoid()
        w = self.w_proj(x).sigmoid()

        dk, dv = self.head_k_dim, self.head_v_dim
        q, k, g, b = (_heads(t, dk) for t in (q, k, g, b))
        v, w = _heads(v, dv), _heads(w, dv)
        if self.num_v_heads > self.num_heads:
            rep = self.num_v_heads // self.num_heads
            q, k, g, b = (t.repeat_interleave(rep, dim=-2) for t in (q, k, g, b))
            A_log = A_log.repeat_interleave(rep)
            dt_bias = dt_bias.view(self.num_heads, dk).repeat_interleave(rep, dim=0).reshape(-1)
        if self.allow_neg_eigval:
            b = b * 2.0

        if recurrent_state is not None and recurrent_state.dtype != torch.float32:
            recurrent_state = recurrent_state.float()
        op = chunk_gdn2 if mode == "chunk" else fused_recurrent_gdn2
        o, recurrent_state = op(
            q=q, k=k, v=v, g=g, b=b, w=w, A_log=A_log, dt_bias=dt_bias,
            initial_state=recurrent_state, output_final_state=want_cache,
            use_qk_l2norm_in_kernel=True, use_gate_in_kernel=gate_in_kernel,
            cu_seqlens=cu_seqlens)

        if use_cache or past_key_values is not None:
            self._update_cache(past_key_values, recurrent_state,
                               (cq, ck, cv) if self.use_short_conv else None)

        gate = _heads(self.g_proj(x), dv)
        o = self.o_norm(o, gate)
        out = self.o_proj(o.reshape(*o.shape[:-2], -1))
        if padded and indices is not None:
            out = _repad(out.squeeze(0), indices, batch, seq_len)
        return out, None, past_key_values

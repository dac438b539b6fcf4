"""Sequence (context) parallel chunkwise GDN-2 on B200.

The reference has context parallelism only for KDA, through FLA-CP
(``gdn2_ops/chunk_kda.py:182-1299``): each rank runs a pre-scan over its span,
the per-rank results are all-gathered, and each rank folds its predecessors
into its initial state.  This module applies that algorithm to GDN-2 with the
B200 kernels:

forward (rank r owns a contiguous span of whole 64-token chunks):
    1. ``gdn2_chunk_fwd_intra`` on the local span;
    2. ``gdn2_cp_fwd_prescan``: the span's affine map ``S_out = M S_in + h_e``
       as ``hm = [h_e | M]`` (``[N, H, K, V+K]`` fp32);
    3. all-gather of ``hm`` over the group (NCCL on GPUs);
    4. ``gdn2_cp_merge``: ``x = h0;  x = M_j x + h_e_j`` for ``j < r``;
    5. ``gdn2_chunk_fwd_state`` from ``x``: local outputs and end state.
backward:
    1. ``gdn2_cp_bwd_prescan``: the span-start state gradient produced by the
       local outputs and by the gradient of the returned end state ``S_r``;
    2. all-gather of it;
    3. ``gdn2_cp_merge``: ``x = 0;  x = M_j^T x + dh_j`` for ``j > r``, plus
       the gradient of ``S_r`` itself -- the gradient w.r.t. this span's end
       state;
    4. ``gdn2_chunk_bwd`` with that end-state gradient.
Each rank's local backward then yields exact gradients for its own inputs.

The block's causal short convolution needs the W - 1 tokens before a span
(``pre_num_conv_tokens`` in FLA-CP's context, ``fla/ops/cp/context.py``):
:func:`short_conv_cp` gathers every span's last W - 1 rows, runs the
convolution with the previous span's rows as its prefix, and in the backward
sends the prefix gradient back to the rank that owns those rows, so the whole
block, not only the core recurrence, runs sequence-parallel.

The gather is a plain function argument so the same code runs over NCCL,
over gloo (CPU tests of the exchange) or emulated inside one process.
"""

from __future__ import annotations

from typing import Callable

import torch

from .. import _native as N
from .chunk_gdn2 import _aligned16, _require_cuda

__all__ = ["chunk_gdn2_cp", "CPChunkGDN2Function", "ConvHaloFunction", "gather_span_maps",
           "short_conv_cp"]

Gather = Callable[[torch.Tensor], torch.Tensor]


def gather_span_maps(t: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather ``t`` over ``group`` into a rank-major ``[world, *t.shape]``
    tensor (``all_gather_into_tensor`` on NCCL, a list gather otherwise)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    out = t.new_empty((world, *t.shape))
    t = t.contiguous()
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, t, group=group)
    else:
        parts = list(out.unbind(0))
        dist.all_gather(parts, t, group=group)
    return out


def _problem(H, K, V, dtype, l2norm, scale, tables):
    return N.ChunkProblem(H, K, V, N.dtype_code(dtype), int(bool(l2norm)), float(scale),
                          tables.struct())


def _sub_spans(B, T, H, dtype):
    """Sub-spans per sequence inside a rank's span.  The pre-scans and state
    passes walk their span's chunks one after another with one CTA (or a few
    column slices) per sequence-head; cutting the span into S pieces cuts
    every such chain S-fold and multiplies the CTAs by S.  Four pieces while
    the full-width tensor-core state passes (one CTA per sequence-head) still
    fit one wave and each piece keeps 32 chunks; else two while the forward
    pre-scan ([h | M], two 128-column slices per sequence-head) fits one
    wave; else one.  (The forward pre-scan at four pieces runs two waves of
    half-length chains: the same time as one wave at two.)"""
    if dtype != torch.bfloat16:
        return 1
    nch = (T + N.CHUNK - 1) // N.CHUNK
    if B * H * 4 <= 148 and nch >= 4 * 32:
        return 4
    return 2 if (B * H * 2 * 2 <= 148 and nch >= 64) else 1


def sub_spans_single(B, T, H, K, V, dtype):
    """Sub-spans for whole sequences on one GPU (world 1) when few
    sequence-heads would leave the state passes' chains on a handful of SMs:
    the pre-scan, the unfold of the start states and the state passes on S
    pieces replace one walk over every chunk.  The largest power of two with
    B*H*S full-width state-pass CTAs in one wave and 64 chunks per piece,
    used from S = 8 on (below that the pre-scan costs what it saves); 1 means
    the plain chunk path."""
    if dtype != torch.bfloat16 or K != 128 or V != 128:
        return 1
    nch = (T + N.CHUNK - 1) // N.CHUNK
    S = 1
    while B * H * S * 2 <= 148 and nch // (S * 2) >= 64:
        S *= 2
    return S if S >= 8 else 1


def _unfold_kernel_ok(hm_sub):
    B, S, H, K, VK = hm_sub.shape
    return B == 1 and K == 128 and VK - K == 128 and hm_sub.is_cuda


# The span-map folds run as fp32 torch products on the device (a few batched
# K x K by K x (V+K) products per step) with TF32 switched off for their
# duration, so they keep fp32 accuracy whatever the caller's matmul setting.
class _NoTF32:
    def __enter__(self):
        self.prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False

    def __exit__(self, *exc):
        torch.backends.cuda.matmul.allow_tf32 = self.prev


def _compose_maps(hm_sub):
    """[h_e | M] of consecutive sub-spans ([B, S, H, K, V+K]) -> the map of the
    whole span: x = [0 | I];  x = M_s x + [h_e_s | 0]  for s = 0 .. S-1."""
    B, S, H, K, VK = hm_sub.shape
    V = VK - K
    x = hm_sub[:, 0].clone()
    with _NoTF32():
        for j in range(1, S):
            x = torch.matmul(hm_sub[:, j, ..., V:], x)
            x[..., :V] += hm_sub[:, j, ..., :V]
    return x.contiguous()


def _unfold_states(h0, hm_sub, kern=None):
    """Initial state of every sub-span from the span's: s_0 = h0,
    s_j = M_{j-1} s_{j-1} + h_e_{j-1}.  Returns [B*S, H, K, V].  With
    ``kern = (lib, prob_span, stream)`` and one sequence, one gdn2_cp_unfold
    launch does the whole scan."""
    B, S, H, K, VK = hm_sub.shape
    V = VK - K
    if kern is not None and _unfold_kernel_ok(hm_sub):
        lib, prob_span, st = kern
        out = torch.empty(B * S, H, K, V, dtype=torch.float32, device=hm_sub.device)
        N.check(lib.gdn2_cp_unfold(prob_span, N.ptr(hm_sub), None, S, 1, N.ptr(h0), N.ptr(out),
                                   st), "gdn2_cp_unfold")
        return out
    out = [h0]
    with _NoTF32():
        for j in range(1, S):
            out.append(torch.baddbmm(hm_sub[:, j - 1, ..., :V].reshape(B * H, K, V),
                                     hm_sub[:, j - 1, ..., V:].reshape(B * H, K, K),
                                     out[-1].reshape(B * H, K, V)).view(B, H, K, V))
    return torch.stack(out, 1).reshape(B * S, H, K, V).contiguous()


def _compose_grads(dhm_sub, hm_sub, dht):
    """Span-start gradient of consecutive sub-spans' outputs (dhm_sub
    [B, S, H, K, V], zero end gradient each) and of the span's end-state
    gradient dht (or None): x = dht;  x = M_s^T x + dhm_s  for s = S-1 .. 0."""
    B, S, H, K, V = dhm_sub.shape
    x = dht if dht is not None else torch.zeros_like(dhm_sub[:, 0])
    with _NoTF32():
        for j in range(S - 1, -1, -1):
            x = torch.baddbmm(dhm_sub[:, j].reshape(B * H, K, V),
                              hm_sub[:, j, ..., V:].reshape(B * H, K, K).transpose(-1, -2),
                              x.reshape(B * H, K, V)).view(B, H, K, V)
    return x.contiguous()


def _unfold_grads(dht_span, dhm_sub, hm_sub, kern=None):
    """End-state gradient of every sub-span from the span's: g_{S-1} =
    dht_span,  g_j = M_{j+1}^T g_{j+1} + dhm_{j+1}.  Returns [B*S, H, K, V]
    (one gdn2_cp_unfold launch with ``kern`` and one sequence)."""
    B, S, H, K, V = dhm_sub.shape
    if kern is not None and _unfold_kernel_ok(hm_sub):
        lib, prob_span, st = kern
        out = torch.empty(B * S, H, K, V, dtype=torch.float32, device=hm_sub.device)
        dhm = dhm_sub.contiguous()
        N.check(lib.gdn2_cp_unfold(prob_span, N.ptr(hm_sub), N.ptr(dhm), S, 0,
                                   N.ptr(dht_span.contiguous()), N.ptr(out), st),
                "gdn2_cp_unfold (backward)")
        return out
    out = [dht_span]
    with _NoTF32():
        for j in range(S - 2, -1, -1):
            out.append(torch.baddbmm(dhm_sub[:, j + 1].reshape(B * H, K, V),
                                     hm_sub[:, j + 1, ..., V:].reshape(B * H, K, K).transpose(-1, -2),
                                     out[-1].reshape(B * H, K, V)).view(B, H, K, V))
    out.reverse()
    return torch.stack(out, 1).reshape(B * S, H, K, V).contiguous()


class CPChunkGDN2Function(torch.autograd.Function):
    """Autograd wrapper of the sequence-parallel forward/backward for one rank."""

    @staticmethod
    def forward(ctx, q, k, v, g, b, w, initial_state, scale, l2norm, rank, world, gather):
        lib = N.load()
        q, k, v, g, b, w = _aligned16(q, k, v, g, b, w)
        B, T, H, K = q.shape
        V = v.shape[-1]
        dev = q.device
        S = sub_spans_single(B, T, H, K, V, q.dtype) if world == 1 else _sub_spans(B, T, H, q.dtype)
        # the kernels see the span as B*S sequences (same chunks)
        tables = N.split_tables(B, T, S, dev) if S > 1 else N.seq_tables(B, T, dev)
        prob = _problem(H, K, V, q.dtype, l2norm, scale, tables)
        prob_span = _problem(H, K, V, q.dtype, l2norm, scale, N.seq_tables(B, T, dev))
        st = N.stream_of(dev)
        sbytes = lib.gdn2_chunk_saved_bytes(prob)
        saved = torch.empty(max(sbytes, 1), dtype=torch.uint8, device=dev)
        with N.phase("fwd_intra"):
            N.check(lib.gdn2_chunk_fwd_intra(prob, N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(g),
                                             N.ptr(b), N.ptr(w), N.ptr(saved), sbytes, st),
                    "gdn2_chunk_fwd_intra")
        hm_sub = torch.empty(B * S, H, K, V + K, dtype=torch.float32, device=dev)
        with N.phase("fwd_prescan"):
            N.check(lib.gdn2_cp_fwd_prescan(prob, N.ptr(saved), sbytes, N.ptr(hm_sub), None, 0,
                                            st), "gdn2_cp_fwd_prescan")
        hm_sub = hm_sub.view(B, S, H, K, V + K)
        kern = (lib, prob_span, st)
        if world > 1:
            with N.phase("fwd_fold"):
                hm = hm_sub[:, 0] if S == 1 else _compose_maps(hm_sub)
            with N.phase("fwd_gather"):
                hm_all = gather(hm.contiguous())
            h0 = torch.empty(B, H, K, V, dtype=torch.float32, device=dev)
            with N.phase("fwd_merge"):
                N.check(lib.gdn2_cp_merge(prob_span, N.ptr(hm_all), None, rank, world, 1,
                                          N.ptr(initial_state), N.ptr(h0), st), "gdn2_cp_merge")
        else:  # one span: no maps to exchange, its start state is the initial state
            hm_all = hm_sub.new_empty(0)
            h0 = (initial_state.float().contiguous() if initial_state is not None
                  else torch.zeros(B, H, K, V, dtype=torch.float32, device=dev))
        with N.phase("fwd_unfold" if S > 1 and _unfold_kernel_ok(hm_sub) else "fwd_fold"):
            h0_sub = h0 if S == 1 else _unfold_states(h0, hm_sub, kern)
        o = torch.empty_like(v)
        ht_sub = torch.empty(B * S, H, K, V, dtype=torch.float32, device=dev)
        with N.phase("fwd_state"):
            N.check(lib.gdn2_chunk_fwd_state(prob, N.ptr(h0_sub), N.ptr(o), N.ptr(ht_sub),
                                             N.ptr(saved), sbytes, st), "gdn2_chunk_fwd_state")
        ht = ht_sub.view(B, S, H, K, V)[:, S - 1].contiguous()
        ctx.save_for_backward(q, k, v, g, b, w, saved, h0, hm_all, hm_sub)
        ctx.meta = (scale, l2norm, rank, world, gather, tables, initial_state is not None, S)
        return o, ht

    @staticmethod
    def backward(ctx, do, dht):
        q, k, v, g, b, w, saved, h0, hm_all, hm_sub = ctx.saved_tensors
        scale, l2norm, rank, world, gather, tables, had_h0, S = ctx.meta
        lib = N.load()
        B, T, H, K = q.shape
        V = v.shape[-1]
        dev = q.device
        prob = _problem(H, K, V, q.dtype, l2norm, scale, tables)
        prob_span = _problem(H, K, V, q.dtype, l2norm, scale, N.seq_tables(B, T, dev))
        st = N.stream_of(dev)
        sbytes = lib.gdn2_chunk_saved_bytes(prob)
        (do,) = _aligned16(do.to(q.dtype).contiguous())
        last = rank == world - 1
        # dht is the gradient that reaches this rank's end state S_r directly
        # (a loss on the returned state; on the last rank S_r is the
        # sequence's final state).  It enters the span-start gradient sent to
        # the earlier ranks, and it adds to what the later ranks' outputs
        # send back through S_r.
        dht_direct = dht.float().contiguous() if dht is not None else None
        # The backward workspace also serves the pre-scan (it then runs as the
        # tensor-core state pass, whose per-chunk tiles the real pass rewrites).
        wbytes = lib.gdn2_chunk_bwd_workspace_bytes(prob)
        ws = torch.empty(max(wbytes, 1), dtype=torch.uint8, device=dev)
        pbytes = lib.gdn2_cp_workspace_bytes(prob)
        pws, pwb = (N.ptr(ws), wbytes) if 0 < pbytes <= wbytes else (None, 0)
        # Span-start gradient of the local outputs and of dht_direct.
        if S == 1:
            dhm = torch.empty(B, H, K, V, dtype=torch.float32, device=dev)
            with N.phase("bwd_prescan"):
                N.check(lib.gdn2_cp_bwd_prescan(prob, N.ptr(saved), sbytes, N.ptr(do),
                                                N.ptr(dht_direct), N.ptr(dhm), pws, pwb, st),
                        "gdn2_cp_bwd_prescan")
        else:
            dhm_sub = torch.empty(B * S, H, K, V, dtype=torch.float32, device=dev)
            with N.phase("bwd_prescan"):
                N.check(lib.gdn2_cp_bwd_prescan(prob, N.ptr(saved), sbytes, N.ptr(do), None,
                                                N.ptr(dhm_sub), pws, pwb, st),
                        "gdn2_cp_bwd_prescan")
            dhm_sub = dhm_sub.view(B, S, H, K, V)
            if world > 1:
                with N.phase("bwd_fold"):
                    dhm = _compose_grads(dhm_sub, hm_sub, dht_direct)
        if world > 1:
            with N.phase("bwd_gather"):
                dhm_all = gather(dhm)
        if last:
            dht_local = dht_direct
        else:
            # x = 0;  x = M_j^T x + dh_j  for j = world-1 .. r+1, then + dht_direct
            dht_local = torch.empty(B, H, K, V, dtype=torch.float32, device=dev)
            with N.phase("bwd_merge"):
                N.check(lib.gdn2_cp_merge(prob_span, N.ptr(hm_all), N.ptr(dhm_all), rank, world,
                                          0, None, N.ptr(dht_local), st),
                        "gdn2_cp_merge (backward)")
                if dht_direct is not None:
                    dht_local += dht_direct
        if S > 1:
            end = dht_local if dht_local is not None else torch.zeros_like(h0)
            with N.phase("bwd_unfold" if _unfold_kernel_ok(hm_sub) else "bwd_fold"):
                dht_local = _unfold_grads(end, dhm_sub, hm_sub, (lib, prob_span, st))
        grads = {n: torch.empty_like(t) for n, t in zip("qkvgbw", (q, k, v, g, b, w))}
        dh0_sub = torch.empty(B * S, H, K, V, dtype=torch.float32, device=dev)
        # gdn2_chunk_bwd's two phases, called one by one so each can be timed
        with N.phase("bwd_state"):
            N.check(lib.gdn2_chunk_bwd_state(prob, N.ptr(saved), sbytes, N.ptr(do),
                                             N.ptr(dht_local), N.ptr(dh0_sub), N.ptr(ws), wbytes,
                                             st), "gdn2_chunk_bwd_state")
        with N.phase("bwd_intra"):
            N.check(lib.gdn2_chunk_bwd_intra(prob, N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(g),
                                             N.ptr(b), N.ptr(w), N.ptr(saved), sbytes, N.ptr(do),
                                             *(N.ptr(grads[n]) for n in "qkvgbw"), N.ptr(ws),
                                             wbytes, st), "gdn2_chunk_bwd_intra")
        dh0 = dh0_sub.view(B, S, H, K, V)[:, 0].contiguous()
        # dh0 on rank 0 is the gradient of the global initial state; on later
        # ranks the initial state is an internal value whose gradient has been
        # routed to the earlier ranks through their end-state gradients.
        dinit = dh0 if (had_h0 and rank == 0) else None
        return (grads["q"], grads["k"], grads["v"], grads["g"], grads["b"], grads["w"], dinit,
                None, None, None, None, None)


def chunk_gdn2_cp(q, k, v, g, b, w, *, rank: int, world: int, gather: Gather,
                  scale: float | None = None, initial_state: torch.Tensor | None = None,
                  use_qk_l2norm_in_kernel: bool = True):
    """Sequence-parallel GDN-2 for the span this rank owns.

    q, k, b, g: ``[B, T_r, H, K]``; v, w: ``[B, T_r, H, V]`` -- rank r's
    contiguous slice of every sequence; every rank but the last must hold a
    whole number of 64-token chunks.  ``initial_state`` is the global initial
    state (``[B, H, K, V]`` fp32, the same on every rank, or None).
    ``gather(t)`` must return the rank-major all-gather ``[world, *t.shape]``
    (:func:`gather_span_maps` over a process group).

    Returns ``(o_r, S_r)``: the local outputs and the state at the end of this
    rank's span (on the last rank: the sequence's final state).  Both are
    differentiable on every rank: a loss on a middle rank's ``S_r`` sends its
    gradient to this rank's inputs and, through the gathered span-start
    gradients, to every earlier rank's.
    """
    _require_cuda(q, k, v, g, b, w, initial_state)
    assert q.shape == k.shape == g.shape == b.shape, "q, k, g, b must have the same shape."
    assert w.shape == v.shape and v.shape[:3] == q.shape[:3], "v, w must be [B, T, H, V]."
    if rank < world - 1 and q.shape[1] % N.CHUNK != 0:
        raise ValueError(
            f"rank {rank} holds {q.shape[1]} tokens: every rank but the last must own whole "
            f"{N.CHUNK}-token chunks")
    if initial_state is not None:
        assert initial_state.dtype == torch.float32, "initial_state must be in float32."
        initial_state = initial_state.contiguous()
    if scale is None:
        scale = k.shape[-1] ** -0.5
    if world == 1:
        # a single span: no span maps to exchange
        from .chunk_gdn2 import chunk_gdn2

        return chunk_gdn2(q, k, v, g, b, w, scale=scale, initial_state=initial_state,
                          output_final_state=True,
                          use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel)
    dt = q.dtype
    q, k, v, b, w = (x.to(dt).contiguous() for x in (q, k, v, b, w))
    g = g.float().contiguous()
    with torch.cuda.device(q.device):
        return CPChunkGDN2Function.apply(q, k, v, g, b, w, initial_state, scale,
                                         use_qk_l2norm_in_kernel, rank, world, gather)


class ConvHaloFunction(torch.autograd.Function):
    """Boundary rows of the causal convolution across spans.

    forward: every rank contributes its span's last W - 1 rows ``tail``
    ``[B, W-1, D]``; rank r receives rank r-1's rows as its prefix (zeros on
    rank 0, the sequence start).  backward: the prefix gradients are gathered
    and rank r takes rank r+1's as the gradient of its own tail (zero on the
    last rank).  Every rank takes part in both gathers."""

    @staticmethod
    def forward(ctx, tail, rank, world, gather):
        ctx.rank, ctx.world, ctx.gather = rank, world, gather
        tails = gather(tail.contiguous())
        return tails[rank - 1].clone() if rank > 0 else torch.zeros_like(tail)

    @staticmethod
    def backward(ctx, dprefix):
        grads = ctx.gather(dprefix.contiguous())
        dtail = (grads[ctx.rank + 1].clone() if ctx.rank + 1 < ctx.world
                 else torch.zeros_like(dprefix))
        return dtail, None, None, None


def short_conv_cp(x, weight, bias=None, activation="silu", *, rank: int, world: int,
                  gather: Gather):
    """Sequence-parallel ``ShortConvolution`` (gdn2.py:372-430) for rank r's
    contiguous span ``x`` ``[B, T_r, D]`` of every sequence (T_r >= W - 1):
    the outputs equal the single-device convolution's rows of that span, and
    the backward gives this span's dx, including the part that reaches it
    through the next span's prefix.  The weight and bias gradients are this
    span's share; summing them over the ranks (as a data-parallel all-reduce
    of parameter gradients does) gives the whole sequence's."""
    from .block_ops import short_conv

    W = weight.shape[-1]
    if W == 1 or world == 1:
        return short_conv(x, weight, bias, activation)[0]
    if x.shape[1] < W - 1:
        raise ValueError(f"rank {rank} holds {x.shape[1]} tokens; the convolution's halo needs "
                         f"at least {W - 1} per span")
    prefix = ConvHaloFunction.apply(x[:, -(W - 1):], rank, world, gather)
    return short_conv(x, weight, bias, activation, prefix=prefix)[0]


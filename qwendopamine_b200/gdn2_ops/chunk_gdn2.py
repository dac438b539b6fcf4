"""Chunkwise GDN-2 forward/backward on B200 -- drop-in for the reference's
``qwendopamine.models.gdn2.gdn2_ops.chunk_gdn2``.

Same public names, argument meanings and error behaviour as the reference
(``chunk_gdn2.py:1267-1434`` and ``ChunkGDN2Function`` :2328-2547); the work is
done by ``libgdn2_b200.so`` through its C ABI (``include/gdn2_b200.h``):

* ``gdn2_chunk_fwd``  -- intra-chunk solve + state pass with fused output;
* ``gdn2_chunk_bwd``  -- reverse state pass + fused per-chunk gradients.

Tensors must live on a CUDA device: there is no CPU path (the reference's
``not q.is_cuda`` branch, :1396-1410, falls back to torch; this build raises).
"""

from __future__ import annotations

import torch

from .. import _native as N

__all__ = ["ChunkGDN2Function", "chunk_gdn2", "chunk_gdn2_fwd", "chunk_gdn2_bwd"]


class GateParams:
    """Gate-in-kernel parameters for the C ABI: fp32 ``A_log`` [H] and
    ``dt_bias`` [H*K] (or None); mode 1 is ``-exp(A_log) * softplus(g +
    dt_bias)``, mode 2 ``lower_bound * sigmoid(exp(A_log) * (g + dt_bias))``."""

    def __init__(self, A_log, dt_bias, lower_bound):
        self.A_log = A_log
        self.dt_bias = dt_bias
        self.mode = 1 if lower_bound is None else 2
        self.lower_bound = 0.0 if lower_bound is None else float(lower_bound)


def _problem(H, K, V, dtype, l2norm, scale, tables, gate=None, dA_log=None, ddt_bias=None):
    prob = N.ChunkProblem(H, K, V, N.dtype_code(dtype), int(bool(l2norm)), float(scale),
                          tables.struct())
    if gate is not None:
        prob.A_log = N.ptr(gate.A_log)
        prob.dt_bias = N.ptr(gate.dt_bias)
        prob.gate = gate.mode
        prob.lower_bound = gate.lower_bound
        prob.dA_log = N.ptr(dA_log)
        prob.ddt_bias = N.ptr(ddt_bias)
    return prob


def _gate_in_kernel_ok(dtype, K, V):
    """The bf16 kernels apply the gate themselves (the C ABI's 16-bit path:
    bf16, K and V multiples of 8 up to 128); other problems gate with torch
    ops."""
    return dtype == torch.bfloat16 and K % 8 == 0 and V % 8 == 0 and K <= 128 and V <= 128


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "chunk_gdn2: inputs must be CUDA tensors -- the B200 build has no CPU path")


def _aligned16(*ts):
    """The C ABI's 16-bit path moves rows with bulk copies and needs tensors
    that start on a 16-byte boundary; copy the (rare) misaligned views."""
    return tuple(t if t is None or t.data_ptr() % 16 == 0 else t.clone() for t in ts)


def chunk_gdn2_fwd(q, k, v, g, b, w, scale, initial_state, output_final_state, tables,
                   use_qk_l2norm, keep_saved=True, gate=None):
    """Run the forward; returns ``(o, final_state, saved)``.

    q, k, b: [B, T, H, K]; v, w: [B, T, H, V] (one dtype); g: fp32 [B, T, H, K]
    (the raw gate input when ``gate`` is a :class:`GateParams`);
    initial_state: fp32 [N, H, K, V] or None.
    """
    lib = N.load()
    B, T, H, K = q.shape
    V = v.shape[-1]
    q, k, v, g, b, w = _aligned16(q, k, v, g, b, w)
    prob = _problem(H, K, V, q.dtype, use_qk_l2norm, scale, tables, gate)
    nbytes = lib.gdn2_chunk_saved_bytes(prob)
    if nbytes == 0 and tables.n_chunks > 0:
        N.check(N.ERR_INVALID, "gdn2_chunk_saved_bytes")
    saved = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=q.device)
    o = torch.empty_like(v)
    ht = (q.new_empty(tables.n_seqs, H, K, V, dtype=torch.float32)
          if output_final_state else None)
    st = N.stream_of(q.device)
    # gdn2_chunk_fwd's two phases, called one by one so each can be timed
    with N.phase("fwd_intra"):
        N.check(lib.gdn2_chunk_fwd_intra(prob, N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(g), N.ptr(b),
                                         N.ptr(w), N.ptr(saved), nbytes, st),
                "gdn2_chunk_fwd_intra")
    with N.phase("fwd_state"):
        N.check(lib.gdn2_chunk_fwd_state(prob, N.ptr(initial_state), N.ptr(o), N.ptr(ht),
                                         N.ptr(saved), nbytes, st), "gdn2_chunk_fwd_state")
    return o, ht, (saved if keep_saved else None)


def chunk_gdn2_bwd(q, k, v, g, b, w, saved, do, dht, scale, initial_state, tables,
                   use_qk_l2norm, gate=None):
    """Run the backward; returns ``(dq, dk, dv, dg, db, dw, dh0)``, plus
    ``(dA_log, ddt_bias)`` (fp32 [H], [H*K] or None) when ``gate`` is given."""
    lib = N.load()
    B, T, H, K = q.shape
    V = v.shape[-1]
    q, k, v, g, b, w, do = _aligned16(q, k, v, g, b, w, do)
    dA_log = ddt_bias = None
    if gate is not None:
        dA_log = torch.zeros(H, dtype=torch.float32, device=q.device)
        if gate.dt_bias is not None:
            ddt_bias = torch.zeros(H * K, dtype=torch.float32, device=q.device)
    prob = _problem(H, K, V, q.dtype, use_qk_l2norm, scale, tables, gate, dA_log, ddt_bias)
    nbytes = lib.gdn2_chunk_saved_bytes(prob)
    wbytes = lib.gdn2_chunk_bwd_workspace_bytes(prob)
    ws = torch.empty(max(wbytes, 1), dtype=torch.uint8, device=q.device)
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    db = torch.empty_like(b)
    dw = torch.empty_like(w)
    dg = torch.empty_like(g)
    dh0 = torch.empty_like(initial_state) if initial_state is not None else None
    if tables.total < B * T:  # rows outside every sequence get zero gradient
        for t in (dq, dk, dv, db, dw, dg):
            t.zero_()
    st = N.stream_of(q.device)
    # gdn2_chunk_bwd's two phases, called one by one so each can be timed
    with N.phase("bwd_state"):
        N.check(lib.gdn2_chunk_bwd_state(prob, N.ptr(saved), nbytes, N.ptr(do), N.ptr(dht),
                                         N.ptr(dh0), N.ptr(ws), wbytes, st),
                "gdn2_chunk_bwd_state")
    with N.phase("bwd_intra"):
        N.check(lib.gdn2_chunk_bwd_intra(prob, N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(g), N.ptr(b),
                                         N.ptr(w), N.ptr(saved), nbytes, N.ptr(do), N.ptr(dq),
                                         N.ptr(dk), N.ptr(dv), N.ptr(dg), N.ptr(db), N.ptr(dw),
                                         N.ptr(ws), wbytes, st), "gdn2_chunk_bwd_intra")
    if gate is not None:
        return dq, dk, dv, dg, db, dw, dh0, dA_log, ddt_bias
    return dq, dk, dv, dg, db, dw, dh0


def _intermediate_states(saved, tables, B, T, H, K, V, dtype):
    """View the per-chunk entering states kept in ``saved`` as [B, NT, H, K, V]."""
    from .._native import CHUNK

    esize = torch.tensor([], dtype=dtype).element_size()
    nc = tables.n_chunks
    nh = nc * H

    def al(x):
        return (x + 255) & ~255

    off = 0
    for rows in (CHUNK * K, CHUNK * K, CHUNK * K, CHUNK * V, CHUNK * V, CHUNK * CHUNK,
                 CHUNK * CHUNK):
        off = al(off + nh * rows * esize)
    off = al(off + nh * K * 4)
    h = saved[off:off + nh * K * V * esize].view(dtype).view(nc, H, K, V)
    if B > 0 and nc % B == 0:
        h = h.view(B, nc // B, H, K, V)
    return h


class ChunkGDN2Function(torch.autograd.Function):
    """Autograd wrapper around the B200 chunkwise forward/backward.

    Positional arguments after the six token tensors mirror the reference's
    ``ChunkGDN2Function.forward`` (chunk_gdn2.py:2339-2361).  With ``A_log``
    given, ``g`` is the raw gate input and the kernels apply the gate
    (``use_gate_in_kernel``, chunk_gdn2.py:2316-2323); the backward then also
    returns dA_log and d dt_bias.  Otherwise ``g`` is already the log-decay.
    """

    @staticmethod
    def forward(ctx, q, k, v, g, b, w, scale, initial_state, output_final_state,
                use_qk_l2norm_in_kernel, tables, g_dtype, A_log=None, dt_bias=None,
                lower_bound=None):
        gate = GateParams(A_log, dt_bias, lower_bound) if A_log is not None else None
        o, ht, saved = chunk_gdn2_fwd(q, k, v, g, b, w, scale, initial_state,
                                      output_final_state, tables, use_qk_l2norm_in_kernel,
                                      gate=gate)
        ctx.save_for_backward(q, k, v, g, b, w, initial_state, saved, A_log, dt_bias)
        ctx.lower_bound = lower_bound
        ctx.scale = scale
        ctx.tables = tables
        ctx.l2 = use_qk_l2norm_in_kernel
        ctx.g_dtype = g_dtype
        if ht is not None:
            return o, ht
        return o, None

    @staticmethod
    def backward(ctx, do, dht):
        q, k, v, g, b, w, h0, saved, A_log, dt_bias = ctx.saved_tensors
        do = do.contiguous()
        if do.dtype != q.dtype:
            do = do.to(q.dtype)
        if dht is not None:
            dht = dht.float().contiguous()
        gate = GateParams(A_log, dt_bias, ctx.lower_bound) if A_log is not None else None
        grads = chunk_gdn2_bwd(q, k, v, g, b, w, saved, do, dht, ctx.scale, h0, ctx.tables,
                               ctx.l2, gate=gate)
        dq, dk, dv, dg, db, dw, dh0 = grads[:7]
        dA_log, ddt_bias = grads[7:] if gate is not None else (None, None)
        # g, A_log and dt_bias entered as fp32 (chunk_gdn2 casts them), so their
        # gradients stay fp32; autograd casts back through that conversion.
        return (dq, dk, dv, dg, db, dw, None, dh0, None, None, None, None, dA_log, ddt_bias,
                None)


def chunk_gdn2(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor,
    b: torch.Tensor,
    w: torch.Tensor,
    scale: float | None = None,
    initial_state: torch.Tensor | None = None,
    output_final_state: bool = False,
    use_qk_l2norm_in_kernel: bool = False,
    use_gate_in_kernel: bool = False,
    cu_seqlens: torch.LongTensor | None = None,
    cu_seqlens_cpu: torch.LongTensor | None = None,
    safe_gate: bool = False,
    lower_bound: float | None = None,
    disable_recompute: bool = False,
    return_intermediate_states: bool = False,
    transpose_state_layout: bool = False,
    **kwargs,
):
    r"""Chunkwise GDN-2 (Gated DeltaNet 2), ``S_t = (I - k_t (b_t*k_t)^T) Diag(e^{g_t}) S_{t-1}
    + k_t (w_t*v_t)^T``, ``o_t = S_t^T q_t * scale``.

    Args (as in the reference, chunk_gdn2.py:1290-1349):
        q, k: ``[B, T, H, K]``; v: ``[B, T, H, V]``.
        g: log-space decay ``[B, T, H, K]`` (or the raw pre-activation when
            ``use_gate_in_kernel``, then ``-exp(A_log) * softplus(g + dt_bias)``,
            or ``lower_bound * sigmoid(exp(A_log) * g)`` with ``safe_gate``).
        b: channel-wise erase gate ``[B, T, H, K]``; w: write gate ``[B, T, H, V]``.
        scale: defaults to ``K ** -0.5``.
        initial_state: fp32 ``[N, H, K, V]`` (``[N, H, V, K]`` if
            ``transpose_state_layout``).
        cu_seqlens: ``[N+1]`` packed offsets; batch size must then be 1.
        disable_recompute: accepted for API compatibility; the B200 forward
            always keeps the per-chunk intermediates for the backward.
        return_intermediate_states: also return the per-chunk entering states
            ``[B, NT, H, K, V]`` (inference mode only).

    Returns ``(o, final_state)`` or ``(o, final_state, h)``.
    """
    if cu_seqlens is not None:
        if q.shape[0] != 1:
            raise ValueError(
                f"The batch size is expected to be 1 rather than {q.shape[0]} "
                f"when using `cu_seqlens`. Please flatten variable-length "
                f"inputs before processing.",
            )
        if initial_state is not None and initial_state.shape[0] != len(cu_seqlens) - 1:
            raise ValueError(
                f"The number of initial states is expected to be equal to the "
                f"number of input sequences, i.e., {len(cu_seqlens) - 1} rather "
                f"than {initial_state.shape[0]}.",
            )
    if initial_state is not None:
        assert initial_state.dtype == torch.float32, "initial_state must be in float32."

    if safe_gate and use_gate_in_kernel:
        if lower_bound is None:
            raise ValueError(
                "`lower_bound` must be specified when `safe_gate=True` and "
                "`use_gate_in_kernel=True`.")
        if not (-5 <= lower_bound < 0):
            raise ValueError(f"`lower_bound` must be in the safe range [-5, 0), got {lower_bound}.")

    assert q.shape == k.shape == g.shape, "q, k, g must have the same shape."
    assert k.shape[-1] <= 256, "Currently we only support key headdim <=256 for GDN-2 :-("
    assert b.shape == q.shape, (
        "b (channel-wise erase gate) must have shape [B, T, H, K] matching q; "
        f"got {tuple(b.shape)} vs q {tuple(q.shape)}.")
    assert w.shape == v.shape, (
        "w (channel-wise write gate) must have shape [B, T, H, V] matching v; "
        f"got {tuple(w.shape)} vs v {tuple(v.shape)}.")
    assert v.shape == (*q.shape[:3], v.shape[-1]), (
        "v must be of shape (batch size, seq len, num of head, head dim).")
    _require_cuda(q, k, v, g, b, w, initial_state)
    if return_intermediate_states:
        assert torch.is_inference_mode_enabled(), (
            "return_intermediate_states is only allowed in inference mode")

    if scale is None:
        scale = k.shape[-1] ** -0.5

    B, T, H, K = q.shape
    A32 = dt32 = lb = None
    if use_gate_in_kernel:
        assert "A_log" in kwargs, "A_log must be provided when use_gate_in_kernel=True."
        A_log, dt_bias = kwargs["A_log"], kwargs.get("dt_bias")
        lb = lower_bound if safe_gate else None
        if _gate_in_kernel_ok(q.dtype, K, v.shape[-1]):
            A32 = A_log.float().reshape(H).contiguous()
            dt32 = dt_bias.float().reshape(H * K).contiguous() if dt_bias is not None else None
        else:
            g = _gate(g, A_log, dt_bias, lb)
    dt = q.dtype
    g_dtype = g.dtype
    q, k, v, b, w = (x.to(dt).contiguous() for x in (q, k, v, b, w))
    g = g.float().contiguous()
    h0 = initial_state
    if h0 is not None and transpose_state_layout:
        h0 = h0.transpose(-1, -2)
    if h0 is not None:
        h0 = h0.contiguous()
    with torch.cuda.device(q.device):
        tables = N.seq_tables(B, T, q.device, cu_seqlens, cu_seqlens_cpu)
        if cu_seqlens is not None and tables.total > T:
            raise ValueError(f"cu_seqlens[-1]={tables.total} exceeds the sequence length {T}")
        if return_intermediate_states:
            gate = GateParams(A32, dt32, lb) if A32 is not None else None
            o, ht, saved = chunk_gdn2_fwd(q, k, v, g, b, w, scale, h0, output_final_state,
                                          tables, use_qk_l2norm_in_kernel, gate=gate)
            hs = _intermediate_states(saved, tables, B, T, H, K, v.shape[-1], dt)
            if ht is not None and transpose_state_layout:
                ht = ht.transpose(-1, -2)
            return o, ht, hs
        from .cp import CPChunkGDN2Function, sub_spans_single
        from .overlap import OverlapChunkGDN2Function, overlap_pieces

        V = v.shape[-1]
        pieces = overlap_pieces(B, T, H, K, V, dt, q.device) if cu_seqlens is None else 1
        if (cu_seqlens is None and A32 is None and sub_spans_single(B, T, H, K, V, dt) > 1):
            # few sequence-heads over long sequences: the sub-span pre-scan,
            # the unfold of the start states and S-fold shorter state passes
            o, ht = CPChunkGDN2Function.apply(q, k, v, g, b, w, h0, scale,
                                              use_qk_l2norm_in_kernel, 0, 1, None)
            if not output_final_state:
                ht = None
        elif pieces > 1:
            # one long sequence, a few dozen heads: the state passes of the
            # sequence's pieces overlap the intra-chunk kernels of their
            # neighbours on a second stream
            o, ht = OverlapChunkGDN2Function.apply(q, k, v, g, b, w, scale, h0,
                                                   output_final_state, use_qk_l2norm_in_kernel,
                                                   pieces, A32, dt32, lb)
        else:
            o, ht = ChunkGDN2Function.apply(q, k, v, g, b, w, scale, h0, output_final_state,
                                            use_qk_l2norm_in_kernel, tables, g_dtype, A32, dt32,
                                            lb)
    if ht is not None and transpose_state_layout:
        ht = ht.transpose(-1, -2)
    return o, ht


def _gate(g, A_log, dt_bias, lower_bound):
    """Gate activation of the reference's gate-in-kernel path
    (``kda_gate_chunk_cumsum`` / fused_recurrent_gdn2.py:257-272):
    ``-exp(A_log) * softplus(g + dt_bias)`` or, with a lower bound,
    ``lower_bound * sigmoid(exp(A_log) * (g + dt_bias))``.  Computed with
    device-side torch ops so autograd yields dA_log and d dt_bias."""
    H, K = g.shape[-2], g.shape[-1]
    x = g.float()
    if dt_bias is not None:
        x = x + dt_bias.float().view(H, K)
    a = A_log.float().exp().view(H, 1)
    if lower_bound is not None:
        return lower_bound * torch.sigmoid(a * x)
    return -a * torch.nn.functional.softplus(x)

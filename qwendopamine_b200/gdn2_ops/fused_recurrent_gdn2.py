"""Token-serial GDN-2 forward (decode) on B200 -- drop-in for the reference's
``qwendopamine.models.gdn2.gdn2_ops.fused_recurrent_gdn2``.

``fused_recurrent_gdn2`` and ``fused_recurrent_gdn2_fwd`` keep the reference's
signatures and semantics (fused_recurrent_gdn2.py:344-555): fp32 state
``[N, HV, K, V]`` (``[N, HV, V, K]`` with ``transpose_state_layout``), grouped
value heads (HV a multiple of H), packed sequences through ``cu_seqlens``,
state pools through ``ssm_state_indices`` with an in-place update,
speculative decoding (2-D ``ssm_state_indices`` with ``num_accepted_tokens``:
start from slot ``indices[n, accepted[n]-1]`` and write the state after token
``t`` to slot ``indices[n, t]``, reference :217-226, :311-324), and an
optional preallocated ``out``.  The work is one launch of
``gdn2_recurrent_fwd`` from ``libgdn2_b200.so``; there is no CPU path.
"""

from __future__ import annotations

import torch

from .. import _native as N

__all__ = ["fused_recurrent_gdn2", "fused_recurrent_gdn2_fwd"]


def fused_recurrent_gdn2_fwd(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor,
    b: torch.Tensor,
    w: torch.Tensor,
    A_log: torch.Tensor | None = None,
    dt_bias: torch.Tensor | None = None,
    initial_state: torch.Tensor | None = None,
    scale: float | None = None,
    output_final_state: bool = False,
    inplace_final_state: bool = True,
    cu_seqlens: torch.LongTensor | None = None,
    ssm_state_indices: torch.Tensor | None = None,
    num_accepted_tokens: torch.Tensor | None = None,
    use_qk_l2norm_in_kernel: bool = False,
    use_gate_in_kernel: bool = False,
    lower_bound: float | None = None,
    out: torch.Tensor | None = None,
    transpose_state_layout: bool = False,
    **kwargs,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Allocate buffers and launch the recurrent forward (reference :344-458).

    ``inplace_final_state`` writes the final state back into ``initial_state``
    (indexed through ``ssm_state_indices`` when given); ``output_final_state``
    instead returns a fresh fp32 buffer.
    """
    for t in (q, k, v, g, b, w, initial_state):
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "fused_recurrent_gdn2: inputs must be CUDA tensors -- the B200 build has no "
                "CPU path")
    spec = ssm_state_indices is not None and ssm_state_indices.ndim == 2
    if num_accepted_tokens is not None and not spec:
        raise ValueError(
            "fused_recurrent_gdn2_fwd: num_accepted_tokens needs 2-D ssm_state_indices")
    if spec and not inplace_final_state:
        raise NotImplementedError(
            "fused_recurrent_gdn2_fwd: 2-D ssm_state_indices are served in place (the state "
            "after each token goes to its pool slot); inplace_final_state=False is not "
            "supported with them")
    if spec and transpose_state_layout:
        raise NotImplementedError(
            "fused_recurrent_gdn2_fwd: 2-D ssm_state_indices with transpose_state_layout")
    if scale is None:
        scale = k.shape[-1] ** -0.5
    gate, A32, dt32 = 0, None, None
    if use_gate_in_kernel:
        # fused in the kernel, indexed by key head as the reference does
        # (fused_recurrent_gdn2.py:257-272)
        if A_log is None:
            raise ValueError("A_log must be provided when use_gate_in_kernel=True.")
        gate = 2 if lower_bound is not None else 1
        A32 = A_log.to(device=q.device, dtype=torch.float32).contiguous()
        if A32.numel() < k.shape[2]:
            raise ValueError(f"A_log needs one entry per key head ({k.shape[2]}); "
                             f"got {A32.numel()}")
        if dt_bias is not None:
            dt32 = dt_bias.to(device=q.device, dtype=torch.float32).contiguous()
            if dt32.numel() < k.shape[2] * k.shape[-1]:
                raise ValueError("dt_bias needs H*K entries")

    B, T, H, K = k.shape
    HV, V = v.shape[2], v.shape[-1]
    Nseq = B if cu_seqlens is None else len(cu_seqlens) - 1
    dt = q.dtype
    q, k, v, b, w = (x.to(dt).contiguous() for x in (q, k, v, b, w))
    g = g.float().contiguous()

    if out is None:
        # zeros, as the reference allocates them: the kernel skips the tokens
        # of sequences whose state slot is negative (padding in a pool)
        out = torch.zeros_like(v)
    else:
        assert out.shape == v.shape
    h0 = initial_state
    if h0 is not None and transpose_state_layout:
        h0 = h0.transpose(-1, -2).contiguous()
    elif h0 is not None and not h0.is_contiguous():
        h0 = h0.contiguous()
    if inplace_final_state:
        assert initial_state is not None, "inplace_final_state=True requires an initial_state"
        final_state = h0
    elif output_final_state:
        final_state = q.new_empty(Nseq, HV, K, V, dtype=torch.float32)
    else:
        final_state = None
    if h0 is not None:
        assert h0.dtype == torch.float32, "initial_state must be in float32."

    cu32 = None
    if cu_seqlens is not None:
        cu32 = cu_seqlens.to(device=q.device, dtype=torch.int32).contiguous()
    idx32 = None
    stride = 0
    idx_stride = 0
    nat32 = None
    if ssm_state_indices is not None:
        idx32 = ssm_state_indices.to(device=q.device, dtype=torch.int32).contiguous()
        stride = h0.stride(0) if h0 is not None else HV * K * V
        if spec:
            idx_stride = idx32.shape[1]
        if num_accepted_tokens is not None:
            nat32 = num_accepted_tokens.to(device=q.device, dtype=torch.int32).contiguous()
    lib = N.load()
    prob = N.RecurrentProblem(B, T, H, HV, K, V, N.dtype_code(dt),
                              int(bool(use_qk_l2norm_in_kernel)), float(scale), Nseq,
                              N.ptr(cu32), N.ptr(idx32), stride, idx_stride, N.ptr(nat32),
                              N.ptr(A32), N.ptr(dt32), gate,
                              float(lower_bound) if lower_bound is not None else 0.0)
    with torch.cuda.device(q.device):
        N.check(lib.gdn2_recurrent_fwd(prob, N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(g), N.ptr(b),
                                       N.ptr(w), N.ptr(h0), N.ptr(out), N.ptr(final_state),
                                       N.stream_of(q.device)), "gdn2_recurrent_fwd")
    if final_state is not None and transpose_state_layout:
        if inplace_final_state and initial_state is not None:
            initial_state.copy_(final_state.transpose(-1, -2))
            final_state = initial_state
        else:
            final_state = final_state.transpose(-1, -2)
    elif inplace_final_state and final_state is not initial_state and initial_state is not None:
        initial_state.copy_(final_state)
        final_state = initial_state
    return out, final_state


def fused_recurrent_gdn2(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor,
    b: torch.Tensor,
    w: torch.Tensor,
    A_log: torch.Tensor | None = None,
    dt_bias: torch.Tensor | None = None,
    scale: float | None = None,
    initial_state: torch.Tensor = None,
    output_final_state: bool = False,
    use_qk_l2norm_in_kernel: bool = False,
    use_gate_in_kernel: bool = False,
    lower_bound: float | None = None,
    cu_seqlens: torch.LongTensor | None = None,
    transpose_state_layout: bool = False,
    **kwargs,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    r"""Token-by-token GDN-2 forward (inference only), reference :461-555.

    q, k: ``[B, T, H, K]``; v, w: ``[B, T, HV, V]``; g, b: ``[B, T, HV, K]``;
    initial_state: fp32 ``[N, HV, K, V]``.  Returns ``(o, final_state)``.
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
    assert b.shape == (*q.shape[:3], k.shape[-1]) or b.shape == (*v.shape[:3], k.shape[-1]), (
        f"b must have shape [B, T, HV, K]; got {tuple(b.shape)}.")
    assert w.shape == v.shape, (
        f"w must have shape [B, T, HV, V] matching v; got {tuple(w.shape)} "
        f"vs v {tuple(v.shape)}.")
    if scale is None:
        scale = k.shape[-1] ** -0.5
    return fused_recurrent_gdn2_fwd(
        q=q, k=k, v=v, g=g, b=b, w=w, A_log=A_log, dt_bias=dt_bias, scale=scale,
        initial_state=initial_state, inplace_final_state=False,
        output_final_state=output_final_state, use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel,
        use_gate_in_kernel=use_gate_in_kernel, lower_bound=lower_bound, cu_seqlens=cu_seqlens,
        transpose_state_layout=transpose_state_layout)

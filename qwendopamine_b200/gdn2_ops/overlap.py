"""Chunkwise GDN-2 for one long sequence with a few dozen heads: the state
passes overlapped with the intra-chunk kernels on a second stream.

No counterpart in the reference (its ``chunk_gdn2``, ``chunk_gdn2.py:1267-1434``,
runs the phases one after another on one stream).  With B = 1 and 2H SMs or
fewer, the state passes (``gdn2_chunk_fwd_state`` / ``gdn2_chunk_bwd_state``:
one CTA per head and half of the value columns) walk every chunk of the
sequence on 2H SMs and leave the rest of the GPU idle for the length of that
walk.  Here the sequence is cut into P pieces of whole 64-token chunks, each
an independent problem with its own saved buffer and workspace, and:

forward:  intra(0) on the whole GPU; then, on the side stream (high priority),
          state(p) from the end state of piece p-1 as soon as intra(p) is
          done, while intra(p+1) runs on the main stream with its persistent
          grid capped at the SMs the state pass leaves (``max_ctas``);
backward: on the side stream state(P-1), ..., state(0), each from the start-
          state gradient of the piece after it; on the main stream intra(p)
          as soon as state(p) is done, filling whatever SMs the state pass
          leaves.

Beside the intra kernels the state passes may run at full width (H CTAs, a
longer chain) rather than in value halves (2H CTAs), and a state pass that
runs alone (the backward's first, the forward's once every intra kernel is
done) takes the faster value halves.  A small cost model from measured
per-chunk costs makes both choices.  With 32 heads over 4,096 chunks the
forward runs its first pieces at full width and its last ones in halves,
the backward at full width (one B200: 41.4 ms per forward + backward on one
stream, 36.4 ms overlapped in value halves, 33.4 ms at full width, 32.7 ms
with the planned widths); with 16 heads the forward keeps the value halves,
whose shorter chain is then the limit (21.0 against 28.4 ms on one stream).

The kernels, their per-chunk work and the fp32 state handed from piece to
piece are those of the one-stream path; at the one-stream path's width the
results are the same bit for bit (at full width the state products are
summed in another order).  The main stream waits for the side stream before
either direction returns.
"""

from __future__ import annotations

import torch

from .. import _native as N
from .chunk_gdn2 import GateParams, _aligned16, _problem

__all__ = ["OverlapChunkGDN2Function", "overlap_pieces"]

# Pieces hold at least this many chunks (a piece boundary costs a state-pass
# launch and a few microseconds of refill), at most MAX_PIECES of them.
MIN_PIECE_CHUNKS = 256
MAX_PIECES = 16
# SMs the intra kernels keep at the least while a state pass runs beside them.
MIN_FREE_SMS = 32
# State-pass width beside the intra kernels, per direction: the full-width
# pass (one CTA per head walking all value columns: a slower chain that
# leaves H more SMs to the intra kernels), the value-half pass (two CTAs per
# head), or None: whichever of the two the cost model below expects to end
# the direction sooner.
FULL_WIDTH = {"fwd": None, "bwd": None}
# Cost model, from CUDA-event timings on B200 at K = V = 128, bf16, 4,096
# chunks x 32 heads: the state pass's chain per chunk (ms) at full width /
# in value halves, and the intra kernels' SM-milliseconds per chunk-head.
CHAIN_MS = {("fwd", True): 2.86e-3, ("fwd", False): 2.00e-3,
            ("bwd", True): 2.33e-3, ("bwd", False): 1.98e-3}
INTRA_SM_MS = {"fwd": 8.86e-3, "bwd": 2.04e-2}

_side_streams: dict = {}


def _sm_count(device) -> int:
    return torch.cuda.get_device_properties(device).multi_processor_count


def _side_stream(device) -> torch.cuda.Stream:
    """One high-priority stream per device for the state passes: their CTAs
    are placed before pending intra-kernel CTAs as SMs free up."""
    key = str(device)
    s = _side_streams.get(key)
    if s is None:
        hi = torch.cuda.Stream.priority_range()[1]
        s = torch.cuda.Stream(device=device, priority=hi)
        _side_streams[key] = s
    return s


def estimate_ms(direction: str, full: bool, nch: int, H: int, sms: int) -> float:
    """Expected time of one direction over nch chunks x H heads: the state
    chain, or the intra kernels' work on the SMs the chain leaves them (the
    forward's persistent grid is capped at those SMs for the whole
    direction; the backward's CTAs also take the chain's SMs once it ends),
    whichever is longer."""
    ctas = H if full else 2 * H
    chain = nch * CHAIN_MS[(direction, full)]
    work = nch * H * INTRA_SM_MS[direction]
    if direction == "fwd":
        return max(chain, work / (sms - ctas))
    return max(chain, (work + chain * ctas) / sms)


def full_width(direction: str, nch: int, H: int, sms: int) -> bool:
    """Whether ``direction``'s state passes run at full width (else in value
    halves) beside the intra kernels."""
    forced = FULL_WIDTH[direction]
    if forced is not None:
        return forced
    if sms - 2 * H < MIN_FREE_SMS:
        return True
    return estimate_ms(direction, True, nch, H, sms) < estimate_ms(direction, False, nch, H, sms)


def _state_ctas(direction: str, nch: int, H: int, sms: int) -> int:
    return H if full_width(direction, nch, H, sms) else 2 * H


def _model_fwd(ns, H: int, sms: int, j: int) -> float:
    """Modelled forward time (ms) over pieces of ``ns`` chunks when the first
    ``j`` state passes run at full width beside the intra kernels and the
    rest in value halves: with j = 0 every pass runs in halves beside the
    intra kernels, otherwise the half-width passes wait for the last intra
    kernel and have the GPU to themselves."""
    cap = sms - (H if j > 0 else 2 * H)
    t, ends = 0.0, []
    for p, n in enumerate(ns):
        t += n * H * INTRA_SM_MS["fwd"] / (sms if p == 0 else cap)
        ends.append(t)
    side = 0.0
    for p, n in enumerate(ns):
        full = p < j
        ready = ends[p] if (full or j == 0) else ends[-1]
        side = max(side, ready) + n * CHAIN_MS[("fwd", full)]
    return max(t, side)


def forward_plan(ns, H: int, sms: int) -> int:
    """How many leading pieces' forward state passes run at full width (the
    others in value halves; see :func:`_model_fwd`): all of them or none when
    FULL_WIDTH forces it, else the count the model expects to end soonest
    among those that leave MIN_FREE_SMS SMs to the intra kernels."""
    P = len(ns)
    forced = FULL_WIDTH["fwd"]
    if forced is not None:
        return P if forced else 0
    cands = [j for j in range(P + 1) if sms - (H if j > 0 else 2 * H) >= MIN_FREE_SMS]
    return min(cands, key=lambda j: _model_fwd(ns, H, sms, j))


def _piece_chunks(T: int, P: int):
    cuts = _cuts(T, P)
    return [(cuts[p + 1] + N.CHUNK - 1) // N.CHUNK - cuts[p] // N.CHUNK for p in range(P)]


def overlap_pieces(B, T, H, K, V, dtype, device) -> int:
    """Pieces for the overlapped path (1: not used).  Used for one fixed-length
    bf16 sequence with K = V = 128 whose state passes leave at least
    MIN_FREE_SMS SMs to the intra kernels in both directions and which is
    long enough for two pieces of MIN_PIECE_CHUNKS chunks."""
    if B != 1 or dtype != torch.bfloat16 or K != 128 or V != 128:
        return 1
    sms = _sm_count(device)
    nch = (T + N.CHUNK - 1) // N.CHUNK
    if sms - _state_ctas("bwd", nch, H, sms) < MIN_FREE_SMS:
        return 1
    if sms - (2 * H if FULL_WIDTH["fwd"] is False else H) < MIN_FREE_SMS:
        return 1
    P = min(MAX_PIECES, nch // MIN_PIECE_CHUNKS)
    return P if P >= 2 else 1


def _cuts(T: int, P: int):
    nch = (T + N.CHUNK - 1) // N.CHUNK
    return [min(T, N.CHUNK * (nch * j // P)) for j in range(P)] + [T]


def _al(x: int) -> int:
    return (x + 255) & ~255


class _Pieces:
    """Per-piece problems and the byte offsets of their saved buffers and
    backward workspaces inside one allocation each."""

    def __init__(self, lib, T, P, H, K, V, dtype, l2, scale, gate, device,
                 dA_log=None, ddt_bias=None):
        self.cuts = _cuts(T, P)
        self.probs, self.tabs = [], []
        self.sb, self.so, self.wb, self.wo = [], [], [], []
        s_tot = w_tot = 0
        for p in range(P):
            tab = N.seq_tables(1, self.cuts[p + 1] - self.cuts[p], device)
            prob = _problem(H, K, V, dtype, l2, scale, tab, gate, dA_log, ddt_bias)
            nb = lib.gdn2_chunk_saved_bytes(prob)
            wb = lib.gdn2_chunk_bwd_workspace_bytes(prob)
            if nb == 0 or wb == 0:
                N.check(N.ERR_INVALID, "gdn2_chunk_saved_bytes")
            self.probs.append(prob)
            self.tabs.append(tab)  # keeps the device tables alive
            self.sb.append(nb)
            self.so.append(s_tot)
            self.wb.append(wb)
            self.wo.append(w_tot)
            s_tot += _al(nb)
            w_tot += _al(wb)
        self.saved_total, self.ws_total = s_tot, w_tot

    def rows(self, x, p):
        """Piece p's rows of a [1, T, H, D] tensor (a contiguous view)."""
        return x[:, self.cuts[p]:self.cuts[p + 1]]


def _fwd(q, k, v, g, b, w, scale, h0, want_ht, l2, gate, P):
    lib = N.load()
    dev = q.device
    _, T, H, K = q.shape
    V = v.shape[-1]
    pc = _Pieces(lib, T, P, H, K, V, q.dtype, l2, scale, gate, dev)
    saved = torch.empty(pc.saved_total, dtype=torch.uint8, device=dev)
    o = torch.empty_like(v)
    carry = torch.empty(max(P - 1, 1), 1, H, K, V, dtype=torch.float32, device=dev)
    ht = q.new_empty(1, H, K, V, dtype=torch.float32) if want_ht else None
    main, side = torch.cuda.current_stream(dev), _side_stream(dev)
    sms = _sm_count(dev)
    j = forward_plan(_piece_chunks(T, P), H, sms)
    cap = sms - (H if j > 0 else 2 * H)
    side.wait_stream(main)
    ms, ss = N.c_void_p(main.cuda_stream), N.c_void_p(side.cuda_stream)
    done = []  # per piece: an event after its intra kernel
    for p in range(P):
        prob = pc.probs[p]
        prob.max_ctas = 0 if p == 0 else cap
        with N.phase("fwd_intra", main):
            N.check(lib.gdn2_chunk_fwd_intra(prob, *(N.ptr(pc.rows(t, p)) for t in (q, k, v, g, b, w)),
                                             N.c_void_p(saved.data_ptr() + pc.so[p]), pc.sb[p], ms),
                    "gdn2_chunk_fwd_intra")
        done.append(torch.cuda.Event())
        done[-1].record(main)
    for p in range(P):
        prob = pc.probs[p]
        full = p < j
        # a half-width pass after full-width ones waits for every intra
        # kernel: it then has the GPU to itself
        side.wait_event(done[p] if (full or j == 0) else done[-1])
        h_in = h0 if p == 0 else carry[p - 1]
        h_out = carry[p] if p < P - 1 else ht
        prob.max_ctas = H if full else 2 * H
        with N.phase("fwd_state", side):
            N.check(lib.gdn2_chunk_fwd_state(prob, N.ptr(h_in), N.ptr(pc.rows(o, p)), N.ptr(h_out),
                                             N.c_void_p(saved.data_ptr() + pc.so[p]), pc.sb[p], ss),
                    "gdn2_chunk_fwd_state")
    main.wait_stream(side)
    return o, ht, saved, pc


def _bwd(q, k, v, g, b, w, saved, pc, do, dht, h0, gate):
    lib = N.load()
    dev = q.device
    _, T, H, K = q.shape
    V = v.shape[-1]
    P = len(pc.probs)
    dA_log = ddt_bias = None
    if gate is not None:
        dA_log = torch.zeros(H, dtype=torch.float32, device=dev)
        if gate.dt_bias is not None:
            ddt_bias = torch.zeros(H * K, dtype=torch.float32, device=dev)
        for prob in pc.probs:
            prob.dA_log, prob.ddt_bias = N.ptr(dA_log), N.ptr(ddt_bias)
    ws = torch.empty(pc.ws_total, dtype=torch.uint8, device=dev)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    db, dw, dg = torch.empty_like(b), torch.empty_like(w), torch.empty_like(g)
    dh0 = torch.empty_like(h0) if h0 is not None else None
    dcarry = torch.empty(max(P - 1, 1), 1, H, K, V, dtype=torch.float32, device=dev)
    main, side = torch.cuda.current_stream(dev), _side_stream(dev)
    state_ctas = _state_ctas("bwd", (T + N.CHUNK - 1) // N.CHUNK, H, _sm_count(dev))
    # the last piece's pass runs before any intra kernel can: in value halves
    # unless a width is forced
    first_ctas = 2 * H if FULL_WIDTH["bwd"] is None else state_ctas
    side.wait_stream(main)
    ms, ss = N.c_void_p(main.cuda_stream), N.c_void_p(side.cuda_stream)
    for p in reversed(range(P)):
        prob = pc.probs[p]
        sv = N.c_void_p(saved.data_ptr() + pc.so[p])
        wv = N.c_void_p(ws.data_ptr() + pc.wo[p])
        d_end = dht if p == P - 1 else dcarry[p]
        d_start = dh0 if p == 0 else dcarry[p - 1]
        prob.max_ctas = first_ctas if p == P - 1 else state_ctas
        with N.phase("bwd_state", side):
            N.check(lib.gdn2_chunk_bwd_state(prob, sv, pc.sb[p], N.ptr(pc.rows(do, p)), N.ptr(d_end),
                                             N.ptr(d_start), wv, pc.wb[p], ss),
                    "gdn2_chunk_bwd_state")
        main.wait_stream(side)
        with N.phase("bwd_intra", main):
            N.check(lib.gdn2_chunk_bwd_intra(prob, *(N.ptr(pc.rows(t, p)) for t in (q, k, v, g, b, w)),
                                             sv, pc.sb[p], N.ptr(pc.rows(do, p)),
                                             *(N.ptr(pc.rows(t, p)) for t in (dq, dk, dv, dg, db, dw)),
                                             wv, pc.wb[p], ms), "gdn2_chunk_bwd_intra")
    return dq, dk, dv, dg, db, dw, dh0, dA_log, ddt_bias


class OverlapChunkGDN2Function(torch.autograd.Function):
    """Autograd wrapper of the overlapped path; arguments as
    :class:`~qwendopamine_b200.gdn2_ops.chunk_gdn2.ChunkGDN2Function` (B = 1,
    fixed length) plus the number of pieces."""

    @staticmethod
    def forward(ctx, q, k, v, g, b, w, scale, initial_state, output_final_state,
                use_qk_l2norm_in_kernel, pieces, A_log=None, dt_bias=None, lower_bound=None):
        gate = GateParams(A_log, dt_bias, lower_bound) if A_log is not None else None
        q, k, v, g, b, w = _aligned16(q, k, v, g, b, w)
        o, ht, saved, pc = _fwd(q, k, v, g, b, w, scale, initial_state, output_final_state,
                                use_qk_l2norm_in_kernel, gate, pieces)
        ctx.save_for_backward(q, k, v, g, b, w, initial_state, saved, A_log, dt_bias)
        ctx.pc = pc
        ctx.lower_bound = lower_bound
        return o, ht

    @staticmethod
    def backward(ctx, do, dht):
        q, k, v, g, b, w, h0, saved, A_log, dt_bias = ctx.saved_tensors
        do = do.contiguous()
        if do.dtype != q.dtype:
            do = do.to(q.dtype)
        (do,) = _aligned16(do)
        if dht is not None:
            dht = dht.float().contiguous()
        gate = GateParams(A_log, dt_bias, ctx.lower_bound) if A_log is not None else None
        dq, dk, dv, dg, db, dw, dh0, dA_log, ddt_bias = _bwd(q, k, v, g, b, w, saved, ctx.pc, do,
                                                             dht, h0, gate)
        return (dq, dk, dv, dg, db, dw, None, dh0, None, None, None, dA_log, ddt_bias, None)

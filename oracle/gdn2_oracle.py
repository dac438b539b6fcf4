"""CPU oracle for the GDN-2 core recurrence -- TEST INFRASTRUCTURE ONLY.

This module is a checker. Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it. The
product path (``qwendopamine_b200``) never calls it and raises when its CUDA
library is missing.

It restates, in float64 numpy, the reference's pure-PyTorch GDN-2 maths from
Gabz4200/QwenDopamine ``src/qwendopamine/models/gdn2/gdn2.py``:

* :func:`recurrent_fwd` follows ``torch_recurrent_gdn2`` (gdn2.py:100-184):
  F.normalize(eps=1e-6) on q and k, ``q *= K**-0.5``, then per token
  decay -> erase-read -> write -> read-out *after* the update.
* :func:`recurrent_bwd` is the hand-derived reverse pass of that token loop
  (the reference obtains the same numbers through torch autograd; the golden
  fixtures in ``tests/golden`` pin this function to the reference's autograd).
* :func:`chunk_fwd_absolute` follows ``torch_chunk_gdn2`` (gdn2.py:243-369),
  including its absolute-gamma normalisation ``kbar = k / clamp(gamma, 1e-12)``,
  which underflows once a chunk's cumulative decay passes about -27.6.
* :func:`chunk_fwd_relative` is the chunkwise WY form the CUDA kernels use
  (relative decays ``exp(G_r - G_i)`` as in the Triton path,
  ``chunk_gdn2.py:584-589``).  It returns every per-chunk intermediate so a GPU
  test can localise a mismatch to one stage.

Parity pin: ``tests/golden/make_golden.py`` imports the reference (this
container only) and records its outputs, final states and autograd gradients;
``tests/test_oracle.py`` checks these functions against those fixtures.
"""

from __future__ import annotations

import numpy as np

NORM_EPS = 1e-6


# ----------------------------------------------------------------------------
# helpers
# ----------------------------------------------------------------------------

def _f64(x):
    return None if x is None else np.asarray(x, dtype=np.float64)


def _normalize(x, eps=NORM_EPS, mode="torch"):
    """Row L2 normalisation along the last axis.

    mode="torch": ``x / max(||x||, eps)`` (F.normalize, gdn2.py:142-143).
    mode="fla":   ``x / sqrt(sum(x^2) + eps)`` (FLA ``l2norm_fwd`` used by the
                  Triton path, chunk_gdn2.py:2366-2368).
    """
    ss = np.sum(x * x, axis=-1, keepdims=True)
    if mode == "torch":
        den = np.maximum(np.sqrt(ss), eps)
    else:
        den = np.sqrt(ss + eps)
    return x / den, den


def _normalize_bwd(y, den, dy, eps=NORM_EPS, mode="torch"):
    """Backward of :func:`_normalize` given its output ``y`` and denominator."""
    proj = np.sum(y * dy, axis=-1, keepdims=True)
    if mode == "torch":
        # Where the clamp is active the denominator is a constant.
        active = den > eps
        return np.where(active, (dy - y * proj) / den, dy / den)
    # d/dx [x / sqrt(|x|^2+eps)] = (dy - y * <y,dy>) / den
    return (dy - y * proj) / den


def _bthd_to_bhtd(x):
    return np.ascontiguousarray(np.transpose(x, (0, 2, 1, 3)))


def _bhtd_to_bthd(x):
    return np.ascontiguousarray(np.transpose(x, (0, 2, 1, 3)))


# ----------------------------------------------------------------------------
# token-serial recurrence (ground truth)
# ----------------------------------------------------------------------------

def recurrent_fwd(q, k, v, g, b, w, initial_state=None, scale=None,
                  use_qk_l2norm=True, norm_mode="torch", return_states=False):
    """Token-serial GDN-2 forward (restates gdn2.py:100-184).

    Args are ``[B,T,H,K]`` (q, k, g, b) and ``[B,T,H,V]`` (v, w); the optional
    ``initial_state`` is ``[B,H,K,V]``.  Returns ``(o [B,T,H,V], S_T [B,H,K,V])``
    in float64; with ``return_states`` also every post-token state
    ``[T+1,B,H,K,V]`` (index 0 = initial state).
    """
    q, k, v, g, b, w = (_f64(x) for x in (q, k, v, g, b, w))
    B, T, H, K = q.shape
    V = v.shape[-1]
    if scale is None:
        scale = K ** -0.5
    if use_qk_l2norm:
        q, _ = _normalize(q, mode=norm_mode)
        k, _ = _normalize(k, mode=norm_mode)
    q = q * scale
    S = np.zeros((B, H, K, V)) if initial_state is None else _f64(initial_state).copy()
    states = [S.copy()] if return_states else None
    o = np.zeros((B, T, H, V))
    eg = np.exp(g)
    for t in range(T):
        # 1. decay along key channels (gdn2.py:165)
        S = S * eg[:, t][..., None]
        # 2. erase-read with the erase gate (gdn2.py:168-169)
        kb = b[:, t] * k[:, t]
        r = np.einsum("bhkv,bhk->bhv", S, kb)
        # 3. delta with the write gate (gdn2.py:172)
        d = w[:, t] * v[:, t] - r
        # 4. rank-1 update (gdn2.py:175)
        S = S + k[:, t][..., None] * d[..., None, :]
        # 5. read-out after the update (gdn2.py:178)
        o[:, t] = np.einsum("bhkv,bhk->bhv", S, q[:, t])
        if return_states:
            states.append(S.copy())
    if return_states:
        return o, S, np.stack(states)
    return o, S


def recurrent_bwd(q, k, v, g, b, w, do, initial_state=None, dht=None,
                  scale=None, use_qk_l2norm=True, norm_mode="torch"):
    """Reverse pass of :func:`recurrent_fwd`.

    Returns ``dq, dk, dv, dg, db, dw, dh0`` (float64), the gradients of
    ``sum(o * do) + sum(S_T * dht)``.  The reference computes these with torch
    autograd through ``torch_recurrent_gdn2``; ``tests/golden`` pins the two.
    """
    q, k, v, g, b, w, do = (_f64(x) for x in (q, k, v, g, b, w, do))
    B, T, H, K = q.shape
    V = v.shape[-1]
    if scale is None:
        scale = K ** -0.5
    qr, kr = q, k
    if use_qk_l2norm:
        qn, qden = _normalize(qr, mode=norm_mode)
        kn, kden = _normalize(kr, mode=norm_mode)
    else:
        qn, kn = qr, kr
    qs = qn * scale
    _, _, states = recurrent_fwd(qn, kn, v, g, b, w, initial_state, scale=1.0,
                                 use_qk_l2norm=False, return_states=True)
    # recurrent_fwd with scale=1.0 on pre-normalised q applies no scaling, so
    # rerun the read-out with the scaled query below via states.
    eg = np.exp(g)
    dS = np.zeros((B, H, K, V)) if dht is None else _f64(dht).copy()
    dqs = np.zeros_like(qs)
    dkn = np.zeros_like(kn)
    dv = np.zeros_like(v)
    dw = np.zeros_like(w)
    db = np.zeros_like(b)
    dg = np.zeros_like(g)
    for t in range(T - 1, -1, -1):
        S_t = states[t + 1]
        S_prev = states[t]
        Sd = S_prev * eg[:, t][..., None]
        kb = b[:, t] * kn[:, t]
        d = w[:, t] * v[:, t] - np.einsum("bhkv,bhk->bhv", Sd, kb)
        # o_t = S_t^T qs_t
        dqs[:, t] = np.einsum("bhkv,bhv->bhk", S_t, do[:, t])
        dS = dS + qs[:, t][..., None] * do[:, t][..., None, :]
        # S_t = Sd + k d^T
        dkn[:, t] += np.einsum("bhkv,bhv->bhk", dS, d)
        dd = np.einsum("bhkv,bhk->bhv", dS, kn[:, t])
        # d = w*v - Sd^T kb
        dv[:, t] = dd * w[:, t]
        dw[:, t] = dd * v[:, t]
        dSd = dS - kb[..., None] * dd[..., None, :]
        dkb = -np.einsum("bhkv,bhv->bhk", Sd, dd)
        db[:, t] = dkb * kn[:, t]
        dkn[:, t] += dkb * b[:, t]
        # Sd = S_prev * exp(g)
        dg[:, t] = np.sum(dSd * Sd, axis=-1)
        dS = dSd * eg[:, t][..., None]
    dqn = dqs * scale
    if use_qk_l2norm:
        dq = _normalize_bwd(qn, qden, dqn, mode=norm_mode)
        dk = _normalize_bwd(kn, kden, dkn, mode=norm_mode)
    else:
        dq, dk = dqn, dkn
    return dq, dk, dv, dg, db, dw, dS


# ----------------------------------------------------------------------------
# chunkwise forms
# ----------------------------------------------------------------------------

def _solve_unit_lower(L, rhs):
    """Solve (I + L) X = rhs for strictly-lower L by forward substitution."""
    C = L.shape[-1]
    X = np.array(rhs, dtype=np.float64, copy=True)
    for r in range(C):
        if r:
            X[..., r, :] -= np.einsum("...i,...id->...d", L[..., r, :r], X[..., :r, :])
    return X


def chunk_fwd_absolute(q, k, v, g, b, w, initial_state=None, scale=None,
                       use_qk_l2norm=True, chunk_size=64):
    """Restates ``torch_chunk_gdn2`` (gdn2.py:243-369), absolute-gamma WY form.

    Kept to pin the reference's own fast oracle (and to reproduce its
    underflow under strong decay); the CUDA kernels follow
    :func:`chunk_fwd_relative` instead.
    """
    q, k, v, g, b, w = (_f64(x) for x in (q, k, v, g, b, w))
    B, T, H, K = q.shape
    V = v.shape[-1]
    if scale is None:
        scale = K ** -0.5
    if use_qk_l2norm:
        q, _ = _normalize(q)
        k, _ = _normalize(k)
    q = _bthd_to_bhtd(q * scale)
    k, v, g, b, w = (_bthd_to_bhtd(x) for x in (k, v, g, b, w))
    S = np.zeros((B, H, K, V)) if initial_state is None else _f64(initial_state).copy()
    outs = []
    for s in range(0, T, chunk_size):
        e = min(s + chunk_size, T)
        qc, kc, vc, gc, bc, wc = (x[:, :, s:e] for x in (q, k, v, g, b, w))
        gamma = np.exp(np.cumsum(gc, axis=2))
        gl = gamma[:, :, -1:, :]
        kbar = kc / np.maximum(gamma, 1e-12)
        ebar = gamma * (bc * kc)
        z = wc * vc
        Tm = np.tril(ebar @ np.swapaxes(kbar, -1, -2), -1)
        Y = _solve_unit_lower(Tm, ebar)
        U = _solve_unit_lower(Tm, z)
        delta = U - Y @ S
        qg = gamma * qc
        aqk = np.tril(qg @ np.swapaxes(kbar, -1, -2))
        outs.append(qg @ S + aqk @ delta)
        S = np.swapaxes(gl, -1, -2) * (S + np.swapaxes(kbar, -1, -2) @ delta)
    o = _bhtd_to_bthd(np.concatenate(outs, axis=2))
    return o, S


def chunk_fwd_relative(q, k, v, g, b, w, initial_state=None, scale=None,
                       use_qk_l2norm=True, chunk_size=64, norm_mode="fla"):
    """Chunkwise WY forward with relative decays (the CUDA kernels' algorithm).

    Per chunk with chunk-local cumulative log-decay ``G`` (natural log):

    * ``Akk[r,i] = sum_c (b*k)[r,c] k[i,c] exp(G[r,c]-G[i,c])``  (i < r)
    * ``Aqk[r,i] = scale * sum_c q[r,c] k[i,c] exp(G[r,c]-G[i,c])``  (i <= r)
    * ``A = (I + Akk)^-1``; ``U = A (w*v)``; ``W = A (b*k*exp(G))``
    * ``Qg = scale*q*exp(G)``; ``Kd = k*exp(G_last - G)``; ``gl = exp(G_last)``
    * ``VN = U - W h``; ``o = Qg h + Aqk VN``; ``h' = gl*h + Kd^T VN``

    Returns ``(o, S_T, inter)`` where ``inter`` holds per-chunk arrays
    ``[B,H,NT,...]`` (zero-padded to ``chunk_size`` rows) for every quantity
    above plus ``h`` (the state entering each chunk).
    """
    q, k, v, g, b, w = (_f64(x) for x in (q, k, v, g, b, w))
    B, T, H, K = q.shape
    V = v.shape[-1]
    C = chunk_size
    if scale is None:
        scale = K ** -0.5
    if use_qk_l2norm:
        q, _ = _normalize(q, mode=norm_mode)
        k, _ = _normalize(k, mode=norm_mode)
    q, k, v, g, b, w = (_bthd_to_bhtd(x) for x in (q, k, v, g, b, w))
    NT = (T + C - 1) // C
    S = np.zeros((B, H, K, V)) if initial_state is None else _f64(initial_state).copy()
    names_ck = ("Qg", "Kd", "W", "G")
    inter = {n: np.zeros((B, H, NT, C, K)) for n in names_ck}
    inter.update({n: np.zeros((B, H, NT, C, V)) for n in ("U", "VN")})
    inter.update({n: np.zeros((B, H, NT, C, C)) for n in ("Aqk", "Akk", "A")})
    inter["gl"] = np.zeros((B, H, NT, K))
    inter["h"] = np.zeros((B, H, NT, K, V))
    o = np.zeros((B, H, T, V))
    for c in range(NT):
        s, e = c * C, min((c + 1) * C, T)
        n = e - s
        qc, kc, vc, gc, bc, wc = (x[:, :, s:e] for x in (q, k, v, g, b, w))
        G = np.cumsum(gc, axis=2)
        diff = G[:, :, :, None, :] - G[:, :, None, :, :]          # [B,H,r,i,K]
        mask_le = np.tril(np.ones((n, n), dtype=bool))
        mask_lt = np.tril(np.ones((n, n), dtype=bool), -1)
        dec = np.exp(np.where(mask_le[None, None, :, :, None], diff, -np.inf))
        kb = bc * kc
        Akk = np.einsum("bhrc,bhic,bhric->bhri", kb, kc, dec) * mask_lt
        Aqk = scale * np.einsum("bhrc,bhic,bhric->bhri", qc, kc, dec)
        A = _solve_unit_lower(Akk, np.broadcast_to(np.eye(n), Akk.shape))
        U = A @ (wc * vc)
        W = A @ (kb * np.exp(G))
        Qg = scale * qc * np.exp(G)
        Kd = kc * np.exp(G[:, :, -1:, :] - G)
        gl = np.exp(G[:, :, -1, :])
        VN = U - W @ S
        o[:, :, s:e] = Qg @ S + Aqk @ VN
        inter["h"][:, :, c] = S
        S = gl[..., None] * S + np.swapaxes(Kd, -1, -2) @ VN
        for name, val in (("Qg", Qg), ("Kd", Kd), ("W", W), ("G", G), ("U", U),
                          ("VN", VN)):
            inter[name][:, :, c, :n] = val
        for name, val in (("Aqk", Aqk), ("Akk", Akk), ("A", A)):
            inter[name][:, :, c, :n, :n] = val
        inter["gl"][:, :, c] = gl
    return _bhtd_to_bthd(o), S, inter


# ----------------------------------------------------------------------------
# varlen / sequence-parallel helpers (restating the packed-sequence semantics
# of chunk_gdn2.py:1347-1359 and the FLA context-parallel merge,
# chunk_kda.py:182-1299)
# ----------------------------------------------------------------------------

def recurrent_fwd_varlen(q, k, v, g, b, w, cu_seqlens, initial_state=None,
                         scale=None, use_qk_l2norm=True, norm_mode="torch"):
    """Packed-sequence forward: batch dim 1, sequences delimited by cu_seqlens.

    Each sequence starts from its own initial state (``[N,H,K,V]``) and no
    state crosses a sequence boundary (the Triton semantics; the reference's
    torch path ignores cu_seqlens, gdn2.py:937-949).
    """
    cu = [int(x) for x in cu_seqlens]
    N = len(cu) - 1
    H, K, V = q.shape[2], q.shape[3], v.shape[3]
    o = np.zeros(v.shape[:3] + (V,))
    hT = np.zeros((N, H, K, V))
    for n in range(N):
        s, e = cu[n], cu[n + 1]
        h0 = None if initial_state is None else _f64(initial_state)[n:n + 1]
        if e > s:
            on, hn = recurrent_fwd(q[:, s:e], k[:, s:e], v[:, s:e], g[:, s:e],
                                   b[:, s:e], w[:, s:e], h0, scale, use_qk_l2norm,
                                   norm_mode)
            o[:, s:e] = on
            hT[n] = hn[0]
        elif h0 is not None:
            hT[n] = h0[0]
    return o, hT


def span_transition(q, k, v, g, b, w, scale=None, use_qk_l2norm=True,
                    chunk_size=64, norm_mode="fla"):
    """Affine map of one token span: ``S_out = M S_in + h_e``.

    ``h_e`` is the end state from a zero initial state and ``M`` (``[B,H,K,K]``)
    the product of the per-token transitions
    ``(I - k (b*k)^T) Diag(exp g)``.  This is the pair the context-parallel
    pre-scan exchanges (chunk_kda.py:182-506, ``hm = [h_e | M]``).
    """
    q, k, v, g, b, w = (_f64(x) for x in (q, k, v, g, b, w))
    B, T, H, K = q.shape
    if use_qk_l2norm:
        k, _ = _normalize(k, mode=norm_mode)
    M = np.broadcast_to(np.eye(K), (B, H, K, K)).copy()
    for t in range(T):
        kt = k[:, t]
        kb = b[:, t] * kt
        Dm = np.exp(g[:, t])[..., None] * M
        M = Dm - kt[..., None] * np.einsum("bhk,bhkj->bhj", kb, Dm)[..., None, :]
    _, h_e = recurrent_fwd(q, k, v, g, b, w, None, scale, use_qk_l2norm=False)
    return M, h_e

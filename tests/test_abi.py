"""The C-ABI library loads, exports every symbol its header declares, and
rejects bad arguments with the documented status codes -- all without a GPU
(no call here reaches a CUDA API)."""

import ctypes
import os
import re

import pytest

from qwendopamine_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gdn2_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gdn2_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    return N.load()


def test_header_declares_the_binding_list():
    assert declared_functions() == sorted(N.EXPORTS)


def test_library_exports_every_declared_symbol(lib):
    raw = ctypes.CDLL(N.LIB_PATH)
    for name in declared_functions():
        assert hasattr(raw, name), name


def test_version_and_status_strings(lib):
    assert b"sm_100a" in lib.gdn2_version()
    assert lib.gdn2_status_string(0) == b"ok"
    assert lib.gdn2_status_string(1) == b"invalid argument"
    assert lib.gdn2_status_string(99) == b"unknown status"


def _problem(H=2, K=16, V=16, dtype=1, n_seqs=1, n_chunks=1, ptrs=True):
    p = 0x1000 if ptrs else None
    return N.ChunkProblem(H, K, V, dtype, 1, 0.25,
                          N.Seqs(64, n_seqs, n_chunks, p, p, p))


def test_saved_and_workspace_sizes_follow_the_layout(lib):
    for dt, es in ((0, 4), (1, 2)):
        H, K, V, nc = 3, 64, 32, 5
        prob = _problem(H, K, V, dt, 1, nc)
        nh = nc * H
        al = lambda x: (x + 255) & ~255
        off = 0
        for rows in (64 * K, 64 * K, 64 * K, 64 * V, 64 * V, 64 * 64, 64 * 64):
            off = al(off + nh * rows * es)
        off = al(off + nh * K * 4)
        off = al(off + nh * K * V * es)
        assert lib.gdn2_chunk_saved_bytes(prob) == off
        ws = al(nh * K * V * es)
        ws = al(ws + nh * 64 * V * es)
        assert lib.gdn2_chunk_bwd_workspace_bytes(prob) == ws


def test_invalid_problem_is_rejected_with_message(lib):
    bad = _problem(K=0)
    assert lib.gdn2_chunk_saved_bytes(bad) == 0
    assert b"positive" in lib.gdn2_last_error()
    big = _problem(K=264)  # the reference accepts K <= 256 (chunk_gdn2.py:1380)
    assert lib.gdn2_chunk_fwd_intra(big, *([None] * 6), None, 0, None) == N.ERR_UNSUPPORTED
    assert b"up to 256" in lib.gdn2_last_error()
    assert lib.gdn2_chunk_saved_bytes(_problem(K=256, V=256)) > 0
    with pytest.raises(NotImplementedError):
        N.check(N.ERR_UNSUPPORTED, "x")
    nodtype = _problem(dtype=7)
    assert lib.gdn2_chunk_fwd_state(nodtype, None, None, None, None, 0, None) == N.ERR_INVALID
    notab = _problem(ptrs=False)
    assert lib.gdn2_chunk_fwd(notab, *([None] * 10), 0, None) == N.ERR_INVALID
    assert b"tables" in lib.gdn2_last_error()


def test_null_pointers_and_short_buffers_are_rejected(lib):
    prob = _problem()
    rc = lib.gdn2_chunk_fwd_intra(prob, *([None] * 6), None, 0, None)
    assert rc == N.ERR_INVALID and b"null" in lib.gdn2_last_error()
    fake = ctypes.c_void_p(0x1000)
    rc = lib.gdn2_chunk_fwd_intra(prob, *([fake] * 6), fake, 16, None)
    assert rc == N.ERR_WORKSPACE and b"saved buffer" in lib.gdn2_last_error()
    rc = lib.gdn2_chunk_bwd(prob, *([fake] * 6), fake, 1 << 40, fake, None, *([fake] * 6), None,
                            fake, 1, None)
    assert rc == N.ERR_WORKSPACE


def test_misaligned_16bit_tensors_are_rejected(lib):
    """The bf16 kernels move token rows with bulk async copies: tensors must
    start on a 16-byte boundary (the Python wrappers copy misaligned views)."""
    prob = _problem(K=64, V=64, dtype=1)
    ok, odd = ctypes.c_void_p(0x1000), ctypes.c_void_p(0x1002)
    big = 1 << 40
    rc = lib.gdn2_chunk_fwd_intra(prob, ok, odd, ok, ok, ok, ok, ok, big, None)
    assert rc == N.ERR_INVALID and b"16-byte" in lib.gdn2_last_error()
    rc = lib.gdn2_chunk_bwd_intra(prob, ok, ok, ok, ok, ok, ok, ok, big, odd, *([ok] * 6), ok, big,
                                  None)
    assert rc == N.ERR_INVALID and b"16-byte" in lib.gdn2_last_error()
    # outputs and the state passes' buffers too
    for i in range(6):
        grads = [ok] * 6
        grads[i] = odd
        rc = lib.gdn2_chunk_bwd_intra(prob, ok, ok, ok, ok, ok, ok, ok, big, ok, *grads, ok, big,
                                      None)
        assert rc == N.ERR_INVALID and b"16-byte" in lib.gdn2_last_error(), i
    rc = lib.gdn2_chunk_fwd_state(prob, None, odd, None, ok, big, None)
    assert rc == N.ERR_INVALID and b"16-byte" in lib.gdn2_last_error()
    rc = lib.gdn2_chunk_bwd_state(prob, ok, big, odd, None, None, ok, big, None)
    assert rc == N.ERR_INVALID and b"16-byte" in lib.gdn2_last_error()


def test_recurrent_argument_checks(lib):
    def rp(**kw):
        base = dict(B=2, T=1, H=2, HV=2, K=16, V=16, dtype=1, use_qk_l2norm=1, scale=0.25,
                    n_seqs=2, cu_seqlens=None, state_indices=None, state_stride=0)
        base.update(kw)
        return N.RecurrentProblem(**base)

    f = ctypes.c_void_p(0x1000)
    args = [f] * 6 + [None, f, None, None]
    assert lib.gdn2_recurrent_fwd(rp(HV=3), *args) == N.ERR_INVALID
    assert b"multiple" in lib.gdn2_last_error()
    assert lib.gdn2_recurrent_fwd(rp(K=300), *args) == N.ERR_UNSUPPORTED
    assert lib.gdn2_recurrent_fwd(rp(cu_seqlens=0x1000), *args) == N.ERR_INVALID
    assert lib.gdn2_recurrent_fwd(rp(n_seqs=3), *args) == N.ERR_INVALID
    assert lib.gdn2_recurrent_fwd(rp(state_indices=0x1000, state_stride=5), *args) == N.ERR_INVALID
    assert lib.gdn2_recurrent_fwd(rp(), *([None] * 10)) == N.ERR_INVALID


def test_cp_merge_argument_checks(lib):
    prob = _problem()
    f = ctypes.c_void_p(0x1000)
    assert lib.gdn2_cp_merge(prob, f, f, 3, 2, 1, None, f, None) == N.ERR_INVALID
    assert lib.gdn2_cp_merge(prob, f, None, 0, 2, 0, None, f, None) == N.ERR_INVALID
    # the sub-span scan: sizes, null pointers and the supported shapes
    assert lib.gdn2_cp_unfold(prob, f, f, 0, 1, None, f, None) == N.ERR_INVALID
    assert lib.gdn2_cp_unfold(prob, f, None, 4, 0, None, f, None) == N.ERR_INVALID
    assert lib.gdn2_cp_unfold(prob, None, f, 4, 1, None, f, None) == N.ERR_INVALID


def test_status_maps_to_python_exceptions(lib):
    lib.gdn2_chunk_saved_bytes(_problem(K=0))
    with pytest.raises(ValueError, match="invalid argument"):
        N.check(N.ERR_INVALID, "probe")
    with pytest.raises(N.GDN2Error):
        N.check(N.ERR_CUDA, "probe")
    N.check(N.OK, "probe")


def test_gate_in_kernel_arguments_are_checked(lib):
    """Gate in kernel: modes 0..2 only, A_log required, served by the bf16
    kernels only (fp32 problems gate with torch ops on the Python side)."""
    prob = _problem(dtype=1)
    prob.gate = 3
    prob.A_log = 0x1000
    assert lib.gdn2_chunk_saved_bytes(prob) == 0
    assert b"gate" in lib.gdn2_last_error()
    prob.gate, prob.A_log = 1, None
    assert lib.gdn2_chunk_fwd_intra(prob, *([None] * 6), None, 0, None) == N.ERR_INVALID
    prob.A_log = 0x1000
    assert lib.gdn2_chunk_saved_bytes(prob) > 0
    f32 = _problem(dtype=0)
    f32.gate, f32.A_log = 2, 0x1000
    assert lib.gdn2_chunk_fwd_intra(f32, *([None] * 6), None, 0, None) == N.ERR_UNSUPPORTED


def test_conv_and_norm_arguments_are_checked(lib):
    """Block prologue / epilogue entry points: shapes, dtypes and workspace
    sizes are validated before any CUDA call."""
    conv = N.ConvProblem(2, 100, 64, 4, 1, 1)
    # 64-token strips per batch entry; (W + 1) fp32 partial sums per channel
    assert lib.gdn2_conv_bwd_workspace_bytes(conv) == 2 * 2 * 5 * 64 * 4
    for bad, code in ((N.ConvProblem(2, 100, 64, 5, 1, 1), N.ERR_UNSUPPORTED),
                      (N.ConvProblem(2, 100, 60, 4, 1, 1), N.ERR_UNSUPPORTED),
                      (N.ConvProblem(2, 0, 64, 4, 1, 1), N.ERR_INVALID),
                      (N.ConvProblem(2, 100, 64, 4, 7, 1), N.ERR_INVALID),
                      (N.ConvProblem(2, 100, 64, 4, 1, 2), N.ERR_INVALID)):
        assert lib.gdn2_conv_fwd(bad, *([None] * 6), None) == code
    fake, odd = ctypes.c_void_p(0x1000), ctypes.c_void_p(0x1008)
    assert lib.gdn2_conv_fwd(conv, odd, fake, None, None, fake, None, None) == N.ERR_INVALID
    assert b"16-byte" in lib.gdn2_last_error()
    rc = lib.gdn2_conv_bwd(conv, fake, fake, None, None, fake, fake, fake, None, None, fake, 8,
                           None)
    assert rc == N.ERR_WORKSPACE
    norm = N.NormProblem(1000, 128, 1, 1, 1e-5, 0)
    assert lib.gdn2_gated_norm_bwd_workspace_bytes(norm) == 63 * 128 * 4  # ceil(1000 / 16) blocks
    for bad, code in ((N.NormProblem(10, 300, 1, 1, 1e-5, 0), N.ERR_UNSUPPORTED),
                      (N.NormProblem(10, 12, 1, 1, 1e-5, 0), N.ERR_UNSUPPORTED),
                      (N.NormProblem(10, 64, 1, 2, 1e-5, 0), N.ERR_UNSUPPORTED),
                      (N.NormProblem(10, 64, 1, 1, 1e-5, 1), N.ERR_INVALID),
                      (N.NormProblem(10, 64, 1, 0, 1e-5, 3), N.ERR_INVALID)):
        assert lib.gdn2_gated_norm_fwd(bad, *([None] * 4), None) == code
    assert lib.gdn2_gated_norm_fwd(N.NormProblem(0, 64, 1, 1, 1e-5, 0), *([None] * 4), None) == 0


def test_negative_sm_budget_is_rejected(lib):
    """max_ctas (the SM budget a two-stream caller gives one launch) must be
    >= 0; 0, the default, keeps the whole GPU."""
    p = _problem()
    assert p.max_ctas == 0 and lib.gdn2_chunk_saved_bytes(p) > 0
    p.max_ctas = -1
    assert lib.gdn2_chunk_saved_bytes(p) == 0
    assert b"max_ctas" in lib.gdn2_last_error()
    assert lib.gdn2_chunk_fwd_intra(p, *([None] * 6), None, 0, None) == N.ERR_INVALID
    p.max_ctas = 116
    assert lib.gdn2_chunk_saved_bytes(p) > 0

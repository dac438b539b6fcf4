"""ctypes binding of ``libgdn2_b200.so`` (the C ABI declared in
``include/gdn2_b200.h``).

The library is loaded on first use.  If it is missing or fails to load, every
entry point raises: the package has no CPU or PyTorch fallback for the GDN-2
core recurrence.
"""

from __future__ import annotations

import contextlib
import ctypes
import os
import threading
from ctypes import c_float, c_int32, c_int64, c_size_t, c_void_p

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libgdn2_b200.so")

DTYPE_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_WORKSPACE = range(5)
NOALLOC_SCRATCH_BYTES = 32 << 20  # GDN2_NOALLOC_SCRATCH_BYTES in include/gdn2_b200.h

EXPORTS = (
    "gdn2_version",
    "gdn2_status_string",
    "gdn2_last_error",
    "gdn2_chunk_saved_bytes",
    "gdn2_chunk_fwd",
    "gdn2_chunk_fwd_intra",
    "gdn2_chunk_fwd_state",
    "gdn2_chunk_bwd_workspace_bytes",
    "gdn2_chunk_bwd",
    "gdn2_chunk_bwd_state",
    "gdn2_chunk_bwd_intra",
    "gdn2_chunk_bwd_noalloc",
    "gdn2_recurrent_fwd",
    "gdn2_cp_workspace_bytes",
    "gdn2_cp_fwd_prescan",
    "gdn2_cp_bwd_prescan",
    "gdn2_cp_merge",
    "gdn2_cp_unfold",
    "gdn2_conv_fwd",
    "gdn2_conv_bwd_workspace_bytes",
    "gdn2_conv_bwd",
    "gdn2_gated_norm_fwd",
    "gdn2_gated_norm_bwd_workspace_bytes",
    "gdn2_gated_norm_bwd",
    "gdn2_fault_status",
    "gdn2_test_fwd_state_wait_timeout",
)


class Seqs(ctypes.Structure):
    _fields_ = [
        ("total_tokens", c_int64),
        ("n_seqs", c_int32),
        ("n_chunks", c_int32),
        ("cu_seqlens", c_void_p),
        ("chunk_offsets", c_void_p),
        ("chunk_seq", c_void_p),
    ]


class ChunkProblem(ctypes.Structure):
    _fields_ = [
        ("H", c_int32),
        ("K", c_int32),
        ("V", c_int32),
        ("dtype", c_int32),
        ("use_qk_l2norm", c_int32),
        ("scale", c_float),
        ("seqs", Seqs),
        ("A_log", c_void_p),
        ("dt_bias", c_void_p),
        ("gate", c_int32),
        ("lower_bound", c_float),
        ("dA_log", c_void_p),
        ("ddt_bias", c_void_p),
        ("max_ctas", c_int32),
    ]


class RecurrentProblem(ctypes.Structure):
    _fields_ = [
        ("B", c_int32),
        ("T", c_int32),
        ("H", c_int32),
        ("HV", c_int32),
        ("K", c_int32),
        ("V", c_int32),
        ("dtype", c_int32),
        ("use_qk_l2norm", c_int32),
        ("scale", c_float),
        ("n_seqs", c_int32),
        ("cu_seqlens", c_void_p),
        ("state_indices", c_void_p),
        ("state_stride", c_int64),
        ("state_indices_stride", c_int64),
        ("num_accepted_tokens", c_void_p),
        ("A_log", c_void_p),
        ("dt_bias", c_void_p),
        ("gate", c_int32),
        ("lower_bound", c_float),
    ]


class ConvProblem(ctypes.Structure):
    _fields_ = [
        ("B", c_int32),
        ("T", c_int32),
        ("D", c_int32),
        ("W", c_int32),
        ("dtype", c_int32),
        ("activation", c_int32),
        ("prefix_sb", c_int64),
        ("prefix_sw", c_int64),
        ("prefix_sd", c_int64),
    ]


class NormProblem(ctypes.Structure):
    _fields_ = [
        ("rows", c_int64),
        ("N", c_int32),
        ("dtype", c_int32),
        ("weight_dtype", c_int32),
        ("eps", c_float),
        ("fp32_math", c_int32),
    ]


class GDN2Error(RuntimeError):
    """A libgdn2_b200 entry point returned an error status."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


_lock = threading.Lock()
_lib = None


def _declare(lib):
    P = ctypes.POINTER
    cp = P(ChunkProblem)
    rp = P(RecurrentProblem)
    vp = P(ConvProblem)
    np_ = P(NormProblem)
    v = c_void_p
    sig = {
        "gdn2_version": ([], ctypes.c_char_p),
        "gdn2_status_string": ([ctypes.c_int], ctypes.c_char_p),
        "gdn2_last_error": ([], ctypes.c_char_p),
        "gdn2_chunk_saved_bytes": ([cp], c_size_t),
        "gdn2_chunk_bwd_workspace_bytes": ([cp], c_size_t),
        "gdn2_cp_workspace_bytes": ([cp], c_size_t),
        "gdn2_chunk_fwd": ([cp, v, v, v, v, v, v, v, v, v, v, c_size_t, v], ctypes.c_int),
        "gdn2_chunk_fwd_intra": ([cp, v, v, v, v, v, v, v, c_size_t, v], ctypes.c_int),
        "gdn2_chunk_fwd_state": ([cp, v, v, v, v, c_size_t, v], ctypes.c_int),
        "gdn2_chunk_bwd": ([cp, v, v, v, v, v, v, v, c_size_t, v, v, v, v, v, v, v, v, v, v,
                            c_size_t, v], ctypes.c_int),
        "gdn2_chunk_bwd_state": ([cp, v, c_size_t, v, v, v, v, c_size_t, v], ctypes.c_int),
        "gdn2_chunk_bwd_intra": ([cp, v, v, v, v, v, v, v, c_size_t, v, v, v, v, v, v, v, v,
                                  c_size_t, v], ctypes.c_int),
        "gdn2_chunk_bwd_noalloc": ([cp, v, v, v, v, v, v, v, c_size_t, v, v, v, v, v, v, v, v,
                                    v, v], ctypes.c_int),
        "gdn2_recurrent_fwd": ([rp, v, v, v, v, v, v, v, v, v, v], ctypes.c_int),
        "gdn2_cp_fwd_prescan": ([cp, v, c_size_t, v, v, c_size_t, v], ctypes.c_int),
        "gdn2_cp_bwd_prescan": ([cp, v, c_size_t, v, v, v, v, c_size_t, v], ctypes.c_int),
        "gdn2_cp_merge": ([cp, v, v, c_int32, c_int32, c_int32, v, v, v], ctypes.c_int),
        "gdn2_cp_unfold": ([cp, v, v, c_int32, c_int32, v, v, v], ctypes.c_int),
        "gdn2_fault_status": ([v, c_int32], ctypes.c_int),
        "gdn2_test_fwd_state_wait_timeout": ([cp, v, v, c_size_t, c_int32, ctypes.c_uint64, v],
                                             ctypes.c_int),
        "gdn2_conv_fwd": ([vp, v, v, v, v, v, v, v], ctypes.c_int),
        "gdn2_conv_bwd_workspace_bytes": ([vp], c_size_t),
        "gdn2_conv_bwd": ([vp, v, v, v, v, v, v, v, v, v, v, c_size_t, v], ctypes.c_int),
        "gdn2_gated_norm_fwd": ([np_, v, v, v, v, v], ctypes.c_int),
        "gdn2_gated_norm_bwd_workspace_bytes": ([np_], c_size_t),
        "gdn2_gated_norm_bwd": ([np_, v, v, v, v, v, v, v, v, c_size_t, v], ctypes.c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res


def load():
    """Load (once) and return the ctypes handle; raise if the library is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"libgdn2_b200.so is not built ({LIB_PATH}); run "
                    "`python -m qwendopamine_b200.build`. There is no CPU fallback.")
            lib = ctypes.CDLL(LIB_PATH)
            _declare(lib)
            _lib = lib
    return _lib


def check(status: int, fn: str) -> None:
    if status == OK:
        return
    lib = load()
    msg = lib.gdn2_last_error().decode(errors="replace")
    text = f"{fn}: {lib.gdn2_status_string(status).decode()} ({msg})"
    if status == ERR_INVALID:
        raise ValueError(text)
    if status == ERR_UNSUPPORTED:
        raise NotImplementedError(text)
    raise GDN2Error(status, text)


def fault_status(device=None, clear: bool = True) -> int:
    """Synchronise ``device``'s current stream and return the device fault
    word (nonzero when a kernel's bounded wait ran out); reset it if ``clear``."""
    lib = load()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    r = lib.gdn2_fault_status(stream_of(dev), 1 if clear else 0)
    if r < 0:
        raise GDN2Error(ERR_CUDA, f"gdn2_fault_status: {lib.gdn2_last_error().decode()}")
    return r


# ---------------------------------------------------------------------------
# optional per-phase timing: CUDA events on the launching stream around each
# library phase (forward intra / state pass, pre-scans, exchange, merges,
# backward state / intra pass).  Off unless a caller opens phase_timing().
# The record list is process-wide, not per thread, because autograd runs the
# backward on its own device thread.
# ---------------------------------------------------------------------------
_phase_records = None


@contextlib.contextmanager
def phase_timing():
    """Collect ``(name, start_event, end_event)`` for every phase the package
    runs inside the block (events recorded on the current stream; read them
    after a synchronize).  For benchmarks; one collector at a time."""
    global _phase_records
    prev, rec = _phase_records, []
    _phase_records = rec
    try:
        yield rec
    finally:
        _phase_records = prev


@contextlib.contextmanager
def phase(name: str, stream=None):
    """Bracket one phase with CUDA events while :func:`phase_timing` is open
    (on ``stream``, a ``torch.cuda.Stream``, or the current stream)."""
    rec = _phase_records
    if rec is None:
        yield
        return
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    try:
        yield
    finally:
        e.record(stream)
        rec.append((name, s, e))


def ptr(t):
    """Device address of a tensor (or None -> NULL)."""
    return None if t is None else c_void_p(t.data_ptr())


def stream_of(device: torch.device):
    return c_void_p(torch.cuda.current_stream(device).cuda_stream)


def dtype_code(dt: torch.dtype) -> int:
    try:
        return DTYPE_CODES[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}; expected float32, bfloat16 or float16") from None


# ---------------------------------------------------------------------------
# sequence / chunk tables
# ---------------------------------------------------------------------------
CHUNK = 64
_table_cache: dict = {}


class SeqTables:
    """Device int32 tables describing how rows split into sequences and chunks."""

    def __init__(self, cu: torch.Tensor, coff: torch.Tensor, cseq: torch.Tensor,
                 n_seqs: int, n_chunks: int, total: int):
        self.cu, self.coff, self.cseq = cu, coff, cseq
        self.n_seqs, self.n_chunks, self.total = n_seqs, n_chunks, total

    def struct(self) -> Seqs:
        return Seqs(self.total, self.n_seqs, self.n_chunks, self.cu.data_ptr(),
                    self.coff.data_ptr(), self.cseq.data_ptr())


def _tables_from_lengths(lens, device) -> SeqTables:
    cu = [0]
    coff = [0]
    cseq = []
    for n, L in enumerate(lens):
        cu.append(cu[-1] + L)
        nc = (L + CHUNK - 1) // CHUNK
        coff.append(coff[-1] + nc)
        cseq.extend([n] * nc)
    mk = lambda x: torch.tensor(x if x else [0], dtype=torch.int32, device=device)
    return SeqTables(mk(cu), mk(coff), mk(cseq), len(lens), len(cseq), cu[-1])


def split_tables(B: int, T: int, S: int, device) -> SeqTables:
    """Tables that cut each of B fixed-length sequences of T tokens into S
    sub-spans of whole 64-token chunks (the last one takes the remainder),
    listed sequence by sequence: the kernels treat them as B*S sequences.
    The chunks, and so every per-chunk buffer, are the same as for B
    sequences; only where the state passes start and stop changes."""
    key = ("split", B, T, S, str(device))
    tab = _table_cache.get(key)
    if tab is None:
        nch = (T + CHUNK - 1) // CHUNK
        cuts = [CHUNK * (nch * j // S) for j in range(S)] + [T]
        lens = [cuts[j + 1] - cuts[j] for j in range(S)]
        if any(L <= 0 for L in lens):
            raise ValueError(f"cannot cut {T} tokens into {S} chunk-aligned sub-spans")
        tab = _tables_from_lengths(lens * B, device)
        if len(_table_cache) > 64:
            _table_cache.clear()
        _table_cache[key] = tab
    return tab


def seq_tables(B: int, T: int, device, cu_seqlens=None, cu_seqlens_cpu=None) -> SeqTables:
    """Tables for fixed-length [B, T] input (cached) or packed cu_seqlens."""
    if cu_seqlens is None:
        key = (B, T, str(device))
        tab = _table_cache.get(key)
        if tab is None:
            tab = _tables_from_lengths([T] * B, device)
            if len(_table_cache) > 64:
                _table_cache.clear()
            _table_cache[key] = tab
        return tab
    host = cu_seqlens_cpu if cu_seqlens_cpu is not None else cu_seqlens.detach().cpu()
    cu = [int(x) for x in host.tolist()]
    lens = [cu[i + 1] - cu[i] for i in range(len(cu) - 1)]
    if any(L < 0 for L in lens) or cu[0] != 0:
        raise ValueError("cu_seqlens must start at 0 and be non-decreasing")
    return _tables_from_lengths(lens, device)

"""The backward entry point that allocates nothing (gdn2_chunk_bwd_noalloc).

It exists for callers that cannot allocate device memory while the backward
runs (a plugin host owning all device memory, or a loop that has reserved
nearly all HBM and cannot afford an allocation failure or the device
synchronisation of cudaMalloc / cudaFree mid-step); its scratch is an array
built into the library.  These tests call it through the C ABI on two
different problems in a row and check that each result equals, bit for bit,
the regular entry point gdn2_chunk_bwd's (which takes a caller-allocated
workspace), and check that a problem larger than the built-in scratch is
refused with a clear error.  This file is named
so that pytest collects it last.
"""

import ctypes

import pytest
import torch

from gdn2_testutil import TOL, make_inputs, rel, to_dev
from qwendopamine_b200 import _native as N

pytestmark = pytest.mark.gpu
NAMES = ("q", "k", "v", "g", "b", "w")


def _case(dev, dtype, B, T, H, K, V, seed):
    """Forward on seeded inputs; returns a function that runs the backward
    through either entry point and returns all gradients."""
    lib = N.load()
    d = to_dev(make_inputs(B, T, H, K, V, seed=seed, dtype=dtype), dev, dtype)
    gen = torch.Generator(device=dev).manual_seed(seed + 1)
    do = torch.randn(B, T, H, V, device=dev, generator=gen).to(dtype)
    dht = torch.randn(B, H, K, V, device=dev, generator=gen)
    tables = N.seq_tables(B, T, dev)
    prob = N.ChunkProblem(H, K, V, N.dtype_code(dtype), 1, K ** -0.5, tables.struct())
    st = N.stream_of(dev)
    sbytes = lib.gdn2_chunk_saved_bytes(prob)
    saved = torch.empty(sbytes, dtype=torch.uint8, device=dev)
    o = torch.empty_like(d["v"])
    P = {n: N.ptr(d[n]) for n in NAMES}
    N.check(lib.gdn2_chunk_fwd(prob, *(P[n] for n in NAMES), N.ptr(d["h0"]), N.ptr(o), None,
                               N.ptr(saved), sbytes, st), "gdn2_chunk_fwd")
    wbytes = lib.gdn2_chunk_bwd_workspace_bytes(prob)
    assert 0 < wbytes <= N.NOALLOC_SCRATCH_BYTES

    def grads(noalloc):
        out = {n: torch.empty_like(d[n]) for n in NAMES}
        out["h0"] = torch.empty_like(d["h0"])
        G = [N.ptr(out[n]) for n in NAMES]
        common = (prob, *(P[n] for n in NAMES), N.ptr(saved), sbytes, N.ptr(do), N.ptr(dht), *G,
                  N.ptr(out["h0"]))
        if noalloc:
            rc = lib.gdn2_chunk_bwd_noalloc(*common, st)
            N.check(rc, "gdn2_chunk_bwd_noalloc")
        else:
            ws = torch.empty(wbytes, dtype=torch.uint8, device=dev)
            rc = lib.gdn2_chunk_bwd(*common, N.ptr(ws), wbytes, st)
            N.check(rc, "gdn2_chunk_bwd")
        torch.cuda.synchronize(dev)
        return out

    return grads


def _equal(got, ref):
    # Both entry points run the same deterministic kernels on the same
    # inputs; only the workspace address differs, so the gradients must agree
    # bit for bit -- a read of scratch left behind by an earlier call would
    # show up here even where it stayed inside the rel-L2 tolerance.
    for n in (*NAMES, "h0"):
        assert torch.equal(got[n], ref[n]), (n, rel(got[n], ref[n]), TOL)


@pytest.mark.parametrize("dtype,first,second", [
    (torch.float32, (2, 150, 3, 64, 64), (1, 97, 2, 64, 32)),
    # 24 MiB of the 32 MiB scratch, then a ragged problem whose chunks map
    # onto different parts of the scratch than the first call's
    (torch.bfloat16, (1, 2048, 16, 128, 128), (2, 333, 5, 128, 128)),
])
def test_noalloc_backward_matches_regular_entry_point_twice(cuda_device, dtype, first, second):
    """Two calls in a row on different problems (different inputs, shapes
    and scratch layouts), each equal to the regular entry point's result."""
    for shape, seed in ((first, sum(first)), (second, sum(second) + 7)):
        run = _case(cuda_device, dtype, *shape, seed=seed)
        ref = run(noalloc=False)
        _equal(run(noalloc=True), ref)


def test_noalloc_backward_rejects_problems_beyond_its_scratch(cuda_device):
    lib = N.load()
    fake = ctypes.c_void_p(0x1000)
    # config-1 size: 512 chunks x 16 heads needs ~393 MB of scratch
    prob = N.ChunkProblem(16, 128, 128, N.dtype_code(torch.bfloat16), 1, 128 ** -0.5,
                          N.Seqs(8 * 4096, 8, 512, 0x1000, 0x1000, 0x1000))
    need = lib.gdn2_chunk_bwd_workspace_bytes(prob)
    assert need > N.NOALLOC_SCRATCH_BYTES
    rc = lib.gdn2_chunk_bwd_noalloc(prob, *([fake] * 6), fake, 1 << 40, fake, None,
                                    *([fake] * 6), None, None)
    assert rc == N.ERR_WORKSPACE
    msg = lib.gdn2_last_error().decode()
    assert str(need) in msg and "GDN2_NOALLOC_SCRATCH_BYTES" in msg

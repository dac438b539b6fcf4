"""Block prologue / epilogue kernels on the GPU (through the C ABI):
causal depthwise conv + SiLU (ShortConvolution) and the SiLU-gated RMSNorm
(RMSNormGated).

* fp32: forward and backward against the float64 oracle (rel-L2 <= 1e-5).
* bf16: forward bit-for-bit against torch's CUDA evaluation of the
  reference's own expressions (gdn2.py:396-452: F.conv1d + F.silu; x.pow(2)
  .mean, rsqrt, products in the input dtype) -- at most one bf16 step apart
  and >= 99 % identical; backward against the oracle (rel-L2 <= 2e-2).
* the reference's golden fixture (tests/golden/block_ops.npz) through the
  kernels, the decode-cache step, prefixes given through strides, and
  deterministic weight gradients.
"""

import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import block_oracle as BO

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def rel(a, b):
    a = a.detach().double().cpu().numpy() if isinstance(a, torch.Tensor) else np.asarray(a, np.float64)
    b = b.detach().double().cpu().numpy() if isinstance(b, torch.Tensor) else np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def np64(t):
    return t.detach().double().cpu().numpy()


def bf16_steps(a, b):
    ia = a.detach().float().cpu().view(torch.int32).long() >> 16
    ib = b.detach().float().cpu().view(torch.int32).long() >> 16
    return (ia - ib).abs()


def _conv_inputs(B, T, D, W, bias, dtype, dev, seed):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, D, generator=gen)
    w = torch.randn(D, 1, W, generator=gen) * 0.5
    b = torch.randn(D, generator=gen) * 0.5 if bias else None
    cvt = lambda t: None if t is None else t.to(dev, dtype)
    return cvt(x), cvt(w), cvt(b)


@pytest.mark.parametrize("W", [1, 2, 3, 4])
@pytest.mark.parametrize("B,T,D", [(2, 1, 8), (1, 5, 48), (3, 65, 136), (2, 600, 256)])
@pytest.mark.parametrize("bias,act", [(True, "silu"), (False, None)])
def test_conv_fp32_forward_backward(cuda_device, W, B, T, D, bias, act):
    from qwendopamine_b200.gdn2_ops.block_ops import short_conv

    x, w, b = _conv_inputs(B, T, D, W, bias, torch.float32, cuda_device, seed=W + T + D)
    x.requires_grad_()
    w.requires_grad_()
    if b is not None:
        b.requires_grad_()
    y, _ = short_conv(x, w, b, act)
    assert rel(y, BO.conv_fwd(np64(x), np64(w), None if b is None else np64(b),
                              activation=act)) < 1e-5
    dy = torch.randn_like(y)
    (y * dy).sum().backward()
    dx, dw, db, _ = BO.conv_bwd(np64(x), np64(w), np64(dy), None if b is None else np64(b),
                                activation=act)
    assert rel(x.grad, dx) < 1e-5
    assert rel(w.grad.view(D, W), dw) < 1e-5
    if b is not None:
        assert rel(b.grad, db) < 1e-5


def test_conv_golden_fixture(cuda_device):
    from qwendopamine_b200 import ShortConvolution

    g = np.load(os.path.join(GOLD, "block_ops.npz"))
    m = ShortConvolution(48, kernel_size=4, bias=True).to(cuda_device)
    with torch.no_grad():
        m.conv1d.weight.copy_(torch.from_numpy(g["conv_a_w"]))
        m.conv1d.bias.copy_(torch.from_numpy(g["conv_a_bias"]))
    x = torch.from_numpy(g["conv_a_x"]).to(cuda_device).requires_grad_()
    y, cache = m(x, output_final_state=True)
    assert rel(y, g["conv_a_y"]) < 1e-6
    assert torch.equal(cache.cpu(), torch.from_numpy(g["conv_a_cache"]))
    (y * torch.from_numpy(g["conv_a_dy"]).to(cuda_device)).sum().backward()
    assert rel(x.grad, g["conv_a_dx"]) < 1e-6
    assert rel(m.conv1d.weight.grad, g["conv_a_dw"]) < 1e-5
    assert rel(m.conv1d.bias.grad, g["conv_a_dbias"]) < 1e-5
    # one decode token with a cache [B, D, W-1] (a strided prefix)
    with torch.no_grad():
        yt, c1 = m(torch.from_numpy(g["conv_dec_x"]).to(cuda_device),
                   cache=torch.from_numpy(g["conv_dec_cache"]).to(cuda_device),
                   output_final_state=True)
    assert rel(yt, g["conv_dec_y"]) < 1e-6
    assert torch.equal(c1.cpu(), torch.from_numpy(g["conv_dec_new_cache"]))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_conv_prefix_and_state(cuda_device, dtype):
    """A prefix given through strides (the transposed [B, D, W-1] cache view)
    equals running the concatenation; dprefix is the gradient of those rows;
    new_state is the last W-1 rows of [prefix; x] in the cache layout."""
    from qwendopamine_b200.gdn2_ops.block_ops import short_conv

    B, T, D, W = 2, 70, 64, 4
    x, w, b = _conv_inputs(B, T, D, W, True, dtype, cuda_device, seed=5)
    cache = torch.randn(B, D, W - 1, device=cuda_device).to(dtype)
    pre = cache.transpose(1, 2).requires_grad_() if dtype == torch.float32 else cache.transpose(1, 2)
    y, state = short_conv(x, w, b, "silu", prefix=pre, output_final_state=True)
    full, _ = short_conv(torch.cat([pre.detach(), x], 1), w, b, "silu")
    assert torch.equal(y, full[:, W - 1:])
    assert torch.equal(state, torch.cat([pre.detach(), x], 1)[:, -(W - 1):].transpose(1, 2))
    if dtype == torch.float32:
        dy = torch.randn_like(y)
        (y * dy).sum().backward()
        _, _, _, dpre = BO.conv_bwd(np64(x), np64(w), np64(dy), np64(b),
                                    prefix=np64(pre.detach()))
        assert rel(pre.grad, dpre) < 1e-5
    # a prefix shorter than the window: T = 1, 2
    for t in (1, 2):
        yt, st = short_conv(x[:, :t], w, b, "silu", prefix=pre.detach(), output_final_state=True)
        ft, _ = short_conv(torch.cat([pre.detach(), x[:, :t]], 1), w, b, "silu")
        assert torch.equal(yt, ft[:, W - 1:])
        assert torch.equal(st, torch.cat([pre.detach(), x[:, :t]], 1)[:, -(W - 1):].transpose(1, 2))


@pytest.mark.parametrize("W", [2, 4])
@pytest.mark.parametrize("act", ["silu", None])
def test_conv_bf16_matches_torch_cuda_expression(cuda_device, W, act):
    from qwendopamine_b200.gdn2_ops.block_ops import short_conv

    B, T, D = 4, 333, 2048
    x, w, b = _conv_inputs(B, T, D, W, True, torch.bfloat16, cuda_device, seed=W)
    y, _ = short_conv(x, w, b, act)
    ref = F.conv1d(x.transpose(1, 2), w, b, padding=W - 1, groups=D)[:, :, :T]
    if act == "silu":
        ref = F.silu(ref)
    ref = ref.transpose(1, 2)
    steps = bf16_steps(y, ref)
    assert steps.max() <= 1 and (steps == 0).float().mean() > 0.99
    # backward against the oracle
    xg = x.clone().requires_grad_()
    wg = w.clone().requires_grad_()
    bg = b.clone().requires_grad_()
    y2, _ = short_conv(xg, wg, bg, act)
    dy = torch.randn_like(y2)
    (y2.float() * dy.float()).sum().backward()
    dx, dw, db, _ = BO.conv_bwd(np64(x), np64(w), np64(dy), np64(b), activation=act)
    assert rel(xg.grad, dx) < 2e-2
    assert rel(wg.grad.view(D, W), dw) < 2e-2
    assert rel(bg.grad, db) < 2e-2


def test_conv_weight_gradient_is_deterministic(cuda_device):
    from qwendopamine_b200.gdn2_ops.block_ops import short_conv

    x, w, b = _conv_inputs(8, 1024, 512, 4, True, torch.bfloat16, cuda_device, seed=3)
    grads = []
    for _ in range(2):
        wg = w.clone().requires_grad_()
        bg = b.clone().requires_grad_()
        y, _ = short_conv(x, wg, bg)
        y.float().sum().backward()
        grads.append((wg.grad.clone(), bg.grad.clone()))
    assert torch.equal(grads[0][0], grads[1][0]) and torch.equal(grads[0][1], grads[1][1])


def _norm_inputs(shape, dtype, dev, seed, wdtype=None):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=gen)
    z = torch.randn(*shape, generator=gen) * 2
    w = 1 + 0.3 * torch.randn(shape[-1], generator=gen)
    return x.to(dev, dtype), z.to(dev, dtype), w.to(dev, wdtype or dtype)


def _ref_norm(x, z, w, eps=1e-5):
    """The reference's RMSNormGated.forward expression (gdn2.py:449-452)."""
    variance = x.pow(2).mean(-1, keepdim=True)
    normed = x * torch.rsqrt(variance + eps) * w
    return normed * F.silu(z)


@pytest.mark.parametrize("N", [8, 32, 64, 128, 200, 256])
def test_gated_norm_fp32_forward_backward(cuda_device, N):
    from qwendopamine_b200.gdn2_ops.block_ops import gated_rms_norm

    x, z, w = _norm_inputs((3, 77, 5, N), torch.float32, cuda_device, seed=N)
    x.requires_grad_()
    z.requires_grad_()
    w.requires_grad_()
    y = gated_rms_norm(x, z, w)
    assert rel(y, BO.gated_norm_fwd(np64(x), np64(z), np64(w))) < 1e-5
    dy = torch.randn_like(y)
    (y * dy).sum().backward()
    dx, dz, dw = BO.gated_norm_bwd(np64(x), np64(z), np64(w), np64(dy))
    assert rel(x.grad, dx) < 1e-5
    assert rel(z.grad, dz) < 1e-5
    assert rel(w.grad, dw) < 1e-5


@pytest.mark.parametrize("wdtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("N", [64, 128])
def test_gated_norm_bf16_matches_torch_cuda_expression(cuda_device, wdtype, N):
    """Input-dtype evaluation: bit-for-bit against torch's CUDA kernels running
    the reference's expression, and against the rounding restatement."""
    from qwendopamine_b200.gdn2_ops.block_ops import gated_rms_norm

    x, z, w = _norm_inputs((8, 512, 16, N), torch.bfloat16, cuda_device, seed=N + 1, wdtype=wdtype)
    y = gated_rms_norm(x, z, w)
    ref = _ref_norm(x, z, w)
    assert y.dtype == ref.dtype
    if y.dtype == torch.bfloat16:
        steps = bf16_steps(y, ref)
        assert steps.max() <= 1 and (steps == 0).float().mean() > 0.999
    else:
        assert rel(y, ref) < 1e-6
    xs, zs = x[:2, :16].float().cpu().numpy(), z[:2, :16].float().cpu().numpy()
    oy = BO.gated_norm_fwd_rounded(xs, zs, w.float().cpu().numpy(),
                                   weight_fp32=wdtype == torch.float32)
    assert (y[:2, :16].float().cpu().numpy() == oy).mean() > 0.99


def test_gated_norm_under_autocast_matches_reference(cuda_device):
    """Under CUDA autocast the reference's pow / rsqrt run in fp32 and its
    result is fp32; the module's kernel follows (fp32_math)."""
    from qwendopamine_b200 import RMSNormGated

    x, z, _ = _norm_inputs((4, 256, 8, 128), torch.bfloat16, cuda_device, seed=9)
    m = RMSNormGated(128).to(cuda_device)
    with torch.no_grad():
        m.weight.normal_(1.0, 0.3)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = m(x, z)
        ref = _ref_norm(x, z, m.weight)
    assert y.dtype == ref.dtype == torch.float32
    assert rel(y, ref) < 1e-6
    xg = x.clone().requires_grad_()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = m(xg, z)
    dy = torch.randn_like(y)
    (y * dy).sum().backward()
    dx, _, dw = BO.gated_norm_bwd(np64(x), np64(z), np64(m.weight), np64(dy))
    assert rel(xg.grad, dx) < 2e-2
    assert rel(m.weight.grad, dw) < 1e-3


def test_gated_norm_bf16_backward_and_determinism(cuda_device):
    from qwendopamine_b200.gdn2_ops.block_ops import gated_rms_norm

    x, z, w = _norm_inputs((4, 300, 16, 128), torch.bfloat16, cuda_device, seed=2)
    gen = torch.Generator().manual_seed(4)
    dy = torch.randn(x.shape, generator=gen).to(cuda_device, torch.bfloat16)
    outs = []
    for _ in range(2):
        xg, zg, wg = (t.clone().requires_grad_() for t in (x, z, w))
        y = gated_rms_norm(xg, zg, wg)
        (y.float() * dy.float()).sum().backward()
        outs.append((xg.grad, zg.grad, wg.grad))
    dx, dz, dw = BO.gated_norm_bwd(np64(x), np64(z), np64(w), np64(dy))
    assert rel(outs[0][0], dx) < 2e-2
    assert rel(outs[0][1], dz) < 2e-2
    assert rel(outs[0][2], dw) < 2e-2
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_gated_norm_empty_rows(cuda_device):
    from qwendopamine_b200.gdn2_ops.block_ops import gated_rms_norm

    x, z, w = _norm_inputs((0, 64), torch.float32, cuda_device, seed=1)
    w.requires_grad_()
    y = gated_rms_norm(x, z, w)
    assert y.shape == (0, 64)
    y.sum().backward()
    assert torch.equal(w.grad, torch.zeros_like(w))


class _ThreadGather:
    """All-gather among ``world`` threads of one process (emulated ranks)."""

    def __init__(self, world):
        import threading

        self.world = world
        self.slots = [None] * world
        self.barrier = threading.Barrier(world, timeout=60)

    def __call__(self, rank):
        def gather(t):
            torch.cuda.synchronize()
            self.slots[rank] = t
            self.barrier.wait()
            out = torch.stack([s.to(t.device) for s in self.slots])
            self.barrier.wait()
            return out
        return gather


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_short_conv_sequence_parallel_equals_single_device(cuda_device, dtype):
    """short_conv_cp over 3 emulated ranks (threads, one GPU) gives the spans
    of the single-device convolution.  Gradients: each span's local backward
    with the halo as a prefix, plus the prefix gradient returned to the
    previous span (the routing ConvHaloFunction does over a process group,
    tested over gloo in test_cp_gloo.py), equal the single-device dx; the
    spans' weight / bias gradients sum to the single-device ones.  (The
    emulation stops at the forward: on one GPU every rank's backward runs on
    torch's one autograd thread per device, so a blocking gather there
    cannot be emulated.)"""
    import threading

    from qwendopamine_b200.gdn2_ops.block_ops import short_conv
    from qwendopamine_b200.gdn2_ops.cp import short_conv_cp

    world, B, T, D, W = 3, 2, 3 * 50, 256, 4
    x, w, b = _conv_inputs(B, T, D, W, True, dtype, cuda_device, seed=21)
    dy = torch.randn(B, T, D, device=cuda_device).to(dtype)
    xf, wf, bf = (t.clone().requires_grad_() for t in (x, w, b))
    yf, _ = short_conv(xf, wf, bf)
    (yf.float() * dy.float()).sum().backward()
    span = T // world

    gat = _ThreadGather(world)
    outs, errs = [None] * world, []

    def run(r):
        try:
            torch.cuda.set_device(cuda_device)
            with torch.no_grad():
                outs[r] = short_conv_cp(x[:, r * span:(r + 1) * span], w, b, rank=r, world=world,
                                        gather=gat(r))
            torch.cuda.synchronize()
        except Exception as exc:  # surfaced below
            errs.append(exc)
            gat.barrier.abort()

    ths = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in ths:
        t.start()
    for t in ths:
        t.join(timeout=120)
    assert not errs, errs
    assert torch.equal(torch.cat(outs, 1), yf.detach())

    dxs, dws, dbs, dpres = [], [], [], []
    for r in range(world):
        xs = x[:, r * span:(r + 1) * span].clone().requires_grad_()
        ws, bs = w.clone().requires_grad_(), b.clone().requires_grad_()
        pre = (x[:, r * span - (W - 1):r * span] if r else torch.zeros_like(x[:, :W - 1]))
        pre = pre.clone().requires_grad_()
        y, _ = short_conv(xs, ws, bs, prefix=pre)
        (y.float() * dy[:, r * span:(r + 1) * span].float()).sum().backward()
        dxs.append(xs.grad.float())
        dws.append(ws.grad.float())
        dbs.append(bs.grad.float())
        dpres.append(pre.grad.float())
    for r in range(world - 1):  # the next span's prefix gradient belongs to this span's tail
        dxs[r][:, -(W - 1):] += dpres[r + 1]
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert rel(torch.cat(dxs, 1), xf.grad) < tol
    assert rel(sum(dws), wf.grad.float()) < tol
    assert rel(sum(dbs), bf.grad.float()) < tol

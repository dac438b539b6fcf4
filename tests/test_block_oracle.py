"""The block prologue / epilogue oracle (oracle/block_oracle.py) against the
reference's own ShortConvolution and RMSNormGated outputs and autograd
gradients (tests/golden/block_ops.npz, made by tests/golden/make_golden.py).
CPU only."""

import os

import numpy as np
import pytest

from oracle import block_oracle as BO

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def gold():
    return np.load(os.path.join(GOLD, "block_ops.npz"))


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def bf16_ulps(a, b):
    """Per-element distance in bfloat16 units of the last place."""
    ia = np.asarray(a, np.float32).view(np.int32).astype(np.int64) >> 16
    ib = np.asarray(b, np.float32).view(np.int32).astype(np.int64) >> 16
    return np.abs(ia - ib)


@pytest.mark.parametrize("tag,act", [("a", "silu"), ("b", None)])
def test_conv_forward_backward_match_reference(gold, tag, act):
    g = {k[len(f"conv_{tag}_"):]: gold[k] for k in gold.files if k.startswith(f"conv_{tag}_")}
    bias = g.get("bias")
    y = BO.conv_fwd(g["x"], g["w"], bias, activation=act)
    assert rel(y, g["y"]) < 1e-6
    dx, dw, db, _ = BO.conv_bwd(g["x"], g["w"], g["dy"], bias, activation=act)
    assert rel(dx, g["dx"]) < 1e-6
    assert rel(dw, g["dw"].reshape(dw.shape)) < 1e-6
    if bias is not None:
        assert rel(db, g["dbias"]) < 1e-6
    W = g["w"].shape[-1]
    # the reference's prefill cache: the last W-1 inputs, [B, D, W-1]
    assert np.array_equal(g["cache"], g["x"][:, -(W - 1):].transpose(0, 2, 1))


def test_conv_decode_step_matches_reference(gold):
    cache, x = gold["conv_dec_cache"], gold["conv_dec_x"]
    y = BO.conv_fwd(x, gold["conv_a_w"], gold["conv_a_bias"], prefix=cache.transpose(0, 2, 1))
    assert rel(y, gold["conv_dec_y"]) < 1e-6
    new = np.concatenate([cache, x.transpose(0, 2, 1)], axis=-1)[:, :, 1:]
    assert np.array_equal(new, gold["conv_dec_new_cache"])


def test_conv_bf16_rounding_matches_reference(gold):
    """bf16: the convolution's output is rounded to bf16 before the SiLU and
    the SiLU's result again."""
    x = BO.bf16_round(gold["conv_a_x"])
    c = BO.conv_fwd(x, gold["conv_bf16_w"], gold["conv_bf16_bias"], activation=None)
    c = BO.bf16_round(c.astype(np.float32))
    y = BO.bf16_round((c / (1 + np.exp(-c))).astype(np.float32))
    u = bf16_ulps(y, gold["conv_bf16_y"])
    assert u.max() <= 1 and (u == 0).mean() > 0.99


def test_gated_norm_fp32_matches_reference(gold):
    y = BO.gated_norm_fwd(gold["norm_x"], gold["norm_z"], gold["norm_w"])
    assert rel(y, gold["norm_y"]) < 1e-6
    dx, dz, dw = BO.gated_norm_bwd(gold["norm_x"], gold["norm_z"], gold["norm_w"], gold["norm_dy"])
    assert rel(dx, gold["norm_dx"]) < 1e-5
    assert rel(dz, gold["norm_dz"]) < 1e-6
    assert rel(dw, gold["norm_dw"]) < 1e-6


@pytest.mark.parametrize("w32", [False, True])
def test_gated_norm_bf16_rounding_matches_reference(gold, w32):
    """Every rounding step restated.  The fixture is a CPU run, whose bf16
    rsqrt sometimes rounds twice (one bf16 step off in r for those rows), so
    most rows agree bit for bit and the rest sit within that step of r and
    the roundings after it (< 2 %); the GPU tests check the single-rounding
    form bit-exactly against torch's CUDA evaluation of the same expression."""
    y = BO.gated_norm_fwd_rounded(gold["norm_x"], gold["norm_z"],
                                  gold["norm_w"] if w32 else gold["norm_bf16_w"], weight_fp32=w32)
    ref = gold["norm_bf16w32_y" if w32 else "norm_bf16_y"]
    rows_same = (y == ref).reshape(-1, y.shape[-1]).all(axis=1).mean()
    assert rows_same > 0.85, rows_same
    assert np.all(np.abs(y - ref) <= 0.02 * np.abs(ref) + 1e-6)

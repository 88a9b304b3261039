"""Encoder self-attention prefill on the GPU against the reference's CPU attention.

Reference routines: attention_head_flash (tensor.c:286-332), attention_head
(tensor.c:255-282), the live encoder loop encoder.c:166-205.
"""
import numpy as np
import pytest

import cases
import nllb_attn as na
import pyoracle as po
from helpers import assert_attn_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx(cuda_device):
    c = na.Context(0, n_layers=0, n_heads=16, max_sentences=0, n_beams=4, max_tgt=0, max_src=0)
    yield c
    c.close()


def run_prefill(ctx, q, k, v, valid_len=None, mask=None, mask_strides=(0, 0), scale=0.125):
    import torch
    B, H, S, _ = q.shape
    dq, dk, dv = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (q, k, v))
    dout = torch.full_like(dq, float("nan"))
    dvl = None if valid_len is None else torch.from_numpy(np.asarray(valid_len, np.int32)).cuda()
    dm = None if mask is None else torch.from_numpy(np.ascontiguousarray(mask, np.float32)).cuda()
    args = ctx.prefill_args(dq, dk, dv, dout, B, H, S, (H * S * 64, S * 64, 64), dvl, dm,
                            mask_strides, scale)
    ctx.prefill(args)
    ctx.sync()
    return dout.cpu().numpy()


@pytest.mark.parametrize("name", cases.PREFILL_CASES)
def test_prefill_golden(ctx, name):
    q, k, v, vl = cases.prefill_case(name)
    out = run_prefill(ctx, q, k, v, vl)
    assert_attn_close(out, cases.load_golden()[name], name)


def test_prefill_config1_full():
    """Q,K,V [8,16,128,64] N(0,1), scale 1/8, last 0-31 keys masked per sequence."""
    rng = np.random.default_rng(1)
    B, H, S = 8, 16, 128
    q, k, v = (rng.standard_normal((B, H, S, 64), dtype=np.float32) for _ in range(3))
    vl = (S - rng.integers(0, 32, size=B)).astype(np.int32)
    c = na.Context(0, n_layers=0, max_sentences=0)
    try:
        out = run_prefill(c, q, k, v, vl)
    finally:
        c.close()
    assert_attn_close(out, po.prefill(q, k, v, vl), "config1")


@pytest.mark.parametrize("S", [1, 2, 32, 33, 63, 64, 65, 128, 129, 130, 255, 256, 257, 300, 512])
def test_prefill_lengths(ctx, S):
    rng = np.random.default_rng(S)
    q, k, v = (rng.standard_normal((2, 3, S, 64), dtype=np.float32) for _ in range(3))
    vl = np.array([S, max(1, S // 3)], np.int32)
    assert_attn_close(run_prefill(ctx, q, k, v, vl), po.prefill(q, k, v, vl), f"S={S}")


def test_prefill_interleaved_rows(ctx):
    """The engine's layout: rows [S][n_heads*64], head h at cols 64h (encoder.c:171-178)."""
    import torch
    rng = np.random.default_rng(7)
    S, H = 50, 16
    Q, K, V = (rng.standard_normal((S, H * 64), dtype=np.float32) for _ in range(3))
    strides = (S * H * 64, 64, H * 64)
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (Q, K, V))
    dout = torch.zeros_like(dq)
    ctx.prefill(ctx.prefill_args(dq, dk, dv, dout, 1, H, S, strides))
    ctx.sync()
    ref = po.prefill(Q, K, V, None, strides=strides, shape=(1, H, S))
    assert_attn_close(dout.cpu().numpy(), ref, "interleaved")


def test_prefill_additive_mask_per_head(ctx):
    rng = np.random.default_rng(11)
    B, H, S = 2, 2, 70
    q, k, v = (rng.standard_normal((B, H, S, 64), dtype=np.float32) for _ in range(3))
    mask = np.where(rng.random((B, H, S, S)) < 0.3, -1e9, rng.normal(0, 0.5, (B, H, S, S)))
    mask = mask.astype(np.float32)
    mask[..., 0] = 0.0
    ms = (H * S * S, S * S)
    out = run_prefill(ctx, q, k, v, None, mask, ms)
    ref = po.prefill(q, k, v, None, mask=mask, mask_strides=ms)
    assert_attn_close(out, ref, "mask")


@pytest.mark.parametrize("S", [9, 100])
def test_prefill_all_keys_masked_is_mean_of_v(ctx, S):
    """valid_len 0: the reference's -1e9 on every key gives equal weights
    (S=9 runs on the FFMA kernel, S=100 on the tensor-core kernel)."""
    rng = np.random.default_rng(12)
    q, k, v = (rng.standard_normal((2, 1, S, 64), dtype=np.float32) for _ in range(3))
    vl = np.array([0, S - 3], np.int32)
    out = run_prefill(ctx, q, k, v, vl)
    assert_attn_close(out, po.prefill(q, k, v, vl), "all masked")
    assert_attn_close(out[0, 0, 3], v[0, 0].mean(axis=0), "mean")


def test_prefill_large_values_keep_fp32_accuracy(ctx):
    """Scores far from zero (|q.k/8| ~ 30): the 3xTF32 split keeps softmax
    weights at fp32 accuracy where single-pass TF32 would not."""
    rng = np.random.default_rng(13)
    q, k, v = (3.0 * rng.standard_normal((1, 4, 128, 64), dtype=np.float32) for _ in range(3))
    assert_attn_close(run_prefill(ctx, q, k, v), po.prefill(q, k, v), "large")


def test_prefill_host_variant(ctx):
    q, k, v, vl = cases.prefill_case("prefill_small")
    out = np.zeros_like(q)
    B, H, S, _ = q.shape
    ctx.prefill_host(ctx.prefill_args(q, k, v, out, B, H, S, (H * S * 64, S * 64, 64), vl))
    assert_attn_close(out, cases.load_golden()["prefill_small"], "host")


def test_dropins_match_reference_single_head(cuda_device):
    Q, K, V, mask = cases.head_mask_case()
    g = cases.load_golden()
    out = np.zeros_like(Q)
    assert na.attention_head_flash(Q, K, V, mask, out, Q.shape[0]) == na.OK
    assert_attn_close(out, g["head_flash_mask"], "attention_head_flash")
    out2 = np.zeros_like(Q)
    scratch = np.zeros((Q.shape[0], Q.shape[0]), np.float32)
    assert na.attention_head(Q, K, V, mask, out2, scratch, Q.shape[0]) == na.OK
    assert_attn_close(out2, g["head_mask"], "attention_head")
    # the softmaxed scores the reference leaves in scores_buf (tensor.c:258-277)
    assert_attn_close(scratch, g["head_mask_scores"], "attention_head scores_buf")
    out3 = np.zeros_like(Q)
    assert na.attention_head_flash(Q, K, V, None, out3, Q.shape[0]) == na.OK
    assert_attn_close(out3, po.attention_head_flash(Q, K, V, None), "no mask")


def test_dropin_rejects_other_head_dims(cuda_device):
    q = np.zeros((4, 32), np.float32)
    out = np.full_like(q, 3.0)
    assert na.attention_head_flash(q, q, q, None, out, 4, 32) == na.EINVAL
    assert (out == 3.0).all()


def test_prefill_argument_errors(ctx):
    import torch
    x = torch.zeros(1, 1, 8, 64, device="cuda")
    bad = [
        dict(seq_len=0), dict(batch=0), dict(strides=(512, 512, 62)),
    ]
    for kw in bad:
        a = ctx.prefill_args(x, x, x, x, kw.get("batch", 1), 1, kw.get("seq_len", 8),
                             kw.get("strides", (512, 512, 64)))
        with pytest.raises(na.NllbAttnError) as ei:
            ctx.prefill(a)
        assert ei.value.status == na.EINVAL
    shifted = torch.zeros(8 * 64 + 1, device="cuda")[1:]  # contiguous, 4 bytes off 16-byte alignment
    a = ctx.prefill_args(shifted, x, x, x, 1, 1, 8, (512, 512, 64))
    with pytest.raises(na.NllbAttnError) as ei:
        ctx.prefill(a)
    assert ei.value.status == na.EINVAL

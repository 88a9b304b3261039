"""Decoder self-attention over the per-beam KV cache and cross-attention on the
GPU, against the reference's CPU attention.

Reference routines: decoder_self_attn_cached (decoder.c:48-99) with the beam
reorder by cache copy (main.c:462-488); decoder_cross_attn_cached
(decoder.c:103-152).
"""
import numpy as np
import pytest

import cases
import nllb_attn as na
import pyoracle as po
from helpers import assert_attn_close

pytestmark = pytest.mark.gpu


def gpu_decode_sweep(ctx, q, k, v, parents, layer=0, n_sent=1):
    """q,k,v: [T][n_sent][NB][H*64]; parents [T][n_sent][NB] or None."""
    import torch
    T = q.shape[0]
    dq, dk, dv = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (q, k, v))
    dout = torch.full_like(dq, float("nan"))
    dpar = None if parents is None else torch.from_numpy(np.ascontiguousarray(parents, np.int32)).cuda()
    for t in range(T):
        if dpar is not None:
            ctx.reorder(n_sent, dpar[t])
        ctx.decode_self(layer, t, n_sent, dq[t], dk[t], dv[t], dout[t])
    ctx.sync()
    return dout.cpu().numpy()


@pytest.mark.parametrize("name", sorted(cases.DECODE_CASES))
def test_decode_golden(cuda_device, name):
    q, k, v, parents = cases.decode_case(name)
    T = q.shape[0]
    with na.Context(0, n_layers=1, n_heads=16, max_sentences=1, n_beams=4, max_tgt=T,
                    max_src=1) as ctx:
        out = gpu_decode_sweep(ctx, q[:, None], k[:, None], v[:, None], parents[:, None])[:, 0]
    steps = list(cases.DECODE_CASES[name])
    assert_attn_close(out[steps], cases.load_golden()[name], name)
    assert_attn_close(out, po.decode_sweep(q, k, v, parents), name + " all steps")


def test_decode_config2_normal_inputs(cuda_device):
    """4 beams x 16 heads x 64, cache 1 -> 256, N(0,1), random permutation each step."""
    rng = np.random.default_rng(2)
    T, NB = 256, 4
    q, k, v = (rng.standard_normal((T, NB, 1024), dtype=np.float32) for _ in range(3))
    parents = np.stack([rng.permutation(NB) for _ in range(T)]).astype(np.int32)
    with na.Context(0, n_layers=1, max_sentences=1, n_beams=NB, max_tgt=T, max_src=1) as ctx:
        out = gpu_decode_sweep(ctx, q[:, None], k[:, None], v[:, None], parents[:, None])[:, 0]
    assert_attn_close(out, po.decode_sweep(q, k, v, parents), "config2")


@pytest.mark.parametrize("n_beams", [1, 2, 8])
def test_decode_other_beam_counts(cuda_device, n_beams):
    rng = np.random.default_rng(30 + n_beams)
    T = 70
    q, k, v = (rng.standard_normal((T, n_beams, 1024), dtype=np.float32) for _ in range(3))
    parents = rng.integers(0, n_beams, size=(T, n_beams)).astype(np.int32)
    with na.Context(0, n_layers=1, max_sentences=1, n_beams=n_beams, max_tgt=T, max_src=1) as ctx:
        out = gpu_decode_sweep(ctx, q[:, None], k[:, None], v[:, None], parents[:, None])[:, 0]
    assert_attn_close(out, po.decode_sweep(q, k, v, parents), f"beams={n_beams}")


@pytest.mark.parametrize("n_sent", [3, 40])
def test_decode_many_sentences_two_layers(cuda_device, n_sent):
    """Sentences keep independent histories; layers keep independent caches.
    40 sentences x 16 heads fill the GPU without splitting; 3 sentences split."""
    rng = np.random.default_rng(40 + n_sent)
    T, NB, L = 45, 4, 2
    shape = (L, T, n_sent, NB, 1024)
    q, k, v = (rng.standard_normal(shape, dtype=np.float32) for _ in range(3))
    parents = rng.integers(0, NB, size=(T, n_sent, NB)).astype(np.int32)
    import torch
    with na.Context(0, n_layers=L, max_sentences=n_sent + 1, n_beams=NB, max_tgt=T,
                    max_src=1) as ctx:
        dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
        dout = torch.zeros_like(dq)
        dpar = torch.from_numpy(parents).cuda()
        for t in range(T):
            ctx.reorder(n_sent, dpar[t])
            for layer in range(L):  # reorder once per step, then every layer
                ctx.decode_self(layer, t, n_sent, dq[layer, t], dk[layer, t], dv[layer, t],
                                dout[layer, t])
        ctx.sync()
        out = dout.cpu().numpy()
    for layer in range(L):
        for s in range(0, n_sent, max(1, n_sent // 5)):
            ref = po.decode_sweep(q[layer, :, s], k[layer, :, s], v[layer, :, s], parents[:, s])
            assert_attn_close(out[layer, :, s], ref, f"layer {layer} sentence {s}")


def test_decode_host_variant_and_reorder_host(cuda_device):
    q, k, v, parents = cases.decode_case("decode_dup40")
    T = q.shape[0]
    out = np.zeros_like(q)
    with na.Context(0, n_layers=1, max_sentences=1, n_beams=4, max_tgt=T, max_src=1) as ctx:
        for t in range(T):
            ctx.reorder_host(1, np.ascontiguousarray(parents[t]))
            ctx.decode_self_host(0, t, 1, np.ascontiguousarray(q[t]), np.ascontiguousarray(k[t]),
                                 np.ascontiguousarray(v[t]), out[t])
    steps = list(cases.DECODE_CASES["decode_dup40"])
    assert_attn_close(out[steps], cases.load_golden()["decode_dup40"], "host")


def test_decode_errors(cuda_device):
    import torch
    with na.Context(0, n_layers=1, max_sentences=2, n_beams=4, max_tgt=8, max_src=4) as ctx:
        x = torch.zeros(2, 4, 1024, device="cuda")
        for args, status in [((1, 0, 1), na.EINVAL), ((0, 8, 1), na.ECAPACITY),
                             ((0, 0, 3), na.ECAPACITY), ((0, -1, 1), na.EINVAL),
                             ((0, 0, 0), na.EINVAL)]:
            with pytest.raises(na.NllbAttnError) as ei:
                ctx.decode_self(*args, x, x, x, x)
            assert ei.value.status == status, args
        with pytest.raises(na.NllbAttnError) as ei:
            ctx.reorder_host(1, np.array([0, 1, 4, 0], np.int32))
        assert ei.value.status == na.EINVAL
        # an out-of-range parent that only the device sees: flagged, not applied
        bad = torch.tensor([0, 1, 9, 0], dtype=torch.int32, device="cuda")
        ctx.reorder(1, bad)
        with pytest.raises(na.NllbAttnError) as ei:
            ctx.sync()
        assert ei.value.status == na.EINVAL
        ctx.sync()  # the error word was cleared
        with pytest.raises(na.NllbAttnError) as ei:
            ctx.cross(0, 1, x, x)
        assert ei.value.status == na.ESTATE


def test_reorder_applied_in_the_decode_launch(cuda_device):
    """With every sentence of the context in the call, a pending reorder is
    applied by the self-attention launch itself (no reorder kernel); with a
    spare sentence slot the reorder kernel runs first.  Both must give the
    same results, bit for bit, and the oracle's."""
    rng = np.random.default_rng(77)
    T, NB, S = 60, 4, 3
    q, k, v = (rng.standard_normal((T, S, NB, 1024), dtype=np.float32) for _ in range(3))
    parents = rng.integers(0, NB, size=(T, S, NB)).astype(np.int32)
    outs = []
    for max_sent in (S, S + 1):
        with na.Context(0, n_layers=1, max_sentences=max_sent, n_beams=NB, max_tgt=T, max_src=1) as ctx:
            outs.append(gpu_decode_sweep(ctx, q, k, v, parents, n_sent=S))
    assert np.array_equal(outs[0], outs[1])
    for s in range(S):
        assert_attn_close(outs[0][:, s], po.decode_sweep(q[:, s], k[:, s], v[:, s], parents[:, s]), f"sentence {s}")


def test_bad_parent_seen_by_the_decode_launch(cuda_device):
    """An out-of-range parent applied inside the self-attention launch is
    flagged like the reorder kernel flags it."""
    import torch
    with na.Context(0, n_layers=1, max_sentences=1, n_beams=4, max_tgt=8, max_src=4) as ctx:
        x = torch.zeros(1, 4, 1024, device="cuda")
        ctx.decode_self(0, 0, 1, x, x, x, x)
        bad = torch.tensor([0, 5, 1, 2], dtype=torch.int32, device="cuda")
        ctx.reorder(1, bad)
        ctx.decode_self(0, 1, 1, x, x, x, x)
        with pytest.raises(na.NllbAttnError) as ei:
            ctx.sync()
        assert ei.value.status == na.EINVAL


@pytest.mark.parametrize("n_sent", [1, 40])
def test_bounded_wait_runs_out_and_context_recovers(cuda_device, n_sent):
    """The self-attention launch's wait for a cache chunk runs out (a chunk
    that is never requested, ~1 ms budget): the call reports
    NLLB_ATTN_ETIMEOUT, and the same step made again on the same context gives
    the oracle's outputs, as do the steps after it.  1 sentence splits the
    cache over a cluster of CTAs; 40 sentences do not split."""
    import torch
    rng = np.random.default_rng(91 + n_sent)
    T, NB, t_out = 24, 4, 17
    q, k, v = (rng.standard_normal((T, n_sent, NB, 1024), dtype=np.float32) for _ in range(3))
    parents = rng.integers(0, NB, size=(T, n_sent, NB)).astype(np.int32)
    with na.Context(0, n_layers=1, max_sentences=n_sent, n_beams=NB, max_tgt=T, max_src=1) as ctx:
        dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
        dout = torch.zeros_like(dq)
        dpar = torch.from_numpy(parents).cuda()
        for t in range(T):
            ctx.reorder(n_sent, dpar[t])
            if t == t_out:
                ctx.test_expire_next_wait()
                ctx.decode_self(0, t, n_sent, dq[t], dk[t], dv[t], dout[t])
                with pytest.raises(na.NllbAttnError) as ei:
                    ctx.sync()
                assert ei.value.status == na.ETIMEOUT
            ctx.decode_self(0, t, n_sent, dq[t], dk[t], dv[t], dout[t])
        ctx.sync()
        out = dout.cpu().numpy()
    for s in range(0, n_sent, max(1, n_sent // 4)):
        assert_attn_close(out[:, s], po.decode_sweep(q[:, s], k[:, s], v[:, s], parents[:, s]), f"sentence {s}")


# ---------------------------------------------------------------------------
# cross-attention
# ---------------------------------------------------------------------------
def gpu_cross(ctx, K, V, q, layer=0):
    """K,V: [n_src][1024] engine rows; q: [steps][NB][1024] (sentence 0)."""
    import torch
    n_src = K.shape[0]
    dK, dV = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (K, V))
    ctx.set_memory(layer, 0, n_src, dK, dV, 64, 1024)
    dq = torch.from_numpy(np.ascontiguousarray(q)).cuda()
    dout = torch.full_like(dq, float("nan"))
    for t in range(q.shape[0]):
        ctx.cross(layer, 1, dq[t], dout[t])
    ctx.sync()
    return dout.cpu().numpy()


@pytest.mark.parametrize("name", cases.CROSS_CASES)
def test_cross_golden(cuda_device, name):
    K, V, q = cases.cross_case(name)
    with na.Context(0, n_layers=1, max_sentences=1, n_beams=4, max_tgt=4, max_src=512) as ctx:
        out = gpu_cross(ctx, K, V, q)
    assert_attn_close(out, cases.load_golden()[name], name)


def test_cross_config3_head_major_memory(cuda_device):
    """Q [4,16,1,64] per step, memory K/V [16,512,64] N(0,1), 128 steps, memory resident."""
    import torch
    rng = np.random.default_rng(3)
    H, n_src, T, NB = 16, 512, 128, 4
    Km, Vm = (rng.standard_normal((H, n_src, 64), dtype=np.float32) for _ in range(2))
    q = rng.standard_normal((T, NB, H, 64), dtype=np.float32)
    with na.Context(0, n_layers=1, max_sentences=1, n_beams=NB, max_tgt=4, max_src=n_src) as ctx:
        dK, dV = torch.from_numpy(Km).cuda(), torch.from_numpy(Vm).cuda()
        ctx.set_memory(0, 0, n_src, dK, dV, n_src * 64, 64)  # [H][n_src][64]
        dq = torch.from_numpy(q.reshape(T, NB, H * 64)).cuda()
        dout = torch.zeros_like(dq)
        for t in range(T):
            ctx.cross(0, 1, dq[t], dout[t])
        ctx.sync()
        out = dout.cpu().numpy()
    K_rows = np.ascontiguousarray(Km.transpose(1, 0, 2).reshape(n_src, H * 64))
    V_rows = np.ascontiguousarray(Vm.transpose(1, 0, 2).reshape(n_src, H * 64))
    assert_attn_close(out, po.cross(K_rows, V_rows, q.reshape(T, NB, H * 64)), "config3")


def test_cross_ragged_sentences_and_layers(cuda_device):
    import torch
    rng = np.random.default_rng(5)
    lens = [18, 130, 1, 64, 65, 97]
    L, NB = 2, 4
    n_sent = len(lens)
    with na.Context(0, n_layers=L, max_sentences=n_sent, n_beams=NB, max_tgt=4, max_src=130) as ctx:
        mem = {}
        for layer in range(L):
            for s, n in enumerate(lens):
                K, V = (rng.standard_normal((n, 1024), dtype=np.float32) for _ in range(2))
                mem[layer, s] = (K, V)
                ctx.set_memory_host(layer, s, n, K, V, 64, 1024)
        q = rng.standard_normal((L, n_sent, NB, 1024), dtype=np.float32)
        dq = torch.from_numpy(q).cuda()
        dout = torch.zeros_like(dq)
        for layer in range(L):
            ctx.cross(layer, n_sent, dq[layer], dout[layer])
        ctx.sync()
        out = dout.cpu().numpy()
        out_host = np.zeros_like(q[1])
        ctx.cross_host(1, n_sent, np.ascontiguousarray(q[1]), out_host)
    for layer in range(L):
        for s in range(n_sent):
            K, V = mem[layer, s]
            assert_attn_close(out[layer, s], po.cross(K, V, q[layer, s]), f"l{layer} s{s}")
    np.testing.assert_array_equal(out_host, out[1])


@pytest.mark.parametrize("n_sent", [1, 40])
def test_cross_bounded_wait_runs_out_and_context_recovers(cuda_device, n_sent):
    """The cross-attention launch's wait for a memory chunk runs out (a chunk
    that is never requested, ~1 ms budget): the sync reports
    NLLB_ATTN_ETIMEOUT, nothing is written, and the same call made again on
    the same context gives the oracle's outputs.  1 sentence splits the
    memory over a cluster of CTAs; 40 sentences do not split."""
    import torch
    rng = np.random.default_rng(95 + n_sent)
    NB, n_src = 4, 100
    with na.Context(0, n_layers=1, max_sentences=n_sent, n_beams=NB, max_tgt=4, max_src=n_src) as ctx:
        mem = []
        for s in range(n_sent):
            K, V = (rng.standard_normal((n_src, 1024), dtype=np.float32) for _ in range(2))
            mem.append((K, V))
            ctx.set_memory_host(0, s, n_src, K, V, 64, 1024)
        q = rng.standard_normal((n_sent, NB, 1024), dtype=np.float32)
        dq = torch.from_numpy(q).cuda()
        dout = torch.full_like(dq, 7.0)
        ctx.test_expire_next_cross_wait()
        ctx.cross(0, n_sent, dq, dout)
        with pytest.raises(na.NllbAttnError) as ei:
            ctx.sync()
        assert ei.value.status == na.ETIMEOUT
        assert bool((dout == 7.0).all()), "the timed-out launch wrote output"
        ctx.cross(0, n_sent, dq, dout)
        ctx.sync()
        out = dout.cpu().numpy()
    for s in range(0, n_sent, max(1, n_sent // 4)):
        K, V = mem[s]
        assert_attn_close(out[s], po.cross(K, V, q[s]), f"s{s}")


def test_cross_many_sentences_no_split(cuda_device):
    import torch
    rng = np.random.default_rng(6)
    n_sent, n_src, NB = 64, 40, 4
    with na.Context(0, n_layers=1, max_sentences=n_sent, n_beams=NB, max_tgt=4, max_src=n_src) as ctx:
        K = rng.standard_normal((n_sent, n_src, 1024), dtype=np.float32)
        V = rng.standard_normal((n_sent, n_src, 1024), dtype=np.float32)
        dK, dV = torch.from_numpy(K).cuda(), torch.from_numpy(V).cuda()
        for s in range(n_sent):
            ctx.set_memory(0, s, n_src, dK[s], dV[s], 64, 1024)
        q = rng.standard_normal((n_sent, NB, 1024), dtype=np.float32)
        dq = torch.from_numpy(q).cuda()
        dout = torch.zeros_like(dq)
        ctx.cross(0, n_sent, dq, dout)
        ctx.sync()
        out = dout.cpu().numpy()
    for s in (0, 17, 63):
        assert_attn_close(out[s], po.cross(K[s], V[s], q[s]), f"s{s}")


@pytest.mark.parametrize("max_len", [130, 200])
def test_cross_many_ragged_sentences(cuda_device, max_len):
    """72 sentences (no split-KV) with memories of every length from 1 up
    (16-row chunks up to 160 rows, 32-row chunks beyond): every sentence
    against the oracle."""
    import torch
    rng = np.random.default_rng(7 + max_len)
    NB = 4
    lens = [1, 2, 15, 16, 17, max_len] + [int(x) for x in rng.integers(1, max_len + 1, size=66)]
    n_sent = len(lens)
    with na.Context(0, n_layers=1, max_sentences=n_sent, n_beams=NB, max_tgt=4, max_src=max_len) as ctx:
        mem = []
        for s, n in enumerate(lens):
            K, V = (rng.standard_normal((n, 1024), dtype=np.float32) for _ in range(2))
            mem.append((K, V))
            ctx.set_memory_host(0, s, n, K, V, 64, 1024)
        q = rng.standard_normal((n_sent, NB, 1024), dtype=np.float32)
        dq = torch.from_numpy(q).cuda()
        dout = torch.zeros_like(dq)
        ctx.cross(0, n_sent, dq, dout)
        ctx.sync()
        out = dout.cpu().numpy()
    for s in range(n_sent):
        K, V = mem[s]
        assert_attn_close(out[s], po.cross(K, V, q[s]), f"s{s} len {lens[s]}")

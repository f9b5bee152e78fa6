"""Decode-step linears (one launch each: cluster split-K + finisher) against
fp32 references of the same bf16 inputs and against the unfused operator
sequence.

The input norm is applied inside the kernel from the block statistics of the
producing residual linear, so its rstd can differ from the row-norm kernel's
in the last bits (summation order): those comparisons use one bf16 rounding
of slack (atol 2e-2 / rtol 8e-3 on the normalised values, the reference's
bf16 norm tolerance is 1e-2).  Everything without a norm in between is
compared bit for bit.
"""

import pytest
import torch

from xb200 import XbError, ops

pytestmark = pytest.mark.gpu


def _status_ok():
    assert ops.device_status() == 0


def _data(M, N, K, seed, scale=16):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(M, K, generator=g) / 4).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=g) / scale).to(torch.bfloat16).cuda()
    b = (torch.randn(N, generator=g) / 4).to(torch.bfloat16).cuda()
    r = torch.randn(M, N, generator=g).to(torch.bfloat16).cuda()
    return x, w, b, r


@pytest.mark.parametrize("M,N,K", [(1, 896, 896), (7, 1152, 896), (64, 896, 4864), (64, 9728, 896), (33, 1000, 200),
                                   (64, 3072, 768), (5, 2304, 768)])
def test_decode_linear_matches_fp32_and_small_linear(M, N, K):
    x, w, b, _ = _data(M, N, K, M + N + K)
    y = ops.decode_linear(x, w, b)
    ref = x.float() @ w.float().t() + b.float()
    torch.testing.assert_close(y.float(), ref, atol=2e-3, rtol=2 ** -7)
    assert torch.equal(y, ops.linear(x, w, b))        # same kernel behind the small-M linear
    assert torch.equal(y, ops.decode_linear(x, w, b))  # fixed-order reduction: bit-repeatable
    g = ops.decode_linear(x, w, b, act="gelu_tanh")
    assert torch.equal(g, ops.gelu_tanh(y))            # GELU on the rounded linear, as two kernels
    _status_ok()


@pytest.mark.parametrize("kind", ["rms", "layer"])
@pytest.mark.parametrize("M,N,K", [(64, 896, 896), (7, 768, 3072), (3, 1000, 200), (64, 896, 4864)])
def test_decode_residual_y_and_statistics(kind, M, N, K):
    x, w, b, r = _data(M, N, K, 7 * M + N)
    y, st = ops.decode_linear_residual(x, w, b, r, stats_kind=kind)
    assert torch.equal(y, ops.vecadd(r, ops.linear(x, w, b)))  # bf16(r + bf16(linear)), bit for bit
    nb = (N + 127) // 128
    st = st.view(nb, 64, 2)[:, :M].cpu().double()
    yd = y.cpu().double()
    for blk in range(nb):
        seg = yd[:, blk * 128:min(N, blk * 128 + 128)]
        if kind == "rms":
            torch.testing.assert_close(st[blk, :, 0], (seg * seg).sum(1), rtol=1e-5, atol=1e-4)
        else:
            mean = seg.mean(1)
            torch.testing.assert_close(st[blk, :, 0], mean, rtol=1e-5, atol=1e-5)
            torch.testing.assert_close(st[blk, :, 1], ((seg - mean[:, None]) ** 2).sum(1), rtol=1e-4, atol=1e-3)
    y2, _ = ops.decode_linear_residual(x, w, b, r)  # no statistics: same y
    assert torch.equal(y, y2)
    _status_ok()


def _norm(y, kind, nw, nb, eps):
    return ops.rms_norm(y, nw, eps) if kind == "rms" else ops.layernorm(y, nw, nb, eps)


@pytest.mark.parametrize("kind", ["rms", "layer"])
@pytest.mark.parametrize("M", [1, 13, 64])
def test_pending_norm_equals_norm_kernel_then_linear(kind, M):
    """residual linear -> (norm applied on load) -> next linear, against the
    unfused residual linear -> norm kernel -> linear."""
    D, F = 896, 1152
    x, w, b, r = _data(M, D, 4864 if kind == "rms" else 768, M)
    g = torch.Generator().manual_seed(100 + M)
    nw = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16).cuda()
    nbias = (0.1 * torch.randn(D, generator=g)).to(torch.bfloat16).cuda() if kind == "layer" else None
    w2 = (torch.randn(F, D, generator=g) / 16).to(torch.bfloat16).cuda()
    b2 = (torch.randn(F, generator=g) / 4).to(torch.bfloat16).cuda()
    eps = 1e-6 if kind == "rms" else 1e-5
    y, st = ops.decode_linear_residual(x, w, b, r, stats_kind=kind)
    fused = ops.decode_linear(y, w2, b2, xnorm=(st, nw, nbias, eps, kind))
    yn = _norm(y, kind, nw, nbias, eps)
    unfused = ops.decode_linear(yn, w2, b2)
    ref = yn.float() @ w2.float().t() + b2.float()
    torch.testing.assert_close(fused.float(), ref, atol=1e-2, rtol=2e-2)
    torch.testing.assert_close(fused.float(), unfused.float(), atol=1e-2, rtol=2e-2)
    assert (fused == unfused).float().mean().item() > 0.9
    _status_ok()


@pytest.mark.parametrize("rope", [True, False])
def test_decode_rope_kv_with_pending_norm(rope):
    from oracle.qwen import rope_tables
    B, H, KVH, D, smax, pos, K = 9, 14, 2, 64, 40, 23, 896
    x, w, b, r = _data(B, K, 896, 51)
    g = torch.Generator().manual_seed(52)
    nw = (1 + 0.1 * torch.randn(K, generator=g)).to(torch.bfloat16).cuda()
    wq = (torch.randn((H + 2 * KVH) * D, K, generator=g) / 16).to(torch.bfloat16).cuda()
    bq = (torch.randn((H + 2 * KVH) * D, generator=g) / 4).to(torch.bfloat16).cuda()
    cos, sin = (t.cuda() for t in rope_tables(D, 64, 1e6)) if rope else (None, None)
    y, st = ops.decode_linear_residual(x, w, b, r, stats_kind="rms")
    outs = []
    for fused in (True, False):
        q = torch.empty((B, H, 1, D), dtype=torch.bfloat16, device="cuda")
        kc = torch.zeros((B, KVH, smax, D), dtype=torch.bfloat16, device="cuda")
        vc = torch.zeros_like(kc)
        if fused:
            ops.decode_linear_rope_kv(y, wq, bq, cos, sin, q, kc, vc, H, KVH, D, pos, xnorm=(st, nw, None, 1e-6, "rms"))
        else:
            ops.linear_rope_kv(ops.rms_norm(y, nw, 1e-6), wq, bq, cos, sin, q, kc, vc, H, KVH, D, pos)
        outs.append((q.float().cpu(), kc.float().cpu(), vc.float().cpu()))
    for a, c in zip(*outs):
        torch.testing.assert_close(a, c, atol=1e-2, rtol=2e-2)
    assert torch.count_nonzero(outs[0][1][:, :, pos]) > 0 and torch.count_nonzero(outs[0][1][:, :, pos + 1]) == 0
    _status_ok()


@pytest.mark.parametrize("M", [1, 16, 64])
def test_decode_swiglu_with_and_without_norm(M):
    K, F = 896, 4864
    g = torch.Generator().manual_seed(61 + M)
    x = (torch.randn(M, K, generator=g) / 4).to(torch.bfloat16).cuda()
    wg = (torch.randn(F, K, generator=g) / 16).to(torch.bfloat16).cuda()
    wu = (torch.randn(F, K, generator=g) / 16).to(torch.bfloat16).cuda()
    w = ops.interleave_gate_up(wg, wu)
    h = ops.decode_linear_swiglu(x, w)
    assert torch.equal(h, ops.linear_swiglu(x, w, interleaved=True))  # the same kernel behind it
    ref = ops.silu_mul(ops.linear(x, wg), ops.linear(x, wu))
    torch.testing.assert_close(h.float(), ref.float(), atol=1e-3, rtol=2 ** -7)
    r = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    wo = (torch.randn(K, K, generator=g) / 16).to(torch.bfloat16).cuda()
    nw = (1 + 0.1 * torch.randn(K, generator=g)).to(torch.bfloat16).cuda()
    y, st = ops.decode_linear_residual(x, wo, None, r, stats_kind="rms")
    fused = ops.decode_linear_swiglu(y, w, xnorm=(st, nw, None, 1e-6, "rms"))
    unfused = ops.decode_linear_swiglu(ops.rms_norm(y, nw, 1e-6), w)
    torch.testing.assert_close(fused.float(), unfused.float(), atol=1e-2, rtol=2e-2)
    _status_ok()


def test_decode_linear_rejects_what_it_cannot_take():
    x, w, b, r = _data(65, 896, 896, 1)
    with pytest.raises(ValueError):
        ops.decode_linear(x, w, b)  # more than 64 tokens: host-side check
    x64 = x[:64]
    st = ops.decode_stats(896, x.device)
    nw = torch.ones(896, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(XbError):
        ops.decode_linear(x64[:, :892], w[:, :892], b, xnorm=(st, nw, None, 1e-6, "rms"))  # K % 8 != 0
    _status_ok()


def test_reserved_workspace_is_shared_by_device_spellings():
    """A reservation made for "cuda" is the buffer an operator on cuda:N uses,
    so decode graphs captured after it never see the scratch buffer move."""
    ops.reserve_workspace("cuda", 8 << 20)
    a = ops._workspace(torch.device("cuda", torch.cuda.current_device()), 1 << 20)
    b = ops._workspace("cuda", 2 << 20)
    assert a.data_ptr() == b.data_ptr() and a.numel() * 4 >= 8 << 20


@pytest.mark.parametrize("M,N,K", [(64, 151936, 896), (1, 50257, 768), (7, 1000, 64), (33, 128, 200)])
def test_linear_argmax_equals_argmax_of_logits(M, N, K):
    x, w, _, _ = _data(M, N, K, N + M)
    got = ops.linear_argmax(x, w)
    logits = ops.linear(x, w, out_dtype=torch.float32)
    assert torch.equal(got, torch.argmax(logits, -1))
    assert torch.equal(got, ops.argmax(logits))
    _status_ok()


def test_linear_argmax_ties_take_the_first_row():
    """Equal logits in different 128-row tiles and within one tile: the first
    index wins, as torch.argmax."""
    M, N, K = 5, 3000, 128
    x, w, _, _ = _data(M, N, K, 9)
    big = (torch.ones(K) * 0.5).to(torch.bfloat16).cuda()
    x = x.abs()  # every logit of the `big` rows is the same positive maximum
    for r in (2900, 1700, 1701, 130):
        w[r] = big
    got = ops.linear_argmax(x, w)
    assert torch.equal(got.cpu(), torch.full((M,), 130, dtype=torch.int64))
    assert torch.equal(got, torch.argmax(ops.linear(x, w, out_dtype=torch.float32), -1))
    _status_ok()

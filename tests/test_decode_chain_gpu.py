"""Decode chain (several decode-step linears in one persistent launch)
against the single-launch decode linears and against fp32 references.

The chain splits K into eight rank slices of ceil(K / 512) 64-wide blocks.
Where the single launch picks the same split (o_proj, down_proj and QKV at
the Qwen2.5-0.5B shapes, and every shape of the reduced layer below) the
outputs are compared bit for bit; the Qwen gate/up projection is split
8 ways by the chain and 3 ways by the single launch, so it and everything
after it is compared within one bf16 rounding of the fp32 sums.
"""

import pytest
import torch

from xb200 import XbError, ops

pytestmark = pytest.mark.gpu

BF = torch.bfloat16


def _status_ok(sync=None):
    assert ops.device_status() == 0
    if sync is not None:
        assert int(sync.abs().sum()) == 0, "the chain leaves its counters at zero"


def _t(g, *shape, scale=1.0):
    return (torch.randn(*shape, generator=g) * scale).to(BF).cuda()


def _layer(D, I, H, KVH, HD, seed):
    g = torch.Generator().manual_seed(seed)
    L = {
        "o_w": _t(g, D, H * HD, scale=D ** -0.5),
        "gate_up_w": ops.interleave_gate_up(_t(g, I, D, scale=D ** -0.5), _t(g, I, D, scale=D ** -0.5)),
        "down_w": _t(g, D, I, scale=I ** -0.5),
        "qkv_w": _t(g, (H + 2 * KVH) * HD, D, scale=D ** -0.5),
        "qkv_b": _t(g, (H + 2 * KVH) * HD, scale=0.1),
        "post_ln": (1 + 0.1 * torch.randn(D, generator=g)).to(BF).cuda(),
        "input_ln": (1 + 0.1 * torch.randn(D, generator=g)).to(BF).cuda(),
    }
    return L, g


def _rope(HD, S):
    half = HD // 2
    inv = 1.0 / (1e6 ** (torch.arange(0, half, dtype=torch.float32) / half))
    f = torch.outer(torch.arange(S, dtype=torch.float32), inv)
    e = torch.cat([f, f], -1)
    return e.cos().cuda().contiguous(), e.sin().cuda().contiguous()


def _caches(M, KVH, S, HD, g):
    return _t(g, M, KVH, S, HD), _t(g, M, KVH, S, HD)


def _run_layer(L, attn, x, cos, sin, kc, vc, H, KVH, HD, pos, chain, sync=None):
    """o_proj + residual -> gate/up + SwiGLU (post norm on load) -> down_proj +
    residual -> next QKV + RoPE + KV write (input norm on load), as one chain
    or as four single launches.  Returns every output."""
    M, D = x.shape
    I = L["gate_up_w"].shape[0] // 2
    q = torch.empty((M, H, 1, HD), dtype=BF, device="cuda")
    if chain:
        y = torch.empty((M, D), dtype=BF, device="cuda")
        h = torch.empty((M, I), dtype=BF, device="cuda")
        xo = torch.empty((M, D), dtype=BF, device="cuda")
        st1, st2 = ops.decode_stats(D, "cuda"), ops.decode_stats(D, "cuda")
        ops.decode_chain([
            ops.chain_residual(attn, L["o_w"], None, x, y, st1, "rms"),
            ops.chain_swiglu(y, L["gate_up_w"], h, xnorm=(st1, L["post_ln"], None, 1e-6, "rms")),
            ops.chain_residual(h, L["down_w"], None, y, xo, st2, "rms"),
            ops.chain_rope_kv(xo, L["qkv_w"], L["qkv_b"], cos, sin, q, kc, vc, H, KVH, HD, pos,
                              xnorm=(st2, L["input_ln"], None, 1e-6, "rms")),
        ], sync)
    else:
        y, st1 = ops.decode_linear_residual(attn, L["o_w"], None, x, stats_kind="rms")
        h = ops.decode_linear_swiglu(y, L["gate_up_w"], xnorm=(st1, L["post_ln"], None, 1e-6, "rms"))
        xo, st2 = ops.decode_linear_residual(h, L["down_w"], None, y, stats_kind="rms")
        ops.decode_linear_rope_kv(xo, L["qkv_w"], L["qkv_b"], cos, sin, q, kc, vc, H, KVH, HD, pos,
                                  xnorm=(st2, L["input_ln"], None, 1e-6, "rms"))
    return {"y": y, "st1": st1, "h": h, "x": xo, "st2": st2, "q": q, "k": kc[:, :, pos], "v": vc[:, :, pos]}


@pytest.mark.parametrize("M", [64, 5, 1])
def test_layer_chain_bit_exact_where_the_split_matches(M):
    """Reduced layer (D 896, I 256): the single launches split K exactly as the
    chain does, so every output of the four-phase chain is bit-identical."""
    D, I, H, KVH, HD, S, pos = 896, 256, 14, 2, 64, 40, 33
    L, g = _layer(D, I, H, KVH, HD, 100 + M)
    attn, x = _t(g, M, H * HD), _t(g, M, D)
    cos, sin = _rope(HD, S)
    k1, v1 = _caches(M, KVH, S, HD, g)
    k2, v2 = k1.clone(), v1.clone()
    sync = ops.decode_chain_sync("cuda")
    a = _run_layer(L, attn, x, cos, sin, k1, v1, H, KVH, HD, pos, chain=True, sync=sync)
    b = _run_layer(L, attn, x, cos, sin, k2, v2, H, KVH, HD, pos, chain=False)
    nb = (D + 127) // 128
    for name in ("y", "h", "x", "q", "k", "v"):
        assert torch.equal(a[name], b[name]), name
    for name in ("st1", "st2"):
        assert torch.equal(a[name].view(nb, 64, 2)[:, :M], b[name].view(nb, 64, 2)[:, :M]), name
    assert torch.equal(k1, k2) and torch.equal(v1, v2)  # nothing but row `pos` written
    _status_ok(sync)


def test_qwen_shape_chain_matches_single_launches():
    """Qwen2.5-0.5B layer shapes (gate/up 9728 x 896, down 896 x 4864), batch
    64: o_proj bit-exact, the rest within one bf16 rounding; repeated chains
    are bit-repeatable."""
    D, I, H, KVH, HD, S, pos, M = 896, 4864, 14, 2, 64, 640, 576, 64
    L, g = _layer(D, I, H, KVH, HD, 7)
    attn, x = _t(g, M, H * HD), _t(g, M, D)
    cos, sin = _rope(HD, S)
    k1, v1 = _caches(M, KVH, S, HD, g)
    k2, v2 = k1.clone(), v1.clone()
    sync = ops.decode_chain_sync("cuda")
    a = _run_layer(L, attn, x, cos, sin, k1, v1, H, KVH, HD, pos, chain=True, sync=sync)
    b = _run_layer(L, attn, x, cos, sin, k2, v2, H, KVH, HD, pos, chain=False)
    assert torch.equal(a["y"], b["y"])
    for name in ("h", "x", "q", "k", "v"):
        torch.testing.assert_close(a[name].float(), b[name].float(), atol=3e-2, rtol=2 ** -7, msg=name)
    a2 = _run_layer(L, attn, x, cos, sin, k1, v1, H, KVH, HD, pos, chain=True, sync=sync)
    for name in ("y", "h", "x", "q"):
        assert torch.equal(a[name], a2[name]), name
    _status_ok(sync)


@pytest.mark.parametrize("M,N,K,act", [(64, 1000, 200, None), (7, 3072, 768, "gelu_tanh"), (33, 896, 4864, None),
                                       (64, 131072, 896, None)])
def test_store_phase_matches_decode_linear(M, N, K, act):
    """One-phase chains: y = bf16(x W^T + b) [GELU], against the single launch
    and fp32; N = 131072 gives 1024 units, many per cluster."""
    g = torch.Generator().manual_seed(M + N + K)
    x, w, b = _t(g, M, K, scale=0.25), _t(g, N, K, scale=K ** -0.5), _t(g, N, scale=0.25)
    y = torch.empty((M, N), dtype=BF, device="cuda")
    sync = ops.decode_chain_sync("cuda")
    ops.decode_chain([ops.chain_store(x, w, b, y, act=act)], sync)
    torch.testing.assert_close(y.float(), ops.decode_linear(x, w, b, act=act).float(), atol=2e-2, rtol=2 ** -7)
    if act is None:
        torch.testing.assert_close(y.float(), x.float() @ w.float().t() + b.float(), atol=3e-3, rtol=2 ** -7)
    _status_ok(sync)


def test_phase_reads_what_the_previous_phase_wrote():
    """Two store phases where the second's X is the first's Y (a grid barrier
    between them), against two single launches."""
    g = torch.Generator().manual_seed(5)
    M, K0, N0, N1 = 64, 512, 768, 1024
    x, w0, w1 = _t(g, M, K0), _t(g, N0, K0, scale=K0 ** -0.5), _t(g, N1, N0, scale=N0 ** -0.5)
    y0 = torch.empty((M, N0), dtype=BF, device="cuda")
    y1 = torch.empty((M, N1), dtype=BF, device="cuda")
    sync = ops.decode_chain_sync("cuda")
    for _ in range(3):
        y0.zero_()
        y1.zero_()
        ops.decode_chain([ops.chain_store(x, w0, None, y0), ops.chain_store(y0, w1, None, y1)], sync)
        r0 = ops.decode_linear(x, w0)
        assert torch.equal(y0, r0)
        assert torch.equal(y1, ops.decode_linear(r0, w1))
    _status_ok(sync)


def test_chain_replays_in_a_cuda_graph():
    D, I, H, KVH, HD, S, pos, M = 896, 256, 14, 2, 64, 40, 20, 64
    L, g = _layer(D, I, H, KVH, HD, 3)
    attn, x = _t(g, M, H * HD), _t(g, M, D)
    cos, sin = _rope(HD, S)
    kc, vc = _caches(M, KVH, S, HD, g)
    sync = ops.decode_chain_sync("cuda")
    eager = _run_layer(L, attn, x, cos, sin, kc.clone(), vc.clone(), H, KVH, HD, pos, chain=True, sync=sync)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = _run_layer(L, attn, x, cos, sin, kc, vc, H, KVH, HD, pos, chain=True, sync=sync)
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        for name in ("y", "h", "x", "q"):
            assert torch.equal(out[name], eager[name]), name
    _status_ok(sync)


def test_chain_rejects_what_it_cannot_run():
    g = torch.Generator().manual_seed(0)
    x, w = _t(g, 8, 8192), _t(g, 256, 8192)
    y = torch.empty((8, 256), dtype=BF, device="cuda")
    sync = ops.decode_chain_sync("cuda")
    with pytest.raises(XbError, match="XB_ERR_UNSUPPORTED"):
        ops.decode_chain([ops.chain_store(x, w, None, y)], sync)  # K > 5120
    with pytest.raises(ValueError):
        ops.decode_chain([], sync)
    ph = ops.chain_store(x[:, :512], w[:, :512], None, y)
    with pytest.raises(ValueError):
        ops.decode_chain([ph] * 5, sync)
    _status_ok(sync)

"""Tensor-level operators over the C ABI (device tensors in, device tensors out).

Each function takes CUDA tensors, validates dtype / device / layout on the
host, and enqueues one library call on the current torch CUDA stream.  There
is no PyTorch or CPU fallback: a missing library or an unsupported input
raises.  For the reference's host-tensor launch semantics see
``xb200.kernels``.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

DT = {torch.bfloat16: 0, torch.float32: 1, torch.int8: 2, torch.int16: 3, torch.int32: 4}
FLOAT_DTYPES = (torch.bfloat16, torch.float32)


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _cuda(*ts: torch.Tensor) -> None:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
            raise ValueError("xb200.ops operates on CUDA tensors (use xb200.kernels for host tensors)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")


def _flat(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


def _float_dtype(*ts: torch.Tensor) -> int:
    dt = ts[0].dtype
    if dt not in FLOAT_DTYPES:
        raise TypeError(f"unsupported dtype {dt}: bf16 or fp32 expected")
    for t in ts[1:]:
        if t is not None and t.dtype != dt:
            raise TypeError(f"dtype mismatch: {dt} vs {t.dtype}")
    return DT[dt]


def _out_like(x: torch.Tensor, out: torch.Tensor | None) -> torch.Tensor:
    if out is None:
        return torch.empty_like(x, memory_format=torch.contiguous_format)
    _cuda(out)
    if out.dtype != x.dtype or out.numel() != x.numel():
        raise ValueError("out has the wrong dtype or size")
    return _flat(out, "out")


# --------------------------------------------------------------------------- elementwise


def _binary(fn: str, a: torch.Tensor, b: torch.Tensor, out, *scalar) -> torch.Tensor:
    _cuda(a, b)
    dt = _float_dtype(a, b)
    if a.numel() != b.numel():
        raise ValueError(f"size mismatch: {a.numel()} vs {b.numel()}")
    out = _out_like(a, out)
    _lib.call(fn, _flat(a, "a").data_ptr(), _flat(b, "b").data_ptr(), out.data_ptr(), *scalar[:1], a.numel(), dt,
              _stream())
    return out


def _unary(fn: str, x: torch.Tensor, out, *scalar) -> torch.Tensor:
    _cuda(x)
    dt = _float_dtype(x)
    out = _out_like(x, out)
    if scalar:
        _lib.call(fn, _flat(x, "x").data_ptr(), out.data_ptr(), scalar[0], x.numel(), dt, _stream())
    else:
        _lib.call(fn, _flat(x, "x").data_ptr(), out.data_ptr(), x.numel(), dt, _stream())
    return out


def vecadd(a, b, out=None):
    """c = a + b (examples/vec-add/vec-add.py:16-35)."""
    return _binary("xb_vecadd", a, b, out)


def axpy(x, y, alpha: float, out=None):
    """out = alpha * x + y (examples/axpy/axpy.py:13-29)."""
    _cuda(x, y)
    dt = _float_dtype(x, y)
    if x.numel() != y.numel():
        raise ValueError("size mismatch")
    out = _out_like(x, out)
    _lib.call("xb_axpy", _flat(x, "x").data_ptr(), _flat(y, "y").data_ptr(), out.data_ptr(), float(alpha),
              x.numel(), dt, _stream())
    return out


def relu(x, out=None):
    """max(x, 0) (examples/relu/relu.py:13-26)."""
    return _unary("xb_relu", x, out)


def leaky_relu(x, negative_slope: float = 0.01, out=None):
    """x >= 0 ? x : slope * x (examples/leaky_relu/leaky_relu.py:15-31)."""
    return _unary("xb_leaky_relu", x, out, float(negative_slope))


def gelu(x, out=None):
    """x * sigmoid(1.702 x) (examples/gelu/gelu.py:13-30)."""
    return _unary("xb_gelu", x, out)


def gelu_tanh(x, out=None):
    """tanh-form GELU (examples/gpt2/kernels/gelu.py:25-45)."""
    return _unary("xb_gelu_tanh", x, out)


def sigmoid(x, out=None):
    """1 / (1 + exp(-x)) (examples/sigmoid/sigmoid.py:13-34)."""
    return _unary("xb_sigmoid", x, out)


def silu(x, out=None):
    """x * sigmoid(x) (examples/silu/silu.py:13-30)."""
    return _unary("xb_silu", x, out)


def swiglu(gate, up, out=None):
    """silu(gate) * up (examples/swiglu/swiglu.py:13-33)."""
    return _binary("xb_swiglu", gate, up, out)


def mul(a, b, out=None):
    """c = a * b elementwise."""
    return _binary("xb_mul", a, b, out)


def mul_2d(x, y, out):
    """out[r, c] = x[r, c] * y[r, c] over 2-D views with unit column stride
    (the block-pointer product of examples/load_2d_block)."""
    _cuda(x, y, out)
    dt = _float_dtype(x, y)
    if out.dtype != x.dtype or x.shape != y.shape or out.shape != x.shape or x.dim() != 2:
        raise ValueError("mul_2d takes three 2-D tensors of one shape and dtype")
    rows, cols = x.shape
    _lib.call("xb_mul_2d", x.data_ptr(), y.data_ptr(), out.data_ptr(), rows, cols, _mat(x, "x"), _mat(y, "y"),
              _mat(out, "out"), dt, _stream())
    return out


def silu_mul(gate, up, out=None):
    """silu(gate) * up in fp32, one rounding (examples/qwen2_5/kernels/swiglu.py:29-50)."""
    return _binary("xb_silu_mul", gate, up, out)


# --------------------------------------------------------------------------- row reductions


def _rows(x: torch.Tensor, name: str) -> tuple[int, int, int]:
    if x.dim() < 1:
        raise ValueError(f"{name} needs at least one dimension")
    cols = x.shape[-1]
    if x.stride(-1) != 1 and cols > 1:
        raise ValueError(f"{name}: last dimension must have unit stride")
    if x.dim() == 1:
        return 1, cols, cols
    x2 = x.reshape(-1, cols) if x.dim() > 2 else x
    if x.dim() > 2 and not x.is_contiguous():
        raise ValueError(f"{name}: >2-D input must be contiguous")
    return x2.shape[0], cols, x2.stride(0)


def _row_out(x, out):
    if out is None:
        return torch.empty(x.shape, dtype=x.dtype, device=x.device)
    _cuda(out)
    if out.shape != x.shape or out.dtype != x.dtype:
        raise ValueError("out has the wrong shape or dtype")
    return out


def softmax(x, out=None):
    """Row softmax over the last dim (examples/test_softmax/test_softmax.py:13-45)."""
    _cuda(x)
    dt = _float_dtype(x)
    out = _row_out(x, out)
    rows, cols, xs = _rows(x, "x")
    _, _, ys = _rows(out, "out")
    _lib.call("xb_softmax", x.data_ptr(), out.data_ptr(), rows, cols, xs, ys, dt, _stream())
    return out


def layernorm(x, weight=None, bias=None, eps: float = 1e-5, out=None):
    """(x - mean) * rsqrt(var + eps) * weight + bias over the last dim
    (examples/test_layernorm/test_layernorm.py:13-60)."""
    _cuda(x, weight, bias)
    dt = _float_dtype(x, weight, bias)
    out = _row_out(x, out)
    rows, cols, xs = _rows(x, "x")
    _, _, ys = _rows(out, "out")
    for p, n in ((weight, "weight"), (bias, "bias")):
        if p is not None and (p.numel() != cols or not p.is_contiguous()):
            raise ValueError(f"{n} must be a contiguous vector of {cols} elements")
    _lib.call("xb_layernorm", x.data_ptr(), weight.data_ptr() if weight is not None else None,
              bias.data_ptr() if bias is not None else None, out.data_ptr(), rows, cols, xs, ys, float(eps), dt,
              _stream())
    return out


def rms_norm(x, weight=None, eps: float = 1e-5, out=None):
    """x * rsqrt(mean(x^2) + eps) [* weight] (examples/rms_norm/rms_norm.py:23-55,
    examples/weighted_rms_norm/weighted_rms_norm.py:21-58)."""
    _cuda(x, weight)
    dt = _float_dtype(x, weight)
    out = _row_out(x, out)
    rows, cols, xs = _rows(x, "x")
    _, _, ys = _rows(out, "out")
    if weight is not None and (weight.numel() != cols or not weight.is_contiguous()):
        raise ValueError(f"weight must be a contiguous vector of {cols} elements")
    _lib.call("xb_rms_norm", x.data_ptr(), weight.data_ptr() if weight is not None else None, out.data_ptr(), rows,
              cols, xs, ys, float(eps), dt, _stream())
    return out


def weighted_rms_norm(x, weight, eps: float = 1e-5, out=None):
    return rms_norm(x, weight, eps, out)


def row_center(x, out=None):
    """x - mean(x) over the last dim (examples/average_pool/average_pool.py:24-52)."""
    _cuda(x)
    dt = _float_dtype(x)
    out = _row_out(x, out)
    rows, cols, xs = _rows(x, "x")
    _, _, ys = _rows(out, "out")
    _lib.call("xb_row_center", x.data_ptr(), out.data_ptr(), rows, cols, xs, ys, dt, _stream())
    return out


def avg_pool2d_2x2(x, out=None):
    """2x2 / stride-2 average pooling of a contiguous [..., H, W] tensor."""
    _cuda(x)
    dt = _float_dtype(x)
    if x.dim() < 2 or not x.is_contiguous():
        raise ValueError("x must be a contiguous tensor with at least 2 dims")
    h, w = x.shape[-2], x.shape[-1]
    planes = x.numel() // (h * w) if h * w else 0
    oshape = tuple(x.shape[:-2]) + (h // 2, w // 2)
    if out is None:
        out = torch.empty(oshape, dtype=x.dtype, device=x.device)
    else:
        _cuda(out)
        if tuple(out.shape) != oshape or out.dtype != x.dtype or not out.is_contiguous():
            raise ValueError("out has the wrong shape, dtype or layout")
    _lib.call("xb_avg_pool2d_2x2", x.data_ptr(), out.data_ptr(), planes, h, w, dt, _stream())
    return out


def device_name(device: int = 0) -> tuple[str, int]:
    buf = ctypes.create_string_buffer(256)
    sms = ctypes.c_int(0)
    _lib.call("xb_device_name", device, buf, 256, ctypes.byref(sms))
    return buf.value.decode(), sms.value


# --------------------------------------------------------------------------- GEMMs


def _mat(t: torch.Tensor, name: str) -> int:
    if t.dim() != 2:
        raise ValueError(f"{name} must be 2-D")
    if t.stride(1) != 1 and t.shape[1] > 1:
        raise ValueError(f"{name} must be row-major (unit column stride)")
    return t.stride(0) if t.shape[0] > 1 else max(t.shape[1], 1)


def _gemm_out(a, b_cols, dtype, out):
    M = a.shape[0]
    if out is None:
        return torch.empty((M, b_cols), dtype=dtype, device=a.device)
    _cuda(out)
    if tuple(out.shape) != (M, b_cols) or out.dtype != dtype:
        raise ValueError(f"out must be {(M, b_cols)} {dtype}")
    return out


def matmul_i8(a, b, out=None):
    """int32 C = A (int8 [M,K]) @ B (int8 [K,N]), exact
    (examples/matmul_i8_m128_n64_k64/matmul_i8_m128_n64_k64.py:22-52)."""
    _cuda(a, b, out)
    if a.dtype != torch.int8 or b.dtype != torch.int8:
        raise TypeError("matmul_i8 takes int8 operands")
    if a.shape[1] != b.shape[0]:
        raise ValueError(f"shape mismatch {tuple(a.shape)} @ {tuple(b.shape)}")
    out = _gemm_out(a, b.shape[1], torch.int32, out)
    M, K = a.shape
    N = b.shape[1]
    _lib.call("xb_matmul_i8", a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, _mat(a, "A"), _mat(b, "B"),
              _mat(out, "C"), _stream())
    return out


def linear_i8(x, w, out=None):
    """int32 y = x (int8 [M,K]) @ w^T (int8 [N,K]), exact."""
    _cuda(x, w, out)
    if x.dtype != torch.int8 or w.dtype != torch.int8:
        raise TypeError("linear_i8 takes int8 operands")
    if x.shape[1] != w.shape[1]:
        raise ValueError("shape mismatch")
    out = _gemm_out(x, w.shape[0], torch.int32, out)
    M, K = x.shape
    N = w.shape[0]
    _lib.call("xb_linear_i8", x.data_ptr(), w.data_ptr(), out.data_ptr(), M, N, K, _mat(x, "x"), _mat(w, "w"),
              _mat(out, "y"), _stream())
    return out


def matmul_f32_bf16emu(a, b, a_transposed=False, out=None):
    """C (f32 [M, N]) = bf16(A) @ bf16(B) with f32 accumulation: f32 operands
    rounded to bf16 as the reference's bf16 emulation does
    (examples/matmul_f32_m64_n32_k16_padded_atransposed).  With
    a_transposed, `a` is the [K, M] storage of A."""
    _cuda(a, b, out)
    if a.dtype != torch.float32 or b.dtype != torch.float32:
        raise TypeError("matmul_f32_bf16emu takes f32 operands")
    K, M = (a.shape[0], a.shape[1]) if a_transposed else (a.shape[1], a.shape[0])
    if b.shape[0] != K:
        raise ValueError(f"shape mismatch: K={K} vs B {tuple(b.shape)}")
    N = b.shape[1]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=a.device)
    elif out.dtype != torch.float32 or tuple(out.shape) != (M, N):
        raise ValueError("out must be f32 [M, N]")
    need = ctypes.c_size_t(0)
    _lib.call("xb_matmul_f32_bf16emu_workspace_size", M, N, K, ctypes.byref(need))
    ws = _workspace(a.device, need.value)
    _lib.call("xb_matmul_f32_bf16emu", a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, _mat(a, "a"),
              _mat(b, "b"), _mat(out, "out"), int(a_transposed), ws.data_ptr(), ws.numel() * 4, _stream())
    return out


def matmul_i16(a, b, out=None, workspace=None):
    """int32 C = A (int16) @ B (int16) with int32 wrap-around."""
    _cuda(a, b, out)
    if a.dtype != torch.int16 or b.dtype != torch.int16:
        raise TypeError("matmul_i16 takes int16 operands")
    if a.shape[1] != b.shape[0]:
        raise ValueError(f"shape mismatch {tuple(a.shape)} @ {tuple(b.shape)}")
    out = _gemm_out(a, b.shape[1], torch.int32, out)
    M, K = a.shape
    N = b.shape[1]
    need = ctypes.c_size_t(0)
    _lib.call("xb_matmul_i16_workspace_size", M, N, K, ctypes.byref(need))
    if workspace is None or workspace.numel() * workspace.element_size() < need.value:
        # torch's caching allocator returns 512-byte aligned blocks
        workspace = torch.empty(need.value, dtype=torch.uint8, device=a.device)
    _lib.call("xb_matmul_i16", a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, _mat(a, "A"), _mat(b, "B"),
              _mat(out, "C"), workspace.data_ptr(), workspace.numel() * workspace.element_size(), _stream())
    return out


def matmul_bf16(a, b, out_dtype=torch.float32, out=None):
    """C = A (bf16 [M,K]) @ B (bf16 [K,N]), fp32 accumulation, C in f32 or bf16
    (examples/matmul_bf16_m64_n64_k64/matmul_bf16_m64_n64_k64.py:16-46)."""
    _cuda(a, b, out)
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise TypeError("matmul_bf16 takes bf16 operands")
    if a.shape[1] != b.shape[0]:
        raise ValueError(f"shape mismatch {tuple(a.shape)} @ {tuple(b.shape)}")
    if out is not None:
        out_dtype = out.dtype
    if out_dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("out dtype must be float32 or bfloat16")
    out = _gemm_out(a, b.shape[1], out_dtype, out)
    M, K = a.shape
    N = b.shape[1]
    _lib.call("xb_matmul_bf16", a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, _mat(a, "A"), _mat(b, "B"),
              _mat(out, "C"), DT[out_dtype], _stream())
    return out


SMALL_M = 64  # token counts at or below this take the swap-AB split-K path
_workspaces: dict = {}
_slot = [0]  # workspace slot of the operators being issued (see workspace_slot)


class workspace_slot:
    """Operators issued inside ``with workspace_slot(i):`` use scratch slot i:
    work issued on different streams at the same time (e.g. two decode
    groups replaying their CUDA graphs concurrently) must use different
    slots, because each slot's buffers are reused by every operator issued
    under it."""

    def __init__(self, slot: int):
        self.slot = int(slot)

    def __enter__(self):
        self.prev = _slot[0]
        _slot[0] = self.slot
        return self

    def __exit__(self, *exc):
        _slot[0] = self.prev
        return False


def reserve_workspace(device, nbytes: int) -> None:
    """Grow the shared scratch buffer to at least `nbytes` now.  A captured
    CUDA graph records the buffer's address, so everything a set of graphs
    will need must be reserved before the first capture (a later growth would
    leave earlier graphs pointing at freed memory)."""
    _workspace(torch.device(device), nbytes)


def attention_workspace_bytes(batch, seq, n_head, n_kv_head, pos_offset) -> int:
    need = ctypes.c_size_t(0)
    _lib.call("xb_attention_workspace_size", batch, seq, n_head, n_kv_head, pos_offset, ctypes.byref(need))
    return need.value


def _workspace(device, nbytes: int) -> torch.Tensor:
    """A per-(device, workspace slot) fp32 scratch buffer that only grows
    (kept alive so its address is stable, e.g. across CUDA-graph replays).
    Operators issued under one slot must not run concurrently on two streams."""
    device = torch.device(device)
    if device.index is None:  # "cuda" and "cuda:<current>" name the same buffer
        device = torch.device(device.type, torch.cuda.current_device())
    key = (device, _slot[0])
    ws = _workspaces.get(key)
    if ws is None or ws.numel() * 4 < nbytes:
        ws = torch.empty(max(nbytes // 4, 1 << 20), dtype=torch.float32, device=device)
        _workspaces[key] = ws
    return ws


def linear(x, weight, bias=None, out=None, out_dtype=torch.bfloat16, residual=None, act=None):
    """y = [residual +] x @ weight^T + bias, weight [N, K] (nn.Linear layout),
    bf16 inputs, fp32 accumulation, y in bf16 or fp32
    (examples/qwen2_5/kernels/matmul.py:172-296).  Up to SMALL_M rows use the
    small-M kernel with the residual add fused; larger inputs the tiled GEMM
    with the residual add in its epilogue.  act="gelu_tanh" applies the tanh
    GELU to the bf16 output inside the same launch (GPT-2 c_fc)."""
    _cuda(x, weight, bias, out, residual)
    if act is not None:
        if act != "gelu_tanh" or residual is not None or out_dtype != torch.bfloat16:
            raise ValueError("act='gelu_tanh' takes bf16 output and no residual")
        K = x.shape[-1]
        N = weight.shape[0]
        x2 = x.reshape(-1, K)
        M = x2.shape[0]
        y = out.reshape(M, N) if out is not None else torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
        ws = _small_ws(x, M, N, K) if M <= SMALL_M else None
        _lib.call("xb_linear_gelu_bf16", x2.data_ptr(), weight.data_ptr(),
                  bias.data_ptr() if bias is not None else None, y.data_ptr(), M, N, K, _mat(x2, "x"),
                  _mat(weight, "weight"), _mat(y, "y"), ws.data_ptr() if ws is not None else None,
                  ws.numel() * 4 if ws is not None else 0, _stream())
        return y.reshape(*x.shape[:-1], N) if out is None else out
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise TypeError("linear takes bf16 x and weight")
    if bias is not None and (bias.dtype != torch.bfloat16 or bias.numel() != weight.shape[0]
                             or not bias.is_contiguous()):
        raise ValueError("bias must be a contiguous bf16 vector of N elements")
    K = x.shape[-1]
    N = weight.shape[0]
    if weight.shape[1] != K:
        raise ValueError(f"shape mismatch x[..., {K}] vs weight {tuple(weight.shape)}")
    x2 = x.reshape(-1, K)
    M = x2.shape[0]
    if out is not None:
        out_dtype = out.dtype
    if out_dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("out dtype must be float32 or bfloat16")
    if out is None:
        y = torch.empty((M, N), dtype=out_dtype, device=x.device)
    else:
        if out.numel() != M * N:
            raise ValueError("out has the wrong size")
        y = out.reshape(M, N)
    bptr = bias.data_ptr() if bias is not None else None
    if residual is not None:
        if residual.dtype != torch.bfloat16 or residual.numel() != M * N:
            raise ValueError("residual must be bf16 with M x N elements")
        r2 = residual.reshape(M, N)
    if residual is not None and M > SMALL_M and out_dtype == torch.bfloat16:
        # the residual add happens in the GEMM epilogue
        _lib.call("xb_linear_residual_bf16", x2.data_ptr(), weight.data_ptr(), bptr, r2.data_ptr(), y.data_ptr(), M,
                  N, K, _mat(x2, "x"), _mat(weight, "weight"), _mat(r2, "residual"), _mat(y, "y"), _stream())
        return y.reshape(*x.shape[:-1], N) if out is None else out
    if 0 < M <= SMALL_M:
        splits = ctypes.c_int(0)
        need = ctypes.c_size_t(0)
        _lib.call("xb_linear_small_plan", M, N, K, int(residual is not None), ctypes.byref(splits), ctypes.byref(need))
        ws = _workspace(x.device, need.value) if need.value else None
        _lib.call("xb_linear_small_bf16", x2.data_ptr(), weight.data_ptr(), bptr,
                  r2.data_ptr() if residual is not None else None, y.data_ptr(), M, N, K, _mat(x2, "x"),
                  _mat(weight, "weight"), _mat(r2, "residual") if residual is not None else N, _mat(y, "y"),
                  DT[out_dtype], splits.value, ws.data_ptr() if ws is not None else None,
                  ws.numel() * 4 if ws is not None else 0, _stream())
    else:
        _lib.call("xb_linear_bf16", x2.data_ptr(), weight.data_ptr(), bptr, y.data_ptr(), M, N, K, _mat(x2, "x"),
                  _mat(weight, "weight"), _mat(y, "y"), DT[out_dtype], _stream())
        if residual is not None:
            if out_dtype != torch.bfloat16:
                raise TypeError("a fused residual needs bf16 output")
            vecadd(r2, y, out=y)
    return y.reshape(*x.shape[:-1], N) if out is None else out


def interleave_gate_up(w_gate, w_up, block: int = 64) -> torch.Tensor:
    """[2 n_out, K] weight interleaving 64-row blocks of gate and up rows, the
    layout of the fused SwiGLU linear (xb_linear_swiglu_bf16)."""
    n_out, K = w_gate.shape
    if w_up.shape != w_gate.shape or n_out % block:
        raise ValueError(f"gate and up weights must share a shape with n_out a multiple of {block}")
    g = w_gate.reshape(n_out // block, block, K)
    u = w_up.reshape(n_out // block, block, K)
    return torch.stack([g, u], 1).reshape(2 * n_out, K).contiguous()


def linear_swiglu(x, w_gate_up, interleaved: bool = False):
    """silu(x @ Wg^T) * (x @ Wu^T) with the roundings of two linears then
    silu_mul.  interleaved=False: W = [Wg; Wu] stacked (few tokens only);
    interleaved=True: W from interleave_gate_up (any number of tokens: one GEMM
    whose epilogue applies the SwiGLU)."""
    _cuda(x, w_gate_up)
    K = x.shape[-1]
    x2 = x.reshape(-1, K)
    M = x2.shape[0]
    N = w_gate_up.shape[0]
    if N % 2 or w_gate_up.shape[1] != K:
        raise ValueError("w_gate_up must be [2*n_out, K]")
    if interleaved:
        y = torch.empty((M, N // 2), dtype=torch.bfloat16, device=x.device)
        ws = None
        if M <= SMALL_M:
            splits = ctypes.c_int(0)
            need = ctypes.c_size_t(0)
            _lib.call("xb_linear_small_plan", M, N, K, 1, ctypes.byref(splits), ctypes.byref(need))
            ws = _workspace(x.device, need.value)
        _lib.call("xb_linear_swiglu_bf16", x2.data_ptr(), w_gate_up.data_ptr(), y.data_ptr(), M, N // 2, K,
                  _mat(x2, "x"), _mat(w_gate_up, "w"), N // 2, ws.data_ptr() if ws is not None else None,
                  ws.numel() * 4 if ws is not None else 0, _stream())
        return y.reshape(*x.shape[:-1], N // 2)
    if M > SMALL_M:
        raise ValueError("stacked gate/up weights take at most SMALL_M tokens; use interleave_gate_up")
    splits = ctypes.c_int(0)
    need = ctypes.c_size_t(0)
    _lib.call("xb_linear_small_plan", M, N, K, 1, ctypes.byref(splits), ctypes.byref(need))
    ws = _workspace(x.device, need.value)
    y = torch.empty((M, N // 2), dtype=torch.bfloat16, device=x.device)
    _lib.call("xb_linear_small_swiglu_bf16", x2.data_ptr(), w_gate_up.data_ptr(), y.data_ptr(), M, N // 2, K,
              _mat(x2, "x"), _mat(w_gate_up, "w"), N // 2, ws.data_ptr(), ws.numel() * 4, _stream())
    return y.reshape(*x.shape[:-1], N // 2)


def _small_ws(x, M, N, K):
    splits = ctypes.c_int(0)
    need = ctypes.c_size_t(0)
    _lib.call("xb_linear_small_plan", M, N, K, 1, ctypes.byref(splits), ctypes.byref(need))
    return _workspace(x.device, need.value)


def linear_rope_kv(x, w_qkv, b_qkv, cos_t, sin_t, q_out, k_cache, v_cache, n_head, n_kv_head, head_dim, pos_offset):
    """Decode step (x [B, K], one token per sequence): qkv = x @ w_qkv^T + b,
    rounded to bf16, RoPE (cos_t = sin_t = None: none) and the KV-cache
    write at pos_offset, in one GEMM + one finishing kernel."""
    _cuda(x, w_qkv, b_qkv, cos_t, sin_t, q_out, k_cache, v_cache)
    B, K = x.shape
    N = w_qkv.shape[0]
    if N != (n_head + 2 * n_kv_head) * head_dim or w_qkv.shape[1] != K:
        raise ValueError("w_qkv must be [(H + 2 KVH) * D, K]")
    if cos_t is not None and cos_t.shape[0] <= pos_offset:
        raise ValueError("RoPE tables are shorter than the position")
    ws = _small_ws(x, B, N, K)
    _lib.call("xb_linear_small_rope_kv_bf16", x.data_ptr(), w_qkv.data_ptr(),
              b_qkv.data_ptr() if b_qkv is not None else None,
              cos_t.data_ptr() if cos_t is not None else None, sin_t.data_ptr() if sin_t is not None else None,
              q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), B, n_head, n_kv_head, head_dim,
              k_cache.shape[2], pos_offset, K, _mat(x, "x"), _mat(w_qkv, "w"), ws.data_ptr(), ws.numel() * 4,
              _stream())


def linear_residual_norm(x, weight, bias, residual, norm_w, norm_b=None, eps=1e-6, kind="rms"):
    """Decode step: y = residual + bf16(x @ weight^T + bias) and
    yn = rmsnorm(y) * norm_w (kind "rms") or layernorm(y) * norm_w + norm_b
    (kind "layer"), in one GEMM + one finishing kernel.  Returns (y, yn)."""
    _cuda(x, weight, bias, residual, norm_w, norm_b)
    K = x.shape[-1]
    x2 = x.reshape(-1, K)
    M = x2.shape[0]
    N = weight.shape[0]
    r2 = residual.reshape(M, N)
    y = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    yn = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    ws = _small_ws(x, M, N, K)
    _lib.call("xb_linear_small_residual_norm_bf16", x2.data_ptr(), weight.data_ptr(),
              bias.data_ptr() if bias is not None else None, r2.data_ptr(), y.data_ptr(), yn.data_ptr(),
              norm_w.data_ptr(), norm_b.data_ptr() if norm_b is not None else None, float(eps),
              0 if kind == "rms" else 1, M, N, K, _mat(x2, "x"), _mat(weight, "weight"), _mat(r2, "residual"), N, N,
              ws.data_ptr(), ws.numel() * 4, _stream())
    return y, yn


# --------------------------------------------------------------------------- decode-step linears
#
# One launch each (the cluster split-K kernel, M <= SMALL_M tokens).  `xnorm`
# = (stats, norm_w, norm_b, eps, kind) marks x as carrying a pending norm:
# the statistics come from the decode_linear_residual call that produced x
# with the same kind, and the kernel normalises x as it loads it.

_NORM_KIND = {"rms": 0, "layer": 1}


def decode_stats(n_features: int, device) -> torch.Tensor:
    """Buffer for the per-block row statistics of decode_linear_residual:
    ceil(N / 128) blocks x 64 tokens x 2 floats."""
    return torch.empty(((n_features + 127) // 128) * 128, dtype=torch.float32, device=device)


def _xin(x, xnorm):
    if x.dtype != torch.bfloat16:
        raise TypeError("decode linears take bf16 x")
    M = x.shape[0]
    if not 0 < M <= SMALL_M:
        raise ValueError(f"decode linears take 1..{SMALL_M} tokens, got {M}")
    if xnorm is None:
        return (x.data_ptr(), M, _mat(x, "x"), None, None, None, 0.0, 0)
    stats, w, b, eps, kind = xnorm
    _cuda(stats, w, b)
    if stats.dtype != torch.float32 or stats.numel() < ((x.shape[1] + 127) // 128) * 128:
        raise ValueError("xnorm statistics must be a float32 decode_stats buffer for x's width")
    return (x.data_ptr(), M, _mat(x, "x"), stats.data_ptr(), w.data_ptr(), b.data_ptr() if b is not None else None,
            float(eps), _NORM_KIND[kind])


def decode_linear(x, weight, bias=None, act=None, xnorm=None, out=None):
    """y = bf16(norm?(x) @ weight^T + bias) [GELU] for a decode step, one launch
    (examples/qwen2_5/kernels/matmul.py:172-296; GPT-2 c_fc + gelu)."""
    _cuda(x, weight, bias, out)
    N, K = weight.shape
    if x.shape[-1] != K:
        raise ValueError("shape mismatch")
    if act not in (None, "gelu_tanh"):
        raise ValueError("act must be None or 'gelu_tanh'")
    y = out if out is not None else torch.empty((x.shape[0], N), dtype=torch.bfloat16, device=x.device)
    _lib.call("xb_decode_linear_bf16", *_xin(x, xnorm), weight.data_ptr(),
              bias.data_ptr() if bias is not None else None, y.data_ptr(), N, K, _mat(weight, "weight"),
              _mat(y, "y"), 1 if act else 0, _stream())
    return y


def decode_linear_rope_kv(x, w_qkv, b_qkv, cos_t, sin_t, q_out, k_cache, v_cache, n_head, n_kv_head, head_dim,
                          pos_offset, xnorm=None):
    """Decode QKV projection + RoPE (none when the tables are None) + KV-cache
    write at pos_offset, one launch (examples/qwen2_5/model.py:836-867)."""
    _cuda(x, w_qkv, b_qkv, cos_t, sin_t, q_out, k_cache, v_cache)
    if cos_t is not None and cos_t.shape[0] <= pos_offset:
        raise ValueError("RoPE tables are shorter than the position")
    K = w_qkv.shape[1]
    _lib.call("xb_decode_linear_rope_kv_bf16", *_xin(x, xnorm), w_qkv.data_ptr(),
              b_qkv.data_ptr() if b_qkv is not None else None,
              cos_t.data_ptr() if cos_t is not None else None, sin_t.data_ptr() if sin_t is not None else None,
              q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), n_head, n_kv_head, head_dim,
              k_cache.shape[2], pos_offset, K, _mat(w_qkv, "w"), _stream())


def decode_linear_swiglu(x, w_gate_up, xnorm=None):
    """silu(norm?(x) Wg^T) * (norm?(x) Wu^T) with W from interleave_gate_up, one launch."""
    _cuda(x, w_gate_up)
    N, K = w_gate_up.shape
    y = torch.empty((x.shape[0], N // 2), dtype=torch.bfloat16, device=x.device)
    _lib.call("xb_decode_linear_swiglu_bf16", *_xin(x, xnorm), w_gate_up.data_ptr(), y.data_ptr(), N // 2, K,
              _mat(w_gate_up, "w"), N // 2, _stream())
    return y


def decode_linear_residual(x, weight, bias, residual, stats_kind=None, xnorm=None):
    """y = residual + bf16(norm?(x) @ weight^T + bias), one launch; with
    stats_kind ("rms" / "layer") also the row statistics of y that the next
    decode linear's xnorm takes.  Returns (y, stats or None)."""
    _cuda(x, weight, bias, residual)
    N, K = weight.shape
    M = x.shape[0]
    r2 = residual.reshape(M, N)
    y = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    st = decode_stats(N, x.device) if stats_kind is not None else None
    _lib.call("xb_decode_linear_residual_bf16", *_xin(x, xnorm), weight.data_ptr(),
              bias.data_ptr() if bias is not None else None, r2.data_ptr(), y.data_ptr(),
              st.data_ptr() if st is not None else None, _NORM_KIND[stats_kind] if stats_kind else 0, N, K,
              _mat(weight, "weight"), _mat(r2, "residual"), N, _stream())
    return y, st


# --------------------------------------------------------------------------- decode chain
#
# Up to four decode linears in one persistent launch (xb_decode_chain_bf16):
# each phase is built like the single-launch call of the same kind, and a
# phase may read what an earlier one wrote.  The structures hold raw device
# addresses: the caller keeps the tensors alive until the launch has run.

CHAIN_MAX_PHASES = 4
CHAIN_MAX_K = 5120  # ten 64-wide K blocks per CTA of an 8-CTA cluster


class DecodePhase(ctypes.Structure):
    """Mirror of the C ``xb_decode_phase`` (include/xb200.h)."""

    _fields_ = [
        ("kind", ctypes.c_int32), ("act", ctypes.c_int32),
        ("x", ctypes.c_void_p), ("m", ctypes.c_int64), ("ldx", ctypes.c_int64),
        ("x_stats", ctypes.c_void_p), ("x_norm_w", ctypes.c_void_p), ("x_norm_b", ctypes.c_void_p),
        ("x_eps", ctypes.c_float), ("x_norm_kind", ctypes.c_int32),
        ("w", ctypes.c_void_p), ("n", ctypes.c_int64), ("k", ctypes.c_int64), ("ldw", ctypes.c_int64),
        ("bias", ctypes.c_void_p), ("y", ctypes.c_void_p), ("ldy", ctypes.c_int64),
        ("residual", ctypes.c_void_p), ("ldr", ctypes.c_int64),
        ("stats_out", ctypes.c_void_p), ("stats_kind", ctypes.c_int32), ("reserved", ctypes.c_int32),
        ("cos_t", ctypes.c_void_p), ("sin_t", ctypes.c_void_p),
        ("q_out", ctypes.c_void_p), ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p),
        ("n_head", ctypes.c_int64), ("n_kv_head", ctypes.c_int64), ("head_dim", ctypes.c_int64),
        ("max_seq", ctypes.c_int64), ("pos_offset", ctypes.c_int64),
    ]


XB_DECODE_STORE, XB_DECODE_ROPE_KV, XB_DECODE_SWIGLU, XB_DECODE_RESIDUAL = 0, 1, 2, 3


def _phase(kind, x, weight, xnorm) -> DecodePhase:
    _cuda(x, weight)
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise TypeError("decode chain phases take bf16 x and weight")
    M = x.shape[0]
    if not 0 < M <= SMALL_M:
        raise ValueError(f"decode chain phases take 1..{SMALL_M} tokens, got {M}")
    N, K = weight.shape
    if x.shape[1] != K:
        raise ValueError("shape mismatch")
    ph = DecodePhase()
    ph.kind = kind
    ph.x, ph.m, ph.ldx = x.data_ptr(), M, _mat(x, "x")
    ph.w, ph.n, ph.k, ph.ldw = weight.data_ptr(), N, K, _mat(weight, "weight")
    if xnorm is not None:
        stats, w, b, eps, nk = xnorm
        _cuda(stats, w, b)
        if stats.dtype != torch.float32 or stats.numel() < ((K + 127) // 128) * 128:
            raise ValueError("xnorm statistics must be a float32 decode_stats buffer for x's width")
        ph.x_stats, ph.x_norm_w = stats.data_ptr(), w.data_ptr()
        ph.x_norm_b = b.data_ptr() if b is not None else None
        ph.x_eps, ph.x_norm_kind = float(eps), _NORM_KIND[nk]
    return ph


def chain_store(x, weight, bias, y, act=None, xnorm=None) -> DecodePhase:
    """Phase: y = bf16(norm?(x) @ weight^T + bias) [tanh GELU] (decode_linear)."""
    ph = _phase(XB_DECODE_STORE, x, weight, xnorm)
    _cuda(bias, y)
    if act not in (None, "gelu_tanh"):
        raise ValueError("act must be None or 'gelu_tanh'")
    ph.act = 1 if act else 0
    ph.bias = bias.data_ptr() if bias is not None else None
    ph.y, ph.ldy = y.data_ptr(), _mat(y, "y")
    return ph


def chain_rope_kv(x, w_qkv, b_qkv, cos_t, sin_t, q_out, k_cache, v_cache, n_head, n_kv_head, head_dim,
                  pos_offset, xnorm=None) -> DecodePhase:
    """Phase: QKV projection + RoPE + KV-cache write at pos_offset (decode_linear_rope_kv)."""
    ph = _phase(XB_DECODE_ROPE_KV, x, w_qkv, xnorm)
    _cuda(b_qkv, cos_t, sin_t, q_out, k_cache, v_cache)
    if cos_t is not None and cos_t.shape[0] <= pos_offset:
        raise ValueError("RoPE tables are shorter than the position")
    ph.bias = b_qkv.data_ptr() if b_qkv is not None else None
    ph.cos_t = cos_t.data_ptr() if cos_t is not None else None
    ph.sin_t = sin_t.data_ptr() if sin_t is not None else None
    ph.q_out, ph.k_cache, ph.v_cache = q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr()
    ph.n_head, ph.n_kv_head, ph.head_dim = n_head, n_kv_head, head_dim
    ph.max_seq, ph.pos_offset = k_cache.shape[2], pos_offset
    return ph


def chain_swiglu(x, w_gate_up, y, xnorm=None) -> DecodePhase:
    """Phase: y = silu(norm?(x) Wg^T) * (norm?(x) Wu^T), W from interleave_gate_up (decode_linear_swiglu)."""
    ph = _phase(XB_DECODE_SWIGLU, x, w_gate_up, xnorm)
    _cuda(y)
    if tuple(y.shape) != (x.shape[0], w_gate_up.shape[0] // 2):
        raise ValueError("y must be [M, n_out]")
    ph.y, ph.ldy = y.data_ptr(), _mat(y, "y")
    return ph


def chain_residual(x, weight, bias, residual, y, stats=None, stats_kind=None, xnorm=None) -> DecodePhase:
    """Phase: y = residual + bf16(norm?(x) @ weight^T + bias), with the row
    statistics of y in `stats` (a decode_stats buffer) for the next norm
    (decode_linear_residual)."""
    ph = _phase(XB_DECODE_RESIDUAL, x, weight, xnorm)
    _cuda(bias, residual, y, stats)
    M, N = x.shape[0], weight.shape[0]
    if tuple(residual.shape) != (M, N) or tuple(y.shape) != (M, N):
        raise ValueError("residual and y must be [M, N]")
    ph.bias = bias.data_ptr() if bias is not None else None
    ph.residual, ph.ldr = residual.data_ptr(), _mat(residual, "residual")
    ph.y, ph.ldy = y.data_ptr(), _mat(y, "y")
    if stats is not None:
        if stats.dtype != torch.float32 or stats.numel() < ((N + 127) // 128) * 128:
            raise ValueError("stats must be a float32 decode_stats buffer for N")
        ph.stats_out, ph.stats_kind = stats.data_ptr(), _NORM_KIND[stats_kind]
    return ph


_chain_syncs: dict = {}


def decode_chain_sync(device) -> torch.Tensor:
    """The chain's grid-barrier counters for the current workspace slot: 16
    bytes, zero between launches, one buffer per (device, slot)."""
    device = torch.device(device)
    if device.index is None:
        device = torch.device(device.type, torch.cuda.current_device())
    key = (device, _slot[0])
    if key not in _chain_syncs:
        _chain_syncs[key] = torch.zeros(4, dtype=torch.int32, device=device)
    return _chain_syncs[key]


def decode_chain(phases, sync) -> None:
    """Run 1..4 decode-chain phases in one launch (xb_decode_chain_bf16)."""
    if not 0 < len(phases) <= CHAIN_MAX_PHASES:
        raise ValueError(f"a decode chain has 1..{CHAIN_MAX_PHASES} phases")
    _cuda(sync)
    arr = (DecodePhase * len(phases))(*phases)
    _lib.call("xb_decode_chain_bf16", ctypes.addressof(arr), len(phases), sync.data_ptr(), _stream())


def device_status() -> int:
    """Read and clear the device status word (0 = fine, -4 = a kernel timed out)."""
    st = ctypes.c_int(0)
    _lib.call("xb_device_status", _stream(), ctypes.byref(st))
    return st.value


# --------------------------------------------------------------------------- Qwen2.5 decoder pieces


def embedding(table, ids, out=None):
    """out[..., :] = table[ids] (bf16 rows), as model.py:911."""
    _cuda(table, ids, out)
    if table.dtype != torch.bfloat16 or ids.dtype != torch.int64:
        raise TypeError("embedding takes a bf16 table and int64 ids")
    ids_c = ids.contiguous()
    rows = ids_c.numel()
    dim = table.shape[1]
    if out is None:
        out = torch.empty(tuple(ids.shape) + (dim,), dtype=torch.bfloat16, device=table.device)
    _lib.call("xb_embedding_bf16", table.data_ptr(), ids_c.data_ptr(), out.data_ptr(), rows, dim, table.shape[0],
              _stream())
    return out


def embedding_pos(table, pos_table, ids, pos_offset=0, out=None):
    """out[b, s, :] = bf16(table[ids[b, s]] + pos_table[pos_offset + s]): token
    plus learned position embedding (examples/gpt2/model.py:866-876)."""
    _cuda(table, pos_table, ids, out)
    if table.dtype != torch.bfloat16 or pos_table.dtype != torch.bfloat16 or ids.dtype != torch.int64:
        raise TypeError("embedding_pos takes bf16 tables and int64 ids")
    if ids.dim() != 2:
        raise ValueError("ids must be [batch, seq]")
    ids_c = ids.contiguous()
    B, S = ids_c.shape
    dim = table.shape[1]
    if out is None:
        out = torch.empty((B, S, dim), dtype=torch.bfloat16, device=table.device)
    _lib.call("xb_embedding_pos_bf16", table.data_ptr(), pos_table.data_ptr(), ids_c.data_ptr(), out.data_ptr(),
              B * S, S, dim, table.shape[0], pos_table.shape[0], pos_offset, _stream())
    return out


def launch_count() -> int:
    """Kernels launched by the library so far (graph replays not counted)."""
    n = ctypes.c_uint64(0)
    _lib.call("xb_launch_count", ctypes.byref(n))
    return n.value


def token_status() -> int:
    """1 if an embedding met an out-of-vocabulary id since the last call, else 0."""
    st = ctypes.c_int(0)
    _lib.call("xb_token_status", _stream(), ctypes.byref(st))
    return st.value


_rope_halves: dict = {}


def rope_tables_repeat_halves(cos_t, sin_t) -> bool:
    """Whether every row of both RoPE tables repeats its first half in its
    second (rotate-half tables built from duplicated frequencies); checked
    once per pair of tables (keyed by their address, shape, strides and
    version; the entry keeps the tables alive, so no other tensor can take
    their address while the answer is cached)."""
    key = (cos_t.data_ptr(), sin_t.data_ptr(), cos_t.shape, cos_t.stride(), sin_t.stride(), cos_t._version,
           sin_t._version)
    hit = _rope_halves.get(key)
    if hit is None:
        h = cos_t.shape[-1] // 2
        v = bool(torch.equal(cos_t[..., :h], cos_t[..., h:]) and torch.equal(sin_t[..., :h], sin_t[..., h:]))
        hit = _rope_halves[key] = (v, cos_t, sin_t)
    return hit[0]


def linear_qkv_rope(x, w_qkv, b_qkv, cos_t, sin_t, q_out, k_cache, v_cache, batch, seq, n_head, n_kv_head, head_dim,
                    pos_offset, rope_dup: bool | None = None):
    """Prefill QKV projection + RoPE (none when the tables are None) + KV-cache
    write in one GEMM (the epilogue finishes each head slot): the results of
    linear() followed by rope_kv(), without the qkv activations in memory.

    ``rope_dup`` says that every table row repeats its first half in its
    second (the epilogue then reads half rows); None checks the tables once
    (a device comparison and a host read, cached per table pair)."""
    _cuda(x, w_qkv, b_qkv, cos_t, sin_t, q_out, k_cache, v_cache)
    if (cos_t is None) != (sin_t is None):
        raise ValueError("give both RoPE tables or neither")
    if cos_t is not None and cos_t.shape[0] < pos_offset + seq:
        raise ValueError("RoPE tables are shorter than the positions")
    x2 = x.reshape(-1, x.shape[-1])
    K = x2.shape[1]
    if cos_t is None:
        dup = False
    else:
        dup = rope_tables_repeat_halves(cos_t, sin_t) if rope_dup is None else bool(rope_dup)
    _lib.call("xb_linear_rope_kv_bf16", x2.data_ptr(), w_qkv.data_ptr(),
              b_qkv.data_ptr() if b_qkv is not None else None,
              cos_t.data_ptr() if cos_t is not None else None, sin_t.data_ptr() if sin_t is not None else None,
              int(dup), q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), batch, seq, n_head, n_kv_head,
              head_dim, k_cache.shape[2], pos_offset, K, _mat(x2, "x"), _mat(w_qkv, "w"), _stream())


def rope_kv(qkv, cos_t, sin_t, q_out, k_cache, v_cache, batch, seq, n_head, n_kv_head, head_dim, pos_offset):
    """RoPE on the fused QKV projection + KV-cache write (model.py:851-867).
    cos_t = sin_t = None: heads are split and written unrotated (GPT-2)."""
    _cuda(qkv, cos_t, sin_t, q_out, k_cache, v_cache)
    if (cos_t is None) != (sin_t is None):
        raise ValueError("give both RoPE tables or neither")
    if cos_t is not None and cos_t.shape[0] < pos_offset + seq:
        raise ValueError("RoPE tables are shorter than the positions")
    _lib.call("xb_rope_kv_bf16", qkv.data_ptr(), cos_t.data_ptr() if cos_t is not None else None,
              sin_t.data_ptr() if sin_t is not None else None, q_out.data_ptr(),
              k_cache.data_ptr(), v_cache.data_ptr(), batch, seq, n_head, n_kv_head, head_dim, k_cache.shape[2],
              pos_offset, _stream())


def attention(q, k_cache, v_cache, out, batch, seq, n_head, n_kv_head, head_dim, pos_offset, scale):
    """Causal GQA attention over the cache (kernels/attention.py:27-122)."""
    _cuda(q, k_cache, v_cache, out)
    need = ctypes.c_size_t(0)
    _lib.call("xb_attention_workspace_size", batch, seq, n_head, n_kv_head, pos_offset, ctypes.byref(need))
    ws = _workspace(q.device, need.value) if need.value else None
    _lib.call("xb_attention_bf16", q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(), batch, seq,
              n_head, n_kv_head, head_dim, k_cache.shape[2], pos_offset, float(scale),
              ws.data_ptr() if ws is not None else None, ws.numel() * 4 if ws is not None else 0, _stream())
    return out


def linear_argmax_workspace_bytes(M: int, N: int) -> int:
    need = ctypes.c_size_t(0)
    _lib.call("xb_linear_argmax_workspace_size", M, N, ctypes.byref(need))
    return need.value


def linear_argmax(x, weight, out=None):
    """argmax_n (x @ weight^T)[m, n] per row (int64, torch.argmax semantics on
    the fp32 logits) without writing the logits: the LM head and the greedy
    next token of a decode step in one GEMM plus a small reduction."""
    _cuda(x, weight, out)
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise TypeError("linear_argmax takes bf16 x and weight")
    M, K = x.shape
    N = weight.shape[0]
    if weight.shape[1] != K:
        raise ValueError("shape mismatch")
    if out is None:
        out = torch.empty(M, dtype=torch.int64, device=x.device)
    ws = _workspace(x.device, linear_argmax_workspace_bytes(M, N))
    _lib.call("xb_linear_argmax_bf16", x.data_ptr(), weight.data_ptr(), M, N, K, _mat(x, "x"),
              _mat(weight, "weight"), out.data_ptr(), ws.data_ptr(), ws.numel() * 4, _stream())
    return out


def argmax(x, out=None):
    """First index of the row maximum of a 2-D fp32 tensor (torch.argmax(-1))."""
    _cuda(x, out)
    if x.dtype != torch.float32 or x.dim() != 2 or x.stride(1) != 1:
        raise TypeError("argmax takes a row-major 2-D float32 tensor")
    if out is None:
        out = torch.empty(x.shape[0], dtype=torch.int64, device=x.device)
    _lib.call("xb_argmax_f32", x.data_ptr(), x.shape[0], x.shape[1], x.stride(0), out.data_ptr(), _stream())
    return out

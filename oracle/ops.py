"""ORACLE (test infrastructure): the reference examples' PyTorch CPU checks, restated.

Each function evaluates, on CPU, the expression the cited example compares its
kernel output against (``provider == "torch"`` branch).  Inputs and outputs
are torch CPU tensors in the example's dtype.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def vecadd(a, b):
    """examples/vec-add/vec-add.py:49 -- torch.add(a, b)."""
    return torch.add(a, b)


def axpy(x, y, alpha):
    """examples/axpy/axpy.py:40 -- alpha * x + y (alpha * x rounds to x.dtype first)."""
    return alpha * x + y


def relu(x):
    """examples/relu/relu.py:35 -- torch.relu(x)."""
    return torch.relu(x)


def leaky_relu(x, slope=0.01):
    """examples/leaky_relu/leaky_relu.py:40 -- F.leaky_relu(x, negative_slope=0.01)."""
    return F.leaky_relu(x, negative_slope=slope)


def gelu(x):
    """examples/gelu/gelu.py:40 -- x * torch.sigmoid(1.702 * x.float()).to(dtype)."""
    return x * torch.sigmoid(1.702 * x.float()).to(x.dtype)


def gelu_tanh(x):
    """tanh-form GELU of examples/gpt2/kernels/gelu.py:4-12 (HF gelu_new):
    F.gelu(x, approximate="tanh") evaluated in fp32."""
    return F.gelu(x.float(), approximate="tanh").to(x.dtype)


def sigmoid(x):
    """examples/sigmoid/sigmoid.py:39 -- torch.sigmoid(x)."""
    return torch.sigmoid(x)


def silu(x):
    """examples/silu/silu.py:39 -- F.silu(x)."""
    return F.silu(x)


def swiglu(gate, up):
    """examples/swiglu/swiglu.py:43 -- F.silu(gate) * up."""
    return F.silu(gate) * up


def row_center(x):
    """examples/average_pool/average_pool.py:61-64 -- (x.f32 - mean(x.f32, -1)).to(dtype)."""
    xf = x.float()
    return (xf - xf.mean(dim=-1, keepdim=True)).to(x.dtype)


def avg_pool2d_2x2(x):
    """2x2 / stride-2 torch avg_pool2d (the 2-D pooling workload's oracle)."""
    return F.avg_pool2d(x, 2, 2)


def softmax(x):
    """examples/test_softmax/test_softmax.py:77 -- torch.softmax(x, axis=1)."""
    return torch.softmax(x, axis=-1)


def layernorm(x, gamma=None, beta=None, eps=1e-5):
    """Row layernorm in fp32.  examples/test_layernorm/test_layernorm.py:36-53
    (mean, variance, 1/sqrt(var+eps), gamma=1, beta=0 when absent) with the
    affine form of examples/gpt2/kernels/layernorm.py:114-160."""
    n = x.shape[-1]
    g = gamma.float() if gamma is not None else None
    b = beta.float() if beta is not None else None
    return F.layer_norm(x.float(), (n,), g, b, eps).to(x.dtype)


def rms_norm(x, eps=1e-5):
    """examples/rms_norm/rms_norm.py:64-68."""
    x_f32 = x.float()
    mean_sq = (x_f32 * x_f32).mean(dim=-1, keepdim=True)
    rstd = torch.rsqrt(mean_sq + eps)
    return (x_f32 * rstd).to(x.dtype)


def weighted_rms_norm(x, w, eps=1e-5):
    """examples/weighted_rms_norm/weighted_rms_norm.py:68-73."""
    x_f32 = x.float()
    w_f32 = w.float()
    mean_sq = (x_f32 * x_f32).mean(dim=-1, keepdim=True)
    rstd = torch.rsqrt(mean_sq + eps)
    return (x_f32 * rstd * w_f32.unsqueeze(0)).to(x.dtype)


def matmul_int(a, b):
    """examples/matmul_i8_m128_n64_k64/matmul_i8_m128_n64_k64.py:63 --
    torch.matmul(a.to(int32), b.to(int32)); int32 arithmetic wraps mod 2^32,
    which is also the int16 semantics (int32 accumulator)."""
    return torch.matmul(a.to(torch.int32), b.to(torch.int32))


def matmul_int_exact(a, b):
    """int64 product reduced mod 2^32 into int32 (independent check of matmul_int)."""
    c = torch.matmul(a.to(torch.int64), b.to(torch.int64))
    c = c & 0xFFFFFFFF
    c = torch.where(c >= 2**31, c - 2**32, c)
    return c.to(torch.int32)


def matmul_bf16(a, b):
    """examples/matmul_bf16_m64_n64_k64/matmul_bf16_m64_n64_k64.py:58 --
    torch.matmul(a, b).to(float32) on bf16 inputs."""
    return torch.matmul(a, b).to(torch.float32)


def matmul_bf16_f32acc(a, b):
    """examples/autotune-matmul/matmul.py:78 -- a.to(f32) @ b.to(f32)."""
    return a.to(torch.float32) @ b.to(torch.float32)


# Tolerances the examples assert with (atol, rtol), by op.
EXAMPLE_TOL = {
    "vecadd": (1e-2, 1e-2),  # vec-add.py:62
    "axpy": (1e-2, 1e-2),  # axpy.py:54
    "relu": (1e-2, 1e-2),  # relu.py:48
    "leaky_relu": (1e-2, 1e-2),  # leaky_relu.py:53
    "gelu": (1e-1, 1e-1),  # gelu.py:53
    "sigmoid": (1e-1, 1e-1),  # sigmoid.py:52
    "silu": (1e-1, 1e-1),  # silu.py:52
    "swiglu": (1e-1, 1e-1),  # swiglu.py:56
    "avg_pool": (5e-1, 1e-1),  # average_pool.py:77
    "softmax": (1e-2, 1e-2),  # test_softmax.py:81
    "rms_norm": (5e-1, 1e-1),  # rms_norm.py:82
    "weighted_rms_norm": (5e-1, 1e-1),  # weighted_rms_norm.py:88
    "matmul_i8": (0, 0),  # matmul_i8_m128_n64_k64.py:89
    "matmul_bf16": (1e1, 1e-1),  # matmul_bf16_m64_n64_k64.py:85
}


def matmul_f32_bf16emu(a_km, b):
    """bf16-emulated f32 GEMM with A stored transposed (K x M):
    examples/matmul_f32_m64_n32_k16_padded_atransposed/
    matmul_f32_m64_n32_k16_padded_atransposed.py:140-161 -- the f32 inputs
    rounded to bf16 (ml_dtypes astype, nearest even), products and sums in
    f32.  Returns C [M, N] f32."""
    a = a_km.to(torch.bfloat16).float()
    bb = b.to(torch.bfloat16).float()
    return a.t() @ bb


def mul(x, y):
    """examples/load_2d_block/test_load_2d_tensor_block.py:118 -- expected = x * y."""
    return x * y

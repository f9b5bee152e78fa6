"""Drop-in launchers with the reference examples' kernel signatures.

Each example in the reference defines a ``@triton.jit`` kernel and launches it
as ``kernel[grid](*args, **constexprs)`` (e.g. examples/vec-add/vec-add.py:53-59).
The objects here accept exactly those calls, so an example swaps

    @triton.jit
    def vecadd(A, B, C, n_elements, BLOCK_SIZE_N): ...

for ``from xb200.kernels import vecadd`` and keeps its inputs and checks.

Launch semantics mirror the reference's NPU launcher
(amd_triton_npu/backend/driver.py:1439-1558):

* arguments bind to the kernel's parameter names; a callable grid is called
  with that name -> value dict (Triton's ``META``);
* host (CPU) tensors are copied to the current CUDA device, the operator runs
  there, and only the LAST pointer argument is copied back into its host
  tensor (driver.py:1546-1548, "the last tensor is the only output");
* CUDA tensors are used in place (no copies);
* errors raise ``RuntimeError`` (driver.py:1553-1556) -- here ``XbError``.

The returned object carries ``.asm["ttsharedir"]`` because the examples write
that field to ``tt.shared.mlir`` after each launch; xb200 compiles no MLIR,
so it holds a one-line description of the CUDA entry point that ran.

Where a reference kernel takes no row count (the row-reduction kernels), the
rows processed are ``grid[0] * BLOCK``, exactly the rows its programs cover.
"""

from __future__ import annotations

import inspect
from typing import Callable

import torch

from . import ops


class LaunchResult:
    def __init__(self, name: str, entry: str):
        self.name = name
        self.asm = {"ttsharedir": f"// xb200: {name} ran as CUDA entry point {entry} (sm_100a); no MLIR is produced\n"}

    def __repr__(self) -> str:
        return f"LaunchResult({self.name})"


class XbKernel:
    """A reference kernel signature bound to an xb200 CUDA implementation."""

    def __init__(self, name: str, entry: str, run: Callable):
        self.__name__ = name
        self.name = name
        self.entry = entry
        self.run = run
        sig = inspect.signature(run)
        self.params = [p for p in sig.parameters if p != "grid"]

    def __getitem__(self, grid):
        def launcher(*args, **kwargs):
            return self._launch(grid, args, kwargs)

        return launcher

    def _bind(self, args, kwargs) -> dict:
        if len(args) > len(self.params):
            raise TypeError(f"{self.name}: too many positional arguments")
        bound = dict(zip(self.params, args))
        for k, v in kwargs.items():
            if k not in self.params:
                raise TypeError(f"{self.name}: unexpected argument {k!r}")
            if k in bound:
                raise TypeError(f"{self.name}: argument {k!r} given twice")
            bound[k] = v
        missing = [p for p in self.params if p not in bound]
        if missing:
            raise TypeError(f"{self.name}: missing arguments {missing}")
        return bound

    def _launch(self, grid, args, kwargs) -> LaunchResult:
        bound = self._bind(args, kwargs)
        g = grid(dict(bound)) if callable(grid) else grid
        g = tuple(g) + (1,) * (3 - len(tuple(g)))
        ptr_names = [k for k in self.params if isinstance(bound[k], torch.Tensor)]
        host = [k for k in ptr_names if bound[k].device.type == "cpu"]
        if host:
            if not torch.cuda.is_available():
                raise RuntimeError(f"{self.name}: no CUDA device available (xb200 has no CPU fallback)")
            dev = torch.device("cuda", torch.cuda.current_device())
            dbound = dict(bound)
            for k in ptr_names:
                dbound[k] = bound[k].to(dev)
            self.run(grid=g, **dbound)
            last = ptr_names[-1]
            bound[last].copy_(dbound[last])  # blocking device->host copy
        else:
            self.run(grid=g, **bound)
        return LaunchResult(self.name, self.entry)


def _n(t: torch.Tensor, n: int) -> torch.Tensor:
    flat = t.reshape(-1)
    if flat.numel() < n:
        raise ValueError(f"tensor has {flat.numel()} elements, kernel was told {n}")
    return flat[:n]


def _rows_view(t: torch.Tensor, rows: int, cols: int, stride_row: int, stride_col: int = 1) -> torch.Tensor:
    if stride_col != 1:
        raise ValueError("xb200 row kernels need a unit column stride")
    need = (rows - 1) * stride_row + cols if rows else 0
    if t.numel() < need:
        raise ValueError(f"tensor too small for {rows} rows of stride {stride_row}")
    return torch.as_strided(t, (rows, cols), (stride_row, 1), t.storage_offset())


# ----------------------------------------------------------------------------- elementwise


def _vecadd(A, B, C, n_elements, BLOCK_SIZE_N, grid):
    ops.vecadd(_n(A, n_elements), _n(B, n_elements), out=_n(C, n_elements))


def _axpy(X, Y, OUT, alpha, n_elements, BLOCK_SIZE, grid):
    ops.axpy(_n(X, n_elements), _n(Y, n_elements), alpha, out=_n(OUT, n_elements))


def _unary(fn):
    def run(X, Y, n_elements, BLOCK_SIZE, grid):
        fn(_n(X, n_elements), out=_n(Y, n_elements))

    return run


def _leaky(X, Y, n_elements, BLOCK_SIZE, grid):
    # examples/leaky_relu/leaky_relu.py:30 hard-codes the 0.01 slope in the kernel body
    ops.leaky_relu(_n(X, n_elements), 0.01, out=_n(Y, n_elements))


def _swiglu(GATE, UP, OUT, n_elements, BLOCK_SIZE, grid):
    ops.swiglu(_n(GATE, n_elements), _n(UP, n_elements), out=_n(OUT, n_elements))


vecadd = XbKernel("vecadd", "xb_vecadd", _vecadd)
axpy_kernel = XbKernel("axpy_kernel", "xb_axpy", _axpy)
relu_kernel = XbKernel("relu_kernel", "xb_relu", _unary(ops.relu))
leaky_relu_kernel = XbKernel("leaky_relu_kernel", "xb_leaky_relu", _leaky)
gelu_kernel = XbKernel("gelu_kernel", "xb_gelu", _unary(ops.gelu))
gelu_kernel_gpu = XbKernel("gelu_kernel_gpu", "xb_gelu_tanh", _unary(ops.gelu_tanh))
sigmoid_kernel = XbKernel("sigmoid_kernel", "xb_sigmoid", _unary(ops.sigmoid))
silu_kernel = XbKernel("silu_kernel", "xb_silu", _unary(ops.silu))
swiglu_kernel = XbKernel("swiglu_kernel", "xb_swiglu", _swiglu)


# ----------------------------------------------------------------------------- row reductions


def _avg_pool(X, Y, N, BLOCK_M, BLOCK_N, grid):
    rows = grid[0] * BLOCK_M
    ops.row_center(_rows_view(X, rows, BLOCK_N, N), out=_rows_view(Y, rows, BLOCK_N, N))


def _softmax(input_ptr, output_ptr, input_stride_row, input_stride_col, output_stride_row, output_stride_col, n_cols,
             BLOCK_SIZE, grid):
    rows = grid[0] * BLOCK_SIZE
    ops.softmax(_rows_view(input_ptr, rows, n_cols, input_stride_row, input_stride_col),
                out=_rows_view(output_ptr, rows, n_cols, output_stride_row, output_stride_col))


def _layernorm(input_ptr, output_ptr, input_stride_row, input_stride_col, output_stride_row, output_stride_col, n_cols,
               eps, BLOCK_SIZE, grid):
    rows = grid[0] * BLOCK_SIZE
    ops.layernorm(_rows_view(input_ptr, rows, n_cols, input_stride_row, input_stride_col), None, None, eps,
                  out=_rows_view(output_ptr, rows, n_cols, output_stride_row, output_stride_col))


def _rms(X, Y, N, eps, BLOCK_M, BLOCK_N, grid):
    rows = grid[0] * BLOCK_M
    ops.rms_norm(_rows_view(X, rows, BLOCK_N, N), None, eps, out=_rows_view(Y, rows, BLOCK_N, N))


def _wrms(X, W, Y, N, eps, BLOCK_M, BLOCK_N, grid):
    rows = grid[0] * BLOCK_M
    ops.rms_norm(_rows_view(X, rows, BLOCK_N, N), _n(W, BLOCK_N), eps, out=_rows_view(Y, rows, BLOCK_N, N))


def _avg_pool2d(X, Y, planes, H, W, BLOCK, grid):
    x = X.reshape(-1)[: planes * H * W].view(planes, H, W)
    ops.avg_pool2d_2x2(x, out=Y.reshape(-1)[: planes * (H // 2) * (W // 2)].view(planes, H // 2, W // 2))


avg_pool_kernel = XbKernel("avg_pool_kernel", "xb_row_center", _avg_pool)
# The 2-D (NCHW, 2x2 / stride 2) pooling form has no reference kernel; this
# launcher gives it the same calling convention as the others.
avg_pool2d_kernel = XbKernel("avg_pool2d_kernel", "xb_avg_pool2d_2x2", _avg_pool2d)
softmax_kernel = XbKernel("softmax_kernel", "xb_softmax", _softmax)
_layer_norm_fwd_fused = XbKernel("_layer_norm_fwd_fused", "xb_layernorm", _layernorm)
rms_norm_kernel = XbKernel("rms_norm_kernel", "xb_rms_norm", _rms)
weighted_rms_norm_kernel = XbKernel("weighted_rms_norm_kernel", "xb_rms_norm", _wrms)


# ----------------------------------------------------------------------------- GEMMs


def _mat_view(t, rows, cols, stride_r, stride_c, name):
    if stride_c != 1:
        raise ValueError(f"{name}: xb200 GEMMs need row-major operands (unit column stride)")
    need = (rows - 1) * stride_r + cols if rows else 0
    if t.numel() < need:
        raise ValueError(f"{name}: tensor too small for [{rows}, {cols}] with row stride {stride_r}")
    return torch.as_strided(t, (rows, cols), (stride_r, 1), t.storage_offset())


def _matmul(A, B, C, M, N, K, stride_am, stride_ak, stride_bk, stride_bn, stride_cm, stride_cn, BLOCK_SIZE_M,
            BLOCK_SIZE_N, BLOCK_SIZE_K, grid):
    a = _mat_view(A, M, K, stride_am, stride_ak, "A")
    b = _mat_view(B, K, N, stride_bk, stride_bn, "B")
    c = _mat_view(C, M, N, stride_cm, stride_cn, "C")
    if A.dtype == torch.int8:
        ops.matmul_i8(a, b, out=c)
    elif A.dtype == torch.int16:
        ops.matmul_i16(a, b, out=c)
    else:
        ops.matmul_bf16(a, b, out=c)


class _Autotuned(XbKernel):
    """An autotuned reference kernel: block sizes the caller leaves out come
    from its first config (examples/autotune-matmul/matmul.py:16-19), the way
    Triton's autotuner fills META before calling the grid."""

    def __init__(self, name, entry, run, defaults):
        super().__init__(name, entry, run)
        self.defaults = defaults

    def _bind(self, args, kwargs):
        kw = dict(self.defaults)
        kw.update(kwargs)
        for k in list(self.defaults):
            if k in self.params[: len(args)]:
                kw.pop(k)
        return super()._bind(args, kw)


def _padded_matmul(A, B, C, M, N, K, stride_am, stride_ak, stride_bk, stride_bn, stride_cm, stride_cn, BLOCK_SIZE_M,
                   BLOCK_SIZE_N, BLOCK_SIZE_K, grid):
    # examples/matmul_f32_m64_n32_k16_padded_atransposed: stride_am == 1 means
    # A is stored transposed (K x M, row pitch stride_ak); f32 operands run
    # with bf16 emulation
    if stride_am == 1 and M > 1:
        a, trans = _mat_view(A, K, M, stride_ak, 1, "A"), True
    else:
        a, trans = _mat_view(A, M, K, stride_am, stride_ak, "A"), False
    b = _mat_view(B, K, N, stride_bk, stride_bn, "B")
    c = _mat_view(C, M, N, stride_cm, stride_cn, "C")
    ops.matmul_f32_bf16emu(a, b, a_transposed=trans, out=c)


def _load_2d(x_ptr, y_ptr, z_ptr, n_rows, n_cols, stride_0, stride_1, VEC_REG_SIZE_ROW, VEC_REG_SIZE_COL,
             BLOCK_SIZE_ROW, BLOCK_SIZE_COL, grid):
    # examples/load_2d_block/test_load_2d_tensor_block.py:27-82: program
    # (p0, p1) loads the BLOCK_SIZE_ROW x BLOCK_SIZE_COL block at (p0 * BR,
    # p1 * BC) of x and y through 4-D block pointers of VEC_REG sub-tiles and
    # stores x * y at the same places of z: the grid covers these rows / cols
    rows = min(n_rows, grid[0] * BLOCK_SIZE_ROW)
    cols = min(n_cols, grid[1] * BLOCK_SIZE_COL)
    if BLOCK_SIZE_ROW % VEC_REG_SIZE_ROW or BLOCK_SIZE_COL % VEC_REG_SIZE_COL:
        raise ValueError("block sizes must be whole vector-register tiles")
    views = [_mat_view(t, rows, cols, stride_0, stride_1, n) for t, n in ((x_ptr, "x"), (y_ptr, "y"), (z_ptr, "z"))]
    ops.mul_2d(views[0], views[1], views[2])


bare_matmul_i8 = XbKernel("bare_matmul_i8", "xb_matmul_i8", _matmul)
padded_matmul_kernel = XbKernel("padded_matmul_kernel", "xb_matmul_f32_bf16emu", _padded_matmul)
load_2d_block_kernel = XbKernel("kernel", "xb_mul_2d", _load_2d)
bare_matmul = XbKernel("bare_matmul", "xb_matmul_bf16", _matmul)
bare_matmul_autotuned = _Autotuned("bare_matmul", "xb_matmul_bf16", _matmul, {"BLOCK_SIZE_M": 256})


REGISTRY = {
    k.name: k
    for k in (vecadd, axpy_kernel, relu_kernel, leaky_relu_kernel, gelu_kernel, gelu_kernel_gpu, sigmoid_kernel,
              silu_kernel, swiglu_kernel, avg_pool_kernel, avg_pool2d_kernel, softmax_kernel, _layer_norm_fwd_fused,
              rms_norm_kernel, weighted_rms_norm_kernel, bare_matmul_i8, bare_matmul, padded_matmul_kernel)
}
REGISTRY["load_2d_block_kernel"] = load_2d_block_kernel  # the example names its kernel plain `kernel`

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

Kernels whose programs cover independent units along one leading dimension
(elements, rows, planes, GEMM rows of A and C) carry a ``Split``.  When every
pointer argument is a contiguous host tensor, such a launch copies only what
the kernel reads and brings back only the region of the output it writes, so
the output's other elements stay as they were, as under the copy-everything
path.  With pinned host tensors the launch is cut into pieces of a few tens of
MB: pieces' uploads, kernels and downloads run on three streams, so the
host-to-device and device-to-host copies overlap each other and the kernels.
The call still returns only after the last byte is back in the host tensor.

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


class Split:
    """How a launch divides into independent pieces along its leading dimension.

    ``units(b, g)`` is the number of units the launch covers (elements, rows,
    planes); a piece is a whole number of ``align(b)`` units except the last.
    ``pitch(b)`` maps each pointer that divides to its elements per unit; the
    other pointers are read whole by every piece.  ``span(b)`` is the elements
    of one unit the output is written over: the written region is one
    contiguous range only when it equals the output's pitch.  ``piece(b, g, n)``
    gives the scalar arguments and grid that make a launch cover ``n`` units.
    """

    def __init__(self, units, pitch, span, piece, align=lambda b: 1):
        self.units, self.pitch, self.span, self.piece, self.align = units, pitch, span, piece, align


_PIECE_BYTES = 32 << 20  # bytes crossing PCIe per piece (uploads + download)
_MAX_PIECES = 256
_SIDE_STREAMS: dict = {}


def _side_streams(dev: torch.device):
    if dev.index not in _SIDE_STREAMS:
        _SIDE_STREAMS[dev.index] = (torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev))
    return _SIDE_STREAMS[dev.index]


def _span_bytes(t: torch.Tensor):
    lo = t.data_ptr()
    return lo, lo + t.numel() * t.element_size()


class XbKernel:
    """A reference kernel signature bound to an xb200 CUDA implementation."""

    def __init__(self, name: str, entry: str, run: Callable, split: Split | None = None):
        self.__name__ = name
        self.name = name
        self.entry = entry
        self.run = run
        self.split = split
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
            plan = self._plan(bound, g, ptr_names, host)
            if plan is not None:
                self._launch_pieces(bound, g, ptr_names, dev, *plan)
            else:
                dbound = dict(bound)
                for k in ptr_names:
                    dbound[k] = bound[k].to(dev)
                self.run(grid=g, **dbound)
                last = ptr_names[-1]
                bound[last].copy_(dbound[last])  # blocking device->host copy
        else:
            self.run(grid=g, **bound)
        return LaunchResult(self.name, self.entry)

    def _plan(self, bound, g, ptr_names, host):
        """(units, pitch, units per piece, pinned) when the launch may copy
        only what it reads and writes; None keeps the copy-everything path
        (which also raises the runner's own errors for malformed arguments)."""
        sp = self.split
        if sp is None or len(host) != len(ptr_names) or len(ptr_names) < 2:
            return None
        tensors = [bound[k] for k in ptr_names]
        if not all(t.is_contiguous() for t in tensors):
            return None
        try:
            units, pitch = int(sp.units(bound, g)), sp.pitch(bound)
            span, align = int(sp.span(bound)), int(sp.align(bound))
        except (TypeError, ValueError, ZeroDivisionError):
            return None
        out = ptr_names[-1]
        if units <= 0 or align <= 0 or out not in pitch or span != pitch[out] or span <= 0:
            return None
        for k, p in pitch.items():
            if k not in ptr_names or p <= 0 or bound[k].numel() < units * p:
                return None
        # the output may be one of the inputs exactly (an in-place launch), but
        # must not partly overlap any other pointer's memory
        olo, ohi = _span_bytes(bound[out])
        for k in ptr_names[:-1]:
            lo, hi = _span_bytes(bound[k])
            if lo < ohi and olo < hi:
                same = lo == olo and bound[k].dtype == bound[out].dtype and pitch.get(k) == pitch[out]
                if not same:
                    return None
        unit_bytes = sum(pitch[k] * bound[k].element_size() for k in pitch)
        pinned = all(t.is_pinned() for t in tensors)
        if pinned:
            per = max(align, (_PIECE_BYTES // max(1, unit_bytes)) // align * align)
            fewest = -(-units // _MAX_PIECES)
            per = max(per, -(-fewest // align) * align)
        else:
            per = units  # pageable memory: the copies are synchronous, one piece
        return units, pitch, per, pinned

    def _launch_pieces(self, bound, g, ptr_names, dev, units, pitch, per, nb):
        out = ptr_names[-1]
        cur = torch.cuda.current_stream(dev)
        up, down = _side_streams(dev)
        start = torch.cuda.Event()
        start.record(cur)
        flat = {k: bound[k].reshape(-1) for k in ptr_names}
        dbuf = {k: torch.empty(units * pitch[k] if k in pitch else flat[k].numel(), dtype=flat[k].dtype, device=dev)
                for k in ptr_names}
        up.wait_event(start)
        try:
            with torch.cuda.stream(up):
                for k in ptr_names:
                    if k not in pitch:
                        dbuf[k].copy_(flat[k], non_blocking=nb)
            for lo in range(0, units, per):
                n = min(per, units - lo)
                with torch.cuda.stream(up):
                    for k in ptr_names:
                        if k in pitch and k != out:
                            a, b = lo * pitch[k], (lo + n) * pitch[k]
                            dbuf[k][a:b].copy_(flat[k][a:b], non_blocking=nb)
                    ready = torch.cuda.Event()
                    ready.record(up)
                cur.wait_event(ready)
                args = dict(bound)
                args.update({k: dbuf[k][lo * pitch[k]:] if k in pitch else dbuf[k] for k in ptr_names})
                scal, pg = self.split.piece(bound, g, n)
                args.update(scal)
                self.run(grid=pg, **args)
                computed = torch.cuda.Event()
                computed.record(cur)
                down.wait_event(computed)
                with torch.cuda.stream(down):
                    a, b = lo * pitch[out], (lo + n) * pitch[out]
                    flat[out][a:b].copy_(dbuf[out][a:b], non_blocking=nb)
        finally:
            # every copy into or out of the device buffers ends before they are freed
            done = torch.cuda.Event()
            done.record(down)
            up_done = torch.cuda.Event()
            up_done.record(up)
            cur.wait_event(up_done)
            cur.wait_event(done)
            up_done.synchronize()
            done.synchronize()  # the output is complete in host memory on return


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


def _flat(*ptrs):
    # one unit per element; pieces start on 4096-element boundaries, so each
    # piece's pointers keep the alignment of the vectorised loads
    return Split(units=lambda b, g: b["n_elements"], pitch=lambda b: {k: 1 for k in ptrs}, span=lambda b: 1,
                 piece=lambda b, g, n: ({"n_elements": n}, g), align=lambda b: 4096)


vecadd = XbKernel("vecadd", "xb_vecadd", _vecadd, _flat("A", "B", "C"))
axpy_kernel = XbKernel("axpy_kernel", "xb_axpy", _axpy, _flat("X", "Y", "OUT"))
relu_kernel = XbKernel("relu_kernel", "xb_relu", _unary(ops.relu), _flat("X", "Y"))
leaky_relu_kernel = XbKernel("leaky_relu_kernel", "xb_leaky_relu", _leaky, _flat("X", "Y"))
gelu_kernel = XbKernel("gelu_kernel", "xb_gelu", _unary(ops.gelu), _flat("X", "Y"))
gelu_kernel_gpu = XbKernel("gelu_kernel_gpu", "xb_gelu_tanh", _unary(ops.gelu_tanh), _flat("X", "Y"))
sigmoid_kernel = XbKernel("sigmoid_kernel", "xb_sigmoid", _unary(ops.sigmoid), _flat("X", "Y"))
silu_kernel = XbKernel("silu_kernel", "xb_silu", _unary(ops.silu), _flat("X", "Y"))
swiglu_kernel = XbKernel("swiglu_kernel", "xb_swiglu", _swiglu, _flat("GATE", "UP", "OUT"))


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


def _unit_cols(b, name):
    if b[name] != 1:
        raise ValueError("unit column stride")
    return 1


def _rows(block, pitch, span):
    # one unit per row; a piece is a whole number of the kernel's row blocks,
    # launched over that many programs
    return Split(units=lambda b, g: g[0] * b[block], pitch=pitch, span=span,
                 piece=lambda b, g, n: ({}, (n // b[block], g[1], g[2])), align=lambda b: b[block])


_POOL2D = Split(units=lambda b, g: b["planes"],
                pitch=lambda b: {"X": b["H"] * b["W"], "Y": (b["H"] // 2) * (b["W"] // 2)},
                span=lambda b: (b["H"] // 2) * (b["W"] // 2), piece=lambda b, g, n: ({"planes": n}, (n, 1, 1)))
_STRIDED_ROWS = dict(
    pitch=lambda b: {"input_ptr": b["input_stride_row"] * _unit_cols(b, "input_stride_col"),
                     "output_ptr": b["output_stride_row"] * _unit_cols(b, "output_stride_col")},
    span=lambda b: b["n_cols"])

avg_pool_kernel = XbKernel("avg_pool_kernel", "xb_row_center", _avg_pool,
                           _rows("BLOCK_M", lambda b: {"X": b["N"], "Y": b["N"]}, lambda b: b["BLOCK_N"]))
# The 2-D (NCHW, 2x2 / stride 2) pooling form has no reference kernel; this
# launcher gives it the same calling convention as the others.
avg_pool2d_kernel = XbKernel("avg_pool2d_kernel", "xb_avg_pool2d_2x2", _avg_pool2d, _POOL2D)
softmax_kernel = XbKernel("softmax_kernel", "xb_softmax", _softmax, _rows("BLOCK_SIZE", **_STRIDED_ROWS))
_layer_norm_fwd_fused = XbKernel("_layer_norm_fwd_fused", "xb_layernorm", _layernorm,
                                 _rows("BLOCK_SIZE", **_STRIDED_ROWS))
rms_norm_kernel = XbKernel("rms_norm_kernel", "xb_rms_norm", _rms,
                           _rows("BLOCK_M", lambda b: {"X": b["N"], "Y": b["N"]}, lambda b: b["BLOCK_N"]))
# the weight vector is read whole by every piece
weighted_rms_norm_kernel = XbKernel("weighted_rms_norm_kernel", "xb_rms_norm", _wrms,
                                    _rows("BLOCK_M", lambda b: {"X": b["N"], "Y": b["N"]}, lambda b: b["BLOCK_N"]))


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

    def __init__(self, name, entry, run, defaults, split=None):
        super().__init__(name, entry, run, split)
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


# rows of A and C divide into pieces of whole 128-row tiles; B is read whole
# by every piece
_GEMM_ROWS = Split(units=lambda b, g: b["M"],
                   pitch=lambda b: {"A": b["stride_am"] * _unit_cols(b, "stride_ak"),
                                    "C": b["stride_cm"] * _unit_cols(b, "stride_cn")},
                   span=lambda b: b["N"], piece=lambda b, g, n: ({"M": n}, g), align=lambda b: 128)

bare_matmul_i8 = XbKernel("bare_matmul_i8", "xb_matmul_i8", _matmul, _GEMM_ROWS)
padded_matmul_kernel = XbKernel("padded_matmul_kernel", "xb_matmul_f32_bf16emu", _padded_matmul)
load_2d_block_kernel = XbKernel("kernel", "xb_mul_2d", _load_2d)
bare_matmul = XbKernel("bare_matmul", "xb_matmul_bf16", _matmul, _GEMM_ROWS)
bare_matmul_autotuned = _Autotuned("bare_matmul", "xb_matmul_bf16", _matmul, {"BLOCK_SIZE_M": 256}, _GEMM_ROWS)


REGISTRY = {
    k.name: k
    for k in (vecadd, axpy_kernel, relu_kernel, leaky_relu_kernel, gelu_kernel, gelu_kernel_gpu, sigmoid_kernel,
              silu_kernel, swiglu_kernel, avg_pool_kernel, avg_pool2d_kernel, softmax_kernel, _layer_norm_fwd_fused,
              rms_norm_kernel, weighted_rms_norm_kernel, bare_matmul_i8, bare_matmul, padded_matmul_kernel)
}
REGISTRY["load_2d_block_kernel"] = load_2d_block_kernel  # the example names its kernel plain `kernel`

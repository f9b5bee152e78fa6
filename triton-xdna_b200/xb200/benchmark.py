"""Stand-in for the reference's examples/benchmark.py.

The reference selects its backend with ``select_npu_backend()``
(examples/benchmark.py:12-13, ``triton.runtime.driver.set_active(NPUDriver())``)
and times calls with the ``measure`` decorator (examples/benchmark.py:26-89).
xb200 has one backend -- the CUDA library -- so selecting it means loading the
library and making sure a CUDA device is present; it never falls back.
"""

from __future__ import annotations

import time
from functools import wraps

import numpy as np
import torch

from . import _lib


def select_b200_backend(device: int | None = None) -> str:
    """Load libxb200.so and make ``device`` current; returns the device name."""
    _lib.load()
    if not torch.cuda.is_available():
        raise RuntimeError("select_b200_backend: no CUDA device (xb200 has no CPU fallback)")
    if device is not None:
        torch.cuda.set_device(device)
    from .ops import device_name

    return device_name(torch.cuda.current_device())[0]


# The reference's examples call this name; keep it as an alias so a script
# only has to change its import.
select_npu_backend = select_b200_backend


def select_cpu_backend():
    """The reference switches a process between its NPU driver and a CPU
    driver (examples/multi_drivers/matmul.py:88-92, triton-cpu compiling the
    same kernel for the host).  xb200 has no host execution path by design --
    its operators run only as sm_100a kernels -- so selecting a CPU driver is
    an error rather than a silent fallback."""
    raise NotImplementedError("xb200 runs its operators on the GPU only; there is no CPU driver to select")


def measure(repeats: int = 20, percentiles=(), timers=None):
    """Decorator timing a function (same output format as examples/benchmark.py:26-89).

    The default timers are wall clock and "GPU" wall clock around a device
    synchronisation, since launches are asynchronous here."""

    def _gpu_clock():
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        return time.perf_counter()

    timers = timers or {"Wall": time.perf_counter, "GPU": _gpu_clock}

    def decorator(func):
        @wraps(func)
        def wrapper(*args, **kwargs):
            print(f"{func.__name__}{args} {kwargs}, {repeats} times, all results in seconds")
            times = {t: [] for t in timers}
            result = None
            for _ in range(repeats):
                starts = {t: f() for t, f in timers.items()}
                result = func(*args, **kwargs)
                for t, f in timers.items():
                    times[t].append(f() - starts[t])
            for t in timers:
                arr = np.asarray(times[t])
                print(f"{t}: Avg={arr.mean():.6f}, min={arr.min():.6f}, std={arr.std():.6f},", end=" ")
                for p, v in zip(percentiles, np.percentile(arr, percentiles) if percentiles else []):
                    print(f"{p}pp={v:.6f},", end=" ")
                print(f"max={arr.max():.6f}")
            return result

        return wrapper

    return decorator

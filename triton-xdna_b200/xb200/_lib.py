"""ctypes binding of ``libxb200.so``.

The argument types of every entry point are read from the C header
(``include/xb200.h``), so the header is the single source of truth for the
ABI.  Errors follow the reference's native runtime convention
(amd_triton_npu/backend/include/HsaRuntime/HsaRuntime.cpp:740-794): a negative
status plus a message in the caller's buffer, raised here as ``XbError``
(a ``RuntimeError``, which is what the reference's launcher raises,
amd_triton_npu/backend/driver.py:1553-1556).

There is deliberately no fallback: if the library is missing, every call
raises.
"""

from __future__ import annotations

import ctypes
import os
import re
import threading

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libxb200.so")
HEADER_CANDIDATES = [
    os.path.join(os.path.dirname(os.path.dirname(PKG_DIR)), "include", "xb200.h"),
    os.path.join(PKG_DIR, "xb200.h"),
]

XB_OK = 0
XB_ERR_INVALID = -1
XB_ERR_CUDA = -2
XB_ERR_UNSUPPORTED = -3
XB_ERR_TIMEOUT = -4

XB_DT_BF16, XB_DT_F32, XB_DT_I8, XB_DT_I16, XB_DT_I32 = 0, 1, 2, 3, 4

_ERR_NAMES = {
    XB_ERR_INVALID: "XB_ERR_INVALID",
    XB_ERR_CUDA: "XB_ERR_CUDA",
    XB_ERR_UNSUPPORTED: "XB_ERR_UNSUPPORTED",
    XB_ERR_TIMEOUT: "XB_ERR_TIMEOUT",
}

_CTYPES = {
    "void*": ctypes.c_void_p,
    "const void*": ctypes.c_void_p,
    "void* const*": ctypes.c_void_p,
    "void**": ctypes.POINTER(ctypes.c_void_p),
    "const uint64_t*": ctypes.c_void_p,
    "uint64_t*": ctypes.POINTER(ctypes.c_uint64),  # host out-parameter (xb_launch_count)
    "int": ctypes.c_int,
    # host out-parameters (passed with ctypes.byref)
    "int*": ctypes.POINTER(ctypes.c_int),
    "int64_t": ctypes.c_int64,
    # device pointers travel as plain addresses
    "int64_t*": ctypes.c_void_p,
    "const int64_t*": ctypes.c_void_p,
    "float*": ctypes.c_void_p,
    "const float*": ctypes.c_void_p,
    "size_t": ctypes.c_size_t,
    "size_t*": ctypes.POINTER(ctypes.c_size_t),
    "float": ctypes.c_float,
    "char*": ctypes.c_char_p,
    "const char*": ctypes.c_char_p,
    "uint64_t": ctypes.c_uint64,
    "uint32_t": ctypes.c_uint32,
    # an array of DecodePhase (ops.py), passed by address
    "const xb_decode_phase*": ctypes.c_void_p,
}


class XbError(RuntimeError):
    """A C-ABI call returned a negative status."""

    def __init__(self, func: str, code: int, message: str):
        self.func = func
        self.code = code
        self.message = message
        super().__init__(f"{func} failed ({_ERR_NAMES.get(code, code)}): {message}")


def header_path() -> str:
    for p in HEADER_CANDIDATES:
        if os.path.exists(p):
            return p
    raise RuntimeError("xb200.h not found next to the package; the C-ABI signatures are unknown")


def parse_header(path: str | None = None) -> dict[str, tuple[str, list[str]]]:
    """Return {name: (return_type, [param C types])} for every XB_API function."""
    text = open(path or header_path()).read()
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    text = re.sub(r"//[^\n]*", " ", text)
    out: dict[str, tuple[str, list[str]]] = {}
    for m in re.finditer(r"XB_API\s+(\w+)\s+(xb_\w+)\s*\(([^)]*)\)\s*;", text, flags=re.S):
        ret, name, params = m.group(1), m.group(2), m.group(3)
        types: list[str] = []
        params = " ".join(params.split())
        if params and params != "void":
            for p in params.split(","):
                p = p.strip()
                pm = re.match(r"(.*?)(\w+)$", p)
                ctype = pm.group(1).strip() if pm else p
                ctype = re.sub(r"\s*\*\s*", "*", ctype)
                ctype = ctype.replace("*const*", "* const*")
                types.append(ctype)
        out[name] = (ret, types)
    return out


_lock = threading.Lock()
_lib = None
_sigs: dict[str, tuple[str, list[str]]] = {}


def load() -> ctypes.CDLL:
    """Load the library (once) and declare every header function on it."""
    global _lib, _sigs
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                "(xb200 has no CPU fallback)"
            )
        lib = ctypes.CDLL(LIB_PATH)
        sigs = parse_header()
        for name, (ret, params) in sigs.items():
            fn = getattr(lib, name)  # AttributeError here = header/library mismatch
            fn.restype = ctypes.c_int if ret == "int" else None
            fn.argtypes = [_CTYPES[t] for t in params]
        _sigs = sigs
        _lib = lib
        return lib


def signatures() -> dict[str, tuple[str, list[str]]]:
    load()
    return dict(_sigs)


def call(name: str, *args) -> None:
    """Call ``name(*args, err, errlen)`` and raise XbError on a negative status."""
    lib = load()
    err = ctypes.create_string_buffer(1024)
    rc = getattr(lib, name)(*args, err, ctypes.sizeof(err))
    if rc != XB_OK:
        raise XbError(name, rc, err.value.decode(errors="replace"))


def call_int(name: str, *args) -> int:
    """Call an entry point that returns a plain int (no error buffer)."""
    return getattr(load(), name)(*args)

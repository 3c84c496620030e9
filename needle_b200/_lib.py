"""Loader for the C-ABI library ``libneedle_b200.so``.

The ctypes signatures are derived from ``include/needle_b200.h`` itself, so
the Python binding and the header cannot drift apart.  Loading never falls
back to anything: if the library is missing or cannot be loaded, every op
raises.  ``declared_functions()`` works without a GPU (it only parses the
header), and so does loading the library: the CUDA runtime inside it is
initialised on the first call that needs a device.
"""
from __future__ import annotations

import ctypes
import os
import re
from typing import Dict, List, Tuple

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
HEADER = os.path.join(ROOT, "include", "needle_b200.h")
LIB_PATH = os.path.join(PKG, "_lib", "libneedle_b200.so")

NB_OK = 0
NB_ERR_INVALID_ARG = 1
NB_ERR_UNSUPPORTED = 2
NB_ERR_CUDA = 3

NB_DTYPE_F32 = 0
NB_DTYPE_F16 = 1
NB_DTYPE_BF16 = 2


class NeedleB200Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"needle_b200 error {code}: {msg}")
        self.code = code


_CTYPES = {
    "void": None,
    "int": ctypes.c_int,
    "unsigned": ctypes.c_uint,
    "float": ctypes.c_float,
    "int64_t": ctypes.c_int64,
    "size_t": ctypes.c_size_t,
    "uint64_t": ctypes.c_uint64,
    "const char*": ctypes.c_char_p,
    "int*": ctypes.POINTER(ctypes.c_int),
    "unsigned*": ctypes.POINTER(ctypes.c_uint),
}


def _ctype(decl: str):
    decl = " ".join(decl.split())
    if decl.endswith("*") and decl.replace(" ", "") not in ("constchar*", "int*", "unsigned*"):
        return ctypes.c_void_p  # device / host pointers of any element type
    base = decl.replace("const char *", "const char*")
    return _CTYPES[base]


def declared_functions(header: str = HEADER) -> Dict[str, Tuple[str, List[Tuple[str, str]]]]:
    """``{name: (return type, [(arg type, arg name), ...])}`` for every
    ``NB_API`` function declared in the header."""
    with open(header) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    out = {}
    for m in re.finditer(r"NB_API\s+([\w\s\*]+?)\s*\b(nb_\w+)\s*\(([^)]*)\)\s*;", text):
        ret, name, args = m.group(1).strip(), m.group(2), m.group(3).strip()
        params = []
        if args and args != "void":
            for a in args.split(","):
                a = " ".join(a.split())
                am = re.match(r"(.*?)(\w+)$", a)
                typ, pname = am.group(1).strip(), am.group(2)
                typ = typ.replace(" *", "*")
                params.append((typ, pname))
        out[name] = (ret.replace(" *", "*"), params)
    return out


_lib = None


def lib():
    """The loaded library (loaded once, with signatures from the header)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise NeedleB200Error(NB_ERR_CUDA, f"{LIB_PATH} is missing; run `python -m needle_b200.build`")
    L = ctypes.CDLL(LIB_PATH)
    for name, (ret, params) in declared_functions().items():
        fn = getattr(L, name)
        fn.restype = _ctype(ret) if ret != "void" else None
        fn.argtypes = [_ctype(t) for t, _ in params]
    _lib = L
    return L


def check(rc: int) -> None:
    if rc != NB_OK:
        msg = lib().nb_last_error().decode(errors="replace")
        raise NeedleB200Error(rc, msg)


def device_errors() -> int:
    """Synchronise and return (and clear) the device error word."""
    v = ctypes.c_uint(0)
    check(lib().nb_device_errors(ctypes.byref(v)))
    return int(v.value)

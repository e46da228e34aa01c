"""ctypes binding of the C ABI declared in include/dispatcher_b200.h.

The argument types are derived from the header itself, so the binding cannot
drift from the declarations.  Loading never needs a GPU (the library links
the CUDA runtime statically and touches the driver only on the first call);
calling an op without a CUDA device raises, there is no CPU fallback.
"""

import ctypes
import os
import re
import threading

from . import build as _build

HEADER = os.path.join(_build.INCLUDE, "dispatcher_b200.h")
ERRORS = {0: "DH_OK", 1: "DH_ERR_SHAPE", 2: "DH_ERR_ARG", 3: "DH_ERR_CUDA",
          4: "DH_ERR_TIMEOUT", 5: "DH_ERR_DEVICE"}

_lock = threading.Lock()
_lib = None


class DispatcherB200Error(RuntimeError):
    """A C-ABI entry point returned a nonzero status."""

    def __init__(self, fn, code, msg):
        super().__init__(f"{fn} failed with {ERRORS.get(code, code)}: {msg}")
        self.code = code


def _ctype(decl):
    decl = decl.strip()
    if "*" in decl:
        return ctypes.c_void_p
    base = decl.rsplit(None, 1)[0] if len(decl.split()) > 1 else decl
    base = base.replace("const", "").strip()
    return {"int": ctypes.c_int, "float": ctypes.c_float, "int64_t": ctypes.c_int64,
            "uint32_t": ctypes.c_uint32, "size_t": ctypes.c_size_t,
            "long long": ctypes.c_longlong, "unsigned long long": ctypes.c_ulonglong}[base]


def parse_header(path=HEADER):
    """{name: (restype, [argtypes])} for every DH_API function in the header."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    out = {}
    for m in re.finditer(r"DH_API\s+([\w\s\*]+?)\b(dh_\w+)\s*\(([^)]*)\)\s*;", text):
        ret, name, args = m.group(1).strip(), m.group(2), m.group(3).strip()
        restype = ctypes.c_char_p if "char" in ret else ctypes.c_int
        argtypes = [] if args in ("", "void") else [_ctype(a) for a in args.split(",")]
        out[name] = (restype, argtypes)
    return out


def lib_path():
    return _build.LIB_PATH


def load(build_if_missing=False):
    """Load (once) and return the library with typed entry points."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if not os.path.exists(path):
            if build_if_missing:
                _build.build()
            else:
                raise RuntimeError(
                    f"dispatcher_b200 CUDA library not built ({path} missing); run "
                    f"`python -m dispatcher_b200.build` or __graft_entry__.build()")
        lib = ctypes.CDLL(path)
        for name, (restype, argtypes) in parse_header().items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
        return lib


def call(name, *args):
    """Invoke entry point `name`; raise DispatcherB200Error on nonzero status."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        raise DispatcherB200Error(name, rc, lib.dh_last_error().decode())
    return rc

"""ctypes binding of libdh_b200.so.

Function signatures are read from ``include/dh_b200.h`` (the C ABI), so every
declared entry point is bound with matching argument types.  There is no
fallback: if the shared library is missing or cannot be loaded, every call
raises :class:`DHLibraryError`.
"""

from __future__ import annotations

import ctypes
import re
from functools import lru_cache
from pathlib import Path
from typing import Any, Dict, List, Tuple

PKG = Path(__file__).resolve().parent
HEADER = PKG.parent / "include" / "dh_b200.h"
LIB_PATH = PKG / "lib" / "libdh_b200.so"

STATUS_NAMES = {
    0: "DH_OK",
    100: "DH_ERR_NULL_POINTER",
    101: "DH_ERR_ALIGNMENT",
    102: "DH_ERR_WORKSPACE",
    103: "DH_ERR_UNSUPPORTED_SHAPE",
    104: "DH_ERR_CUDA",
    105: "DH_ERR_INVALID_ARGUMENT",
    106: "DH_ERR_SCRATCH_LIMIT",
    107: "DH_ERR_NCCL",
}


class LinearWeights(ctypes.Structure):
    """dh_linear_weights of include/dh_b200.h (device pointers)."""

    _fields_ = [("weight", ctypes.c_void_p), ("w_scale", ctypes.c_void_p), ("bias", ctypes.c_void_p),
                ("smooth", ctypes.c_void_p), ("inv_smooth", ctypes.c_void_p)]


class MDLMWeights(ctypes.Structure):
    """dh_mdlm_weights of include/dh_b200.h; block_linears points to a host
    array of 4 LinearWeights per block (qkv, out, up, down)."""

    _fields_ = [("blocks", ctypes.c_uint32), ("vocabulary_size", ctypes.c_uint32),
                ("mask_token_id", ctypes.c_uint32), ("max_positions", ctypes.c_uint32),
                ("embedding", ctypes.c_void_p), ("rope_cos", ctypes.c_void_p), ("rope_sin", ctypes.c_void_p),
                ("block_linears", ctypes.POINTER(LinearWeights)), ("head", LinearWeights),
                ("head_rows", ctypes.c_uint32), ("head_vocab_offset", ctypes.c_uint32)]


class DHLibraryError(RuntimeError):
    """The native library is missing or failed to load."""


class DHDeviceError(RuntimeError):
    """A bounded wait inside a kernel gave up (the pipeline barrier it waited
    on never completed): that kernel abandoned its work, so the outputs of the
    work enqueued since the last check are undefined.  The CUDA context stays
    usable."""

    def __init__(self, code: int) -> None:
        self.code = code
        super().__init__(f"a bounded device wait expired (device error word {code})")


class DHStatusError(RuntimeError):
    """An entry point returned a non-zero status."""

    def __init__(self, function: str, status: int) -> None:
        self.function = function
        self.status = status
        super().__init__(f"{function} returned status {status} ({STATUS_NAMES.get(status, 'family code')})")


_CTYPES = {
    "uint32_t": ctypes.c_uint32,
    "int32_t": ctypes.c_int32,
    "uint64_t": ctypes.c_uint64,
    "int64_t": ctypes.c_int64,
    "size_t": ctypes.c_size_t,
    "int": ctypes.c_int,
    "float": ctypes.c_float,
    "double": ctypes.c_double,
    "void": None,
}


def _ctype(decl: str) -> Any:
    decl = decl.replace("const ", "").strip()
    if "*" in decl:
        return ctypes.c_void_p
    base = decl.split()[0]
    if base not in _CTYPES:
        raise ValueError(f"unsupported C type in dh_b200.h: {decl!r}")
    return _CTYPES[base]


def parse_header(path: Path = HEADER) -> Dict[str, Tuple[Any, List[Any]]]:
    """Return {name: (restype, [argtypes])} for every dh_* prototype."""
    text = path.read_text()
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    text = re.sub(r"//[^\n]*", " ", text)
    out: Dict[str, Tuple[Any, List[Any]]] = {}
    for match in re.finditer(r"\b(uint32_t|uint64_t|size_t|void|int32_t|int)\s+(dh_\w+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S):
        restype, name, args = match.group(1), match.group(2), match.group(3)
        argtypes = []
        args = " ".join(args.split())
        if args and args != "void":
            for arg in args.split(","):
                arg = arg.strip()
                # drop the parameter name (last identifier), keep pointer stars
                type_part = re.sub(r"\b\w+$", "", arg).strip() if not arg.endswith("*") else arg
                argtypes.append(_ctype(type_part))
        out[name] = (_CTYPES[restype], argtypes)
    return out


@lru_cache(maxsize=1)
def lib() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise DHLibraryError(
            f"{LIB_PATH} is missing; build it with `python -m diffusionhard_b200.build`")
    try:
        handle = ctypes.CDLL(str(LIB_PATH))
    except OSError as exc:  # pragma: no cover - depends on the host
        raise DHLibraryError(f"cannot load {LIB_PATH}: {exc}") from exc
    for name, (restype, argtypes) in parse_header().items():
        fn = getattr(handle, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return handle


def call(name: str, *args: Any) -> int:
    """Call an entry point and raise DHStatusError on a non-zero status."""
    status = getattr(lib(), name)(*args)
    if status != 0:
        raise DHStatusError(name, int(status))
    return 0


def raw(name: str, *args: Any) -> int:
    """Call an entry point and return its raw status."""
    return int(getattr(lib(), name)(*args))


def check_device_error() -> None:
    """Read and clear the device error word (synchronous); raise
    DHDeviceError if a kernel's bounded wait expired since the last check."""
    word = ctypes.c_uint32(0)
    call("dh_device_error", ctypes.addressof(word), 1)
    if word.value:
        raise DHDeviceError(int(word.value))


def ptr(tensor: Any) -> int | None:
    """Device pointer of a torch tensor (None for None)."""
    if tensor is None:
        return None
    return int(tensor.data_ptr())


def stream_handle(stream: Any = None) -> int | None:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream) or None

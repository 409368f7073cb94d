"""ctypes binding of libkg_sm100.so (include/kg_sm100.h).

The library is built in-tree (``python -m kernelcode_generate_b200._build`` or
``__graft_entry__.build()``). There is no fallback: if the library is missing, every call
raises ``KernelBackendUnavailable``.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_DIR = PKG_DIR / "lib"
LIB_PATH = LIB_DIR / "libkg_sm100.so"
SHIM_PATHS = {
    "matmul": LIB_DIR / "libkg_sm100_matmul.so",
    "conv2d": LIB_DIR / "libkg_sm100_conv2d.so",
    "flash_attention": LIB_DIR / "libkg_sm100_flash_attention.so",
}

KG_SLOT_MEMORY, KG_SLOT_INT, KG_SLOT_FLOAT = 1, 2, 3
KG_DTYPE_F32, KG_DTYPE_F64, KG_DTYPE_I32, KG_DTYPE_I64, KG_DTYPE_BF16 = 1, 2, 3, 4, 5
KG_OK, KG_ERR_INVALID_ARGUMENT, KG_ERR_UNSUPPORTED, KG_ERR_CUDA, KG_ERR_DEVICE_TIMEOUT = 0, 1, 2, 3, 4

EXPORTED_SYMBOLS = (
    "kg_sm100_matmul_entry",
    "kg_sm100_conv2d_entry",
    "kg_sm100_flash_attention_entry",
    "kg_sm100_matmul_capture",
    "kg_sm100_conv2d_capture",
    "kg_sm100_flash_attention_capture",
    "kg_sm100_matmul",
    "kg_sm100_conv2d",
    "kg_sm100_flash_attention",
    "kg_sm100_flash_attention_ex",
    "kg_sm100_device_status",
    "kg_sm100_last_error",
    "kg_sm100_last_kernel",
    "kg_sm100_abi_version",
)


class KernelBackendUnavailable(RuntimeError):
    """The sm_100a library is not built (or cannot be loaded)."""


class KernelError(RuntimeError):
    """A library call returned a non-zero status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"kg_sm100 error {code}: {message}")
        self.code = code


class KgArgSlot(ctypes.Structure):
    """C layout of one entry argument (include/kg_sm100.h KgArgSlot; reference _CArgSlot,
    kernel_gen/execute_engine/runtime_args.py:217-237)."""

    _fields_ = [
        ("kind", ctypes.c_int),
        ("data", ctypes.c_void_p),
        ("shape", ctypes.POINTER(ctypes.c_longlong)),
        ("stride", ctypes.POINTER(ctypes.c_longlong)),
        ("rank", ctypes.c_ulonglong),
        ("dtype_code", ctypes.c_int),
        ("int_value", ctypes.c_longlong),
        ("float_value", ctypes.c_double),
    ]


_LIB: ctypes.CDLL | None = None

_LL = ctypes.c_longlong
_VP = ctypes.c_void_p


def load() -> ctypes.CDLL:
    """Load libkg_sm100.so once and declare its prototypes."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise KernelBackendUnavailable(
            f"{LIB_PATH} is not built; run `python -m kernelcode_generate_b200._build` (nvcc, sm_100a)")
    try:
        lib = ctypes.CDLL(str(LIB_PATH))
    except OSError as exc:
        raise KernelBackendUnavailable(f"cannot load {LIB_PATH}: {exc}") from exc
    slot_p = ctypes.POINTER(KgArgSlot)
    for name in ("kg_sm100_matmul_entry", "kg_sm100_conv2d_entry", "kg_sm100_flash_attention_entry"):
        f = getattr(lib, name)
        f.argtypes = [slot_p, ctypes.c_ulonglong]
        f.restype = ctypes.c_int
    lib.kg_sm100_matmul.argtypes = [_VP, _VP, _VP, ctypes.c_int, _VP, _LL, _LL, _LL, _VP]
    lib.kg_sm100_matmul.restype = ctypes.c_int
    lib.kg_sm100_conv2d.argtypes = [_VP, _VP, _VP, ctypes.c_int, _VP] + [_LL] * 15 + [_VP]
    lib.kg_sm100_conv2d.restype = ctypes.c_int
    lib.kg_sm100_flash_attention.argtypes = [_VP, _VP, _VP, _VP, ctypes.c_int, _LL, _LL, _LL, _LL, ctypes.c_float, ctypes.c_int, _VP]
    lib.kg_sm100_flash_attention.restype = ctypes.c_int
    lib.kg_sm100_flash_attention_ex.argtypes = [_VP, ctypes.c_int, _VP, _VP, _VP, ctypes.c_int, _LL, _LL, _LL, _LL, ctypes.c_float,
                                                ctypes.c_int, _VP]
    lib.kg_sm100_flash_attention_ex.restype = ctypes.c_int
    lib.kg_sm100_device_status.argtypes = [ctypes.POINTER(ctypes.c_int)]
    lib.kg_sm100_device_status.restype = ctypes.c_int
    lib.kg_sm100_last_error.argtypes = []
    lib.kg_sm100_last_error.restype = ctypes.c_char_p
    lib.kg_sm100_last_kernel.argtypes = []
    lib.kg_sm100_last_kernel.restype = ctypes.c_char_p
    lib.kg_sm100_abi_version.argtypes = []
    lib.kg_sm100_abi_version.restype = ctypes.c_int
    _LIB = lib
    return lib


def last_error() -> str:
    return (load().kg_sm100_last_error() or b"").decode()


def last_kernel() -> str:
    return (load().kg_sm100_last_kernel() or b"").decode()


def check(code: int) -> None:
    if code != KG_OK:
        raise KernelError(code, last_error())


def device_status() -> int:
    """Synchronise the current device and return (and clear) its kernel status word."""
    code = ctypes.c_int(0)
    check(load().kg_sm100_device_status(ctypes.byref(code)))
    return code.value

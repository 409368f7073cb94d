"""TEST INFRASTRUCTURE ONLY: ctypes access to the CPU oracle.

Two libraries live under ``oracle/``:

* ``_build/libkg_oracle.so`` -- the C restatement (``kg_oracle.c``) of the reference's three
  tiled kernels. It is the checker the parity tests use, and ``bench.py`` times it as the
  ``"port"`` CPU baseline when the reference build below is absent.
* ``_ref/libkg_ref_O0.so`` / ``_ref/libkg_ref_O2.so`` -- ``ref_harness.cpp`` compiled against
  the reference's own ``include/npu_demo`` helpers (only buildable where the reference tree
  is mounted; the built files travel with the repository snapshot).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (CPU baseline and reference
arm) import this module. The product package never does.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
PORT_LIB = ORACLE_DIR / "_build" / "libkg_oracle.so"
REF_LIB_O0 = ORACLE_DIR / "_ref" / "libkg_ref_O0.so"
REF_LIB_O2 = ORACLE_DIR / "_ref" / "libkg_ref_O2.so"


def reference_root() -> Path | None:
    """The reference checkout (violetDelia/kernelcode_generate) whose npu_demo headers the harness
    compiles against: $KG_REFERENCE_ROOT when set, else a checkout named ``reference`` beside this
    repository. None when neither holds the reference's ``include/npu_demo/npu_demo.h``."""
    env = os.environ.get("KG_REFERENCE_ROOT")
    for cand in ([Path(env)] if env else []) + [ORACLE_DIR.parent.parent / "reference"]:
        if (cand / "include" / "npu_demo" / "npu_demo.h").exists():
            return cand.resolve()
    return None

F32 = 1
BF16 = 5

_LL = ctypes.c_longlong
_VP = ctypes.c_void_p

_PORT = None
_REF: dict[str, ctypes.CDLL] = {}


def build_port() -> Path:
    """Compile kg_oracle.c with gcc (make port) if the library is missing or stale."""
    src = ORACLE_DIR / "kg_oracle.c"
    if not PORT_LIB.exists() or PORT_LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), "port"], check=True)
    return PORT_LIB


def build_ref(root: Path | None = None) -> bool:
    """Compile ref_harness.cpp against the reference's npu_demo headers, when the reference
    checkout is present (``root``, else ``reference_root()``); otherwise keep the libraries already
    built. Returns whether both libraries exist."""
    root = Path(root) if root is not None else reference_root()
    if root is None or not (root / "include" / "npu_demo" / "npu_demo.h").exists():
        return REF_LIB_O2.exists() and REF_LIB_O0.exists()
    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), "ref", f"REF_ROOT={root}"], check=True)
    return True


def _bind(lib: ctypes.CDLL, prefix: str) -> ctypes.CDLL:
    threads = [ctypes.c_int] if prefix == "kgr" else []
    f = getattr(lib, f"{prefix}_matmul")
    f.restype = ctypes.c_int
    f.argtypes = [_VP, _VP, _VP, ctypes.c_int, _VP] + [_LL] * 8 + threads
    f = getattr(lib, f"{prefix}_conv2d")
    f.restype = ctypes.c_int
    f.argtypes = [_VP, _VP, _VP, ctypes.c_int, _VP] + [_LL] * 20 + threads
    f = getattr(lib, f"{prefix}_flash_attention")
    f.restype = ctypes.c_int
    f.argtypes = [_VP, _VP, _VP, _VP, ctypes.c_int] + [_LL] * 6 + [ctypes.c_float, ctypes.c_int] + [_LL] * 4 + threads
    f = getattr(lib, f"{prefix}_tile_matmul")
    f.restype = ctypes.c_int
    f.argtypes = [_VP, _VP, _VP, _LL, _LL, _LL, ctypes.c_int]
    return lib


def port() -> ctypes.CDLL:
    global _PORT
    if _PORT is None:
        _PORT = _bind(ctypes.CDLL(str(build_port())), "kgo")
    return _PORT


def ref_available(opt: str = "O2") -> bool:
    return (REF_LIB_O2 if opt == "O2" else REF_LIB_O0).exists()


def ref(opt: str = "O2") -> ctypes.CDLL:
    if opt not in _REF:
        path = REF_LIB_O2 if opt == "O2" else REF_LIB_O0
        if not path.exists():
            raise FileNotFoundError(f"reference harness not built: {path}")
        _REF[opt] = _bind(ctypes.CDLL(str(path)), "kgr")
    return _REF[opt]


def _ptr(a: np.ndarray | None) -> int | None:
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def _dtype_code(a: np.ndarray) -> int:
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.uint16:  # raw bf16 bits
        return BF16
    raise TypeError(f"unsupported oracle dtype {a.dtype}")


def _lib(impl: str, opt: str) -> tuple[ctypes.CDLL, str]:
    return (port(), "kgo") if impl == "port" else (ref(opt), "kgr")


def matmul(lhs, rhs, bias=None, tiles=(64, 64, 64), rows=None, impl="port", threads=1, opt="O2", out=None):
    """out[H,W] = lhs[H,K] @ rhs[K,W] (+bias) through the tiled loop nest. `rows` limits the
    computed rows (a (begin, end) range); rows outside stay as in `out` (zeros by default).
    bf16 inputs are passed as uint16 bit patterns."""
    H, K = lhs.shape
    W = rhs.shape[1]
    if out is None:
        out = np.zeros((H, W), dtype=np.float32)
    r0, r1 = rows if rows is not None else (0, H)
    lib, prefix = _lib(impl, opt)
    args = [_ptr(out), _ptr(lhs), _ptr(rhs), _dtype_code(lhs), _ptr(bias), H, K, W, *tiles, r0, r1]
    if prefix == "kgr":
        args.append(threads)
    rc = getattr(lib, f"{prefix}_matmul")(*args)
    if rc != 0:
        raise RuntimeError(f"oracle matmul failed rc={rc}")
    return out


def conv2d_out_shape(x_shape, w_shape, stride, dilation, pads):
    B, C, XH, XW = x_shape
    F, _, KH, KW = w_shape
    if min(stride) <= 0 or min(dilation) <= 0:
        raise RuntimeError("oracle conv2d: stride and dilation must be positive")
    HO = (XH + pads[0] + pads[1] - dilation[0] * (KH - 1) - 1) // stride[0] + 1
    WO = (XW + pads[2] + pads[3] - dilation[1] * (KW - 1) - 1) // stride[1] + 1
    return (B, F, HO, WO)


def conv2d(x, w, bias=None, stride=(1, 1), dilation=(1, 1), pads=(0, 0, 0, 0), tiles=(8, 16, 4, 8, 9),
           impl="port", threads=1, opt="O2"):
    """NCHW conv2d through the reference's tiled img2col loop nest; pads = (top, bottom, left, right)."""
    B, C, XH, XW = x.shape
    F, C2, KH, KW = w.shape
    assert C == C2
    out = np.zeros(conv2d_out_shape(x.shape, w.shape, stride, dilation, pads), dtype=np.float32)
    lib, prefix = _lib(impl, opt)
    args = [_ptr(out), _ptr(x), _ptr(w), _dtype_code(x), _ptr(bias), B, C, XH, XW, F, KH, KW,
            stride[0], stride[1], dilation[0], dilation[1], *pads, *tiles]
    if prefix == "kgr":
        args.append(threads)
    rc = getattr(lib, f"{prefix}_conv2d")(*args)
    if rc != 0:
        raise RuntimeError(f"oracle conv2d failed rc={rc}")
    return out


def flash_attention(q, k, v, tiles=(64, 64), scale=1.0, causal=False, bh=None, q_rows=None,
                    impl="port", threads=1, opt="O2", out=None):
    """softmax(q k^T * scale [causal]) v over [B,H,S,D] through the reference's online-softmax
    loop nest. `bh` / `q_rows` restrict the computed (b,h) pairs / query rows."""
    B, H, S, D = q.shape
    if out is None:
        out = np.zeros((B, H, S, D), dtype=np.float32)
    bh0, bh1 = bh if bh is not None else (0, B * H)
    q0, q1 = q_rows if q_rows is not None else (0, S)
    lib, prefix = _lib(impl, opt)
    args = [_ptr(out), _ptr(q), _ptr(k), _ptr(v), _dtype_code(q), B, H, S, D, tiles[0], tiles[1],
            float(scale), int(bool(causal)), bh0, bh1, q0, q1]
    if prefix == "kgr":
        args.append(threads)
    rc = getattr(lib, f"{prefix}_flash_attention")(*args)
    if rc != 0:
        raise RuntimeError(f"oracle flash_attention failed rc={rc}")
    return out


def tile_matmul(lhs, rhs, out=None, acc=False, impl="port", opt="O2"):
    m, k = lhs.shape
    n = rhs.shape[1]
    if out is None:
        out = np.zeros((m, n), dtype=np.float32)
    lib, prefix = _lib(impl, opt)
    rc = getattr(lib, f"{prefix}_tile_matmul")(_ptr(out), _ptr(lhs), _ptr(rhs), m, k, n, int(acc))
    if rc != 0:
        raise RuntimeError(f"oracle tile_matmul failed rc={rc}")
    return out


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16, returned as uint16 bit patterns."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + rounding) >> 16).astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)

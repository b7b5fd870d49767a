"""ctypes binding of ``libglm_b200.so`` (the C ABI declared in ``include/glm_b200.h``).

Every function here takes raw device pointers (integers) and sizes, calls
the library and raises :class:`GlmbError` on a non-zero status.  The
library must have been built (``python -c "import __graft_entry__ as g;
g.build()"`` or ``make -C gpu_algos_b200``); importing this module without
it raises immediately -- there is no host fallback.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libglm_b200.so")

GLMB_OK = 0
GLMB_ERR_INVALID_VALUE = 1001
GLMB_ERR_WORKSPACE = 1002
GLMB_ERR_UNSUPPORTED = 1003
GLMB_ERR_TOO_LARGE = 1004
GLMB_ERR_COLLECTIVE = 1005
GLMB_ERR_PEER_TIMEOUT = 1006

MG_PEER = 0
MG_NCCL = 1

PEER_HANDLE_BYTES = 64

GRAD_REGULARIZE = 0x1
GRAD_WRITE_YHAT = 0x2
GRAD_Y_ZERO = 0x4
GRAD_LOGISTIC = 0x8

#: the eleven element types of the reference mains, by C-ABI suffix
REFERENCE_SUFFIXES = ("f16", "f32", "f64", "i8", "i16", "i32", "i64", "u8", "u16", "u32", "u64")
#: every element type of predict / gradient / loss: the reference's eleven and bfloat16
SUFFIXES = REFERENCE_SUFFIXES + ("bf16",)
FLOATING = ("f32", "f64")
#: 16-bit types with the sharded entry points (partial, finalize, peer exchange) but no fit
HALF16 = ("f16", "bf16")


class GlmbError(RuntimeError):
    def __init__(self, status: int, where: str):
        self.status = int(status)
        super().__init__(f"{where}: status {status} ({status_string(status)})")


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_D = ctypes.c_double
_U32 = ctypes.c_uint32
_U64 = ctypes.c_uint64
_SZ = ctypes.c_size_t
_INT = ctypes.c_int

_lib: ctypes.CDLL | None = None


def _declare(L: ctypes.CDLL) -> None:
    L.glmb_version.restype = _INT
    L.glmb_status_string.restype = ctypes.c_char_p
    L.glmb_status_string.argtypes = [_INT]
    L.glmb_launch_count.restype = _U64
    L.glmb_last_path.restype = ctypes.c_char_p
    for s in SUFFIXES:
        f = getattr(L, f"glmb_predict_{s}")
        f.argtypes = [_P, _P, _P, _I64, _I64, _I64, _I64, _P]
        f.restype = _INT
        f = getattr(L, f"glmb_gradient_workspace_size_{s}")
        f.argtypes = [_I64, _I64, _I64, _I64]
        f.restype = _SZ
        f = getattr(L, f"glmb_gradient_{s}")
        f.argtypes = [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _D, _D, _U32, _P, _SZ, _P]
        f.restype = _INT
        f = getattr(L, f"glmb_loss_{s}")
        f.argtypes = [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _D, _D, _P, _SZ, _P]
        f.restype = _INT
    for s in FLOATING:
        sig = {
            "glmb_gradient_partial": [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _U32, _P, _SZ, _P],
            "glmb_gradient_finalize": [_P, _P, _P, _I64, _I64, _I64, _D, _D, _U32, _P],
            "glmb_prox_step": [_P, _P, _I64, _D, _D, _P],
            "glmb_prox_update": [_P, _P, _P, _I64, _I64, _I64, _D, _D, _P],
            "glmb_power_step": [_P, _P, _P, _P, _I64, _I64, _D, _P],
            "glmb_power_init": [_P, _I64, _I64, _U64, _P],
            "glmb_fit_elastic_net": [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _D, _D, _INT, _INT,
                                     _U64, _P, _SZ, _P],
            "glmb_gradient_loss": [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _D, _D, _U32, _P, _SZ, _P],
        }
        for name, args in sig.items():
            f = getattr(L, f"{name}_{s}")
            f.argtypes = args
            f.restype = _INT
        f = getattr(L, f"glmb_fit_workspace_size_{s}")
        f.argtypes = [_I64, _I64, _I64, _I64]
        f.restype = _SZ
    for s in HALF16:
        f = getattr(L, f"glmb_gradient_partial_{s}")
        f.argtypes = [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _U32, _P, _SZ, _P]
        f.restype = _INT
        f = getattr(L, f"glmb_gradient_finalize_{s}")
        f.argtypes = [_P, _P, _P, _I64, _I64, _I64, _D, _D, _U32, _P]
        f.restype = _INT
        f = getattr(L, f"glmb_gradient_sharded_{s}")
        f.argtypes = [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _D, _D, _U32, _P, _P, _SZ, _P]
        f.restype = _INT
    L.glmb_gradient_noalloc_f32.argtypes = [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _D, _D, _U32, _P]
    L.glmb_gradient_noalloc_f32.restype = _INT
    L.glmb_peer_group_create.argtypes = [_INT, _INT, _I64, _D, ctypes.POINTER(ctypes.c_void_p), _P]
    L.glmb_peer_group_connect.argtypes = [_P, _P]
    L.glmb_peer_group_connect_local.argtypes = [_P, ctypes.POINTER(ctypes.c_void_p)]
    L.glmb_peer_group_buffer.argtypes = [_P]
    L.glmb_peer_group_buffer.restype = _P
    L.glmb_peer_group_status.argtypes = [_P, ctypes.POINTER(ctypes.c_int), _INT]
    L.glmb_peer_group_destroy.argtypes = [_P]
    for name in ("glmb_peer_group_create", "glmb_peer_group_connect", "glmb_peer_group_connect_local",
                 "glmb_peer_group_status", "glmb_peer_group_destroy"):
        getattr(L, name).restype = _INT
    for s in FLOATING:
        f = getattr(L, f"glmb_gradient_sharded_{s}")
        f.argtypes = [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _D, _D, _U32, _P, _P, _SZ, _P]
        f.restype = _INT
        f = getattr(L, f"glmb_fit_elastic_net_sharded_{s}")
        f.argtypes = [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _D, _D, _INT, _INT, _U64, _P, _P, _SZ, _P]
        f.restype = _INT
        _PP = ctypes.POINTER(ctypes.c_void_p)
        f = getattr(L, f"glmb_mg_gradient_{s}")
        f.argtypes = [_P, _PP, _PP, _PP, _PP, ctypes.POINTER(_I64), _I64, _I64, _I64, _D, _D, _U32]
        f.restype = _INT
        f = getattr(L, f"glmb_mg_fit_elastic_net_{s}")
        f.argtypes = [_P, _PP, _PP, _PP, _PP, ctypes.POINTER(_I64), _I64, _I64, _I64, _D, _D, _INT, _INT, _U64]
        f.restype = _INT
    L.glmb_mg_create.argtypes = [_INT, ctypes.POINTER(_INT), _I64, _D, _U32, ctypes.POINTER(ctypes.c_void_p)]
    L.glmb_mg_destroy.argtypes = [_P]
    L.glmb_mg_size.argtypes = [_P]
    L.glmb_mg_stream.argtypes = [_P, _INT, ctypes.POINTER(ctypes.c_void_p)]
    L.glmb_mg_synchronize.argtypes = [_P]
    for name in ("glmb_mg_create", "glmb_mg_destroy", "glmb_mg_size", "glmb_mg_stream", "glmb_mg_synchronize"):
        getattr(L, name).restype = _INT


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `make -C gpu_algos_b200` "
                "(the GLM path has no host fallback)")
        _lib = ctypes.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


def status_string(status: int) -> str:
    return lib().glmb_status_string(int(status)).decode()


def check(status: int, where: str) -> None:
    if status != GLMB_OK:
        raise GlmbError(status, where)


def version() -> int:
    return int(lib().glmb_version())


def launch_count() -> int:
    return int(lib().glmb_launch_count())


def last_path() -> str:
    return lib().glmb_last_path().decode()


def call(name: str, *args) -> int:
    """Call ``name`` with ``args`` and raise on a non-zero status."""
    st = getattr(lib(), name)(*args)
    check(st, name)
    return st


def exported_symbols() -> list[str]:
    """Every entry point declared in include/glm_b200.h (for the load test)."""
    names = ["glmb_version", "glmb_status_string", "glmb_launch_count", "glmb_last_path"]
    for s in SUFFIXES:
        names += [f"glmb_predict_{s}", f"glmb_gradient_workspace_size_{s}", f"glmb_gradient_{s}",
                  f"glmb_loss_{s}"]
    for s in FLOATING:
        names += [f"glmb_gradient_partial_{s}", f"glmb_gradient_finalize_{s}", f"glmb_prox_step_{s}",
                  f"glmb_prox_update_{s}", f"glmb_power_step_{s}", f"glmb_power_init_{s}",
                  f"glmb_fit_workspace_size_{s}", f"glmb_fit_elastic_net_{s}", f"glmb_gradient_loss_{s}"]
    names.append("glmb_gradient_noalloc_f32")
    names += ["glmb_peer_group_create", "glmb_peer_group_connect", "glmb_peer_group_connect_local",
              "glmb_peer_group_buffer", "glmb_peer_group_status", "glmb_peer_group_destroy"]
    names += [f"glmb_gradient_sharded_{s}" for s in FLOATING]
    for s in HALF16:
        names += [f"glmb_gradient_partial_{s}", f"glmb_gradient_finalize_{s}", f"glmb_gradient_sharded_{s}"]
    names += [f"glmb_fit_elastic_net_sharded_{s}" for s in FLOATING]
    names += ["glmb_mg_create", "glmb_mg_destroy", "glmb_mg_size", "glmb_mg_stream", "glmb_mg_synchronize"]
    for s in FLOATING:
        names += [f"glmb_mg_gradient_{s}", f"glmb_mg_fit_elastic_net_{s}"]
    return names

"""ctypes binding of libpagedkv.so (the C ABI declared in include/pagedkv.h).

The library must have been built (pagedkv.build) before import; there is no
fallback implementation, so a missing or unloadable library raises
PagedKVUnavailable immediately.
"""

from __future__ import annotations

import ctypes
import os

from . import build as _build

F32, F16, BF16 = 0, 1, 2

OK = 0
ERR_NULL_POINTER = -1
ERR_BAD_SHAPE = -2
ERR_BAD_DTYPE = -3
ERR_WORKSPACE_TOO_SMALL = -4
ERR_MISALIGNED = -5
ERR_UNSUPPORTED = -6
ERR_DRIVER = -7
ERR_SCRATCH_LIMIT = -8

# device-resident scratch of pkv_paged_decode_attention_noalloc
NOALLOC_SCRATCH_BYTES = 8 << 20

# bytes of a CUDA IPC memory handle (pkv_ipc_export / pkv_ipc_open)
IPC_HANDLE_BYTES = 64

FLAG_SLOT_OUT_OF_RANGE = 1
FLAG_BLOCK_OUT_OF_RANGE = 2
FLAG_CONTEXT_EXCEEDS_TABLE = 4
FLAG_PIPELINE_TIMEOUT = 8
FLAG_BAD_QUERY_LAYOUT = 16
FLAG_POSITION_OUT_OF_RANGE = 32
FLAG_BAD_SCHEDULE = 64

DECODE_AUTO = 0
DECODE_GENERIC = 1

# flags of pkv_paged_decode_append_attention_layers_flags
LAYERS_DEFER_FIRST = 1

# every symbol include/pagedkv.h declares, with (restype, argtypes)
_P, _I, _I64, _F, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
SIGNATURES: dict = {
    "pkv_abi_version": (_I, []),
    "pkv_status_string": (ctypes.c_char_p, [_I]),
    "pkv_reshape_and_cache": (_I, [_P, _P, _I64, _I64, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P]),
    "pkv_copy_blocks": (_I, [_P, _P, _I64, _I, _P, _I, _I, _I64, _P, _P]),
    "pkv_rope_reshape_and_cache": (_I, [_P, _I64, _P, _I64, _P, _P, _P, _I, _P, _P, _P, _I, _I, _I,
                                        _I, _I, _I, _I, _P, _P]),
    "pkv_decode_workspace_bytes": (_SZ, [_I, _I, _I]),
    "pkv_paged_decode_attention": (_I, [_P, _I64, _P, _I64, _P, _P, _I, _P, _I64, _I, _P, _I, _I,
                                        _I, _I, _I, _F, _I, _P, _SZ, _P, _P]),
    "pkv_paged_prefill_attention": (_I, [_P, _I64, _P, _I64, _P, _P, _I, _P, _I64, _I, _P, _P, _I,
                                         _I, _I, _I, _I, _I, _I, _F, _I, _P, _P]),
    "pkv_set_decode_impl": (_I, [_I]),
    "pkv_paged_decode_append_attention": (_I, [_P, _I64, _P, _I64, _P, _P, _I64, _I64, _P, _P, _I, _P,
                                               _I64, _I, _P, _I, _I, _I, _I, _I, _F, _I, _P, _SZ,
                                               _P, _P]),
    "pkv_paged_decode_attention_noalloc": (_I, [_P, _I64, _P, _I64, _P, _P, _I, _P, _I64, _I, _P, _I,
                                                _I, _I, _I, _I, _F, _I, _P, _P]),
    "pkv_reshape_and_cache_fp8": (_I, [_P, _P, _I64, _I64, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I,
                                       _P, _P]),
    "pkv_paged_decode_attention_fp8": (_I, [_P, _I64, _P, _I64, _P, _P, _P, _P, _I, _P, _I64, _I, _P,
                                            _I, _I, _I, _I, _I, _F, _I, _P, _SZ, _P, _P]),
    "pkv_paged_prefill_attention_fp8": (_I, [_P, _I64, _P, _I64, _P, _P, _P, _P, _I, _P, _I64, _I, _P,
                                             _P, _I, _I, _I, _I, _I, _I, _I, _F, _I, _P, _P]),
    "pkv_rope_reshape_and_cache_fp8": (_I, [_P, _I64, _P, _I64, _P, _P, _P, _I, _P, _P, _P, _P, _P,
                                            _I, _I, _I, _I, _I, _I, _I, _P, _P]),
    "pkv_paged_decode_append_attention_fp8": (_I, [_P, _I64, _P, _I64, _P, _P, _I64, _I64, _P, _P, _P,
                                                   _P, _I, _P, _I64, _I, _P, _I, _I, _I, _I, _I, _F,
                                                   _I, _P, _SZ, _P, _P]),
    "pkv_prefill_fp8_scratch_bytes": (_SZ, [_I, _I, _I, _I]),
    "pkv_paged_prefill_attention_fp8_tc": (_I, [_P, _I64, _P, _I64, _P, _P, _P, _P, _I, _P, _I64, _I,
                                                _P, _P, _I, _I, _I, _I, _I, _I, _I, _F, _I, _P, _P]),
    "pkv_paged_prefill_attention_fp8_scratch": (_I, [_P, _I64, _P, _I64, _P, _P, _P, _P, _I, _P,
                                                     _I64, _I, _P, _P, _I, _I, _I, _I, _I, _I, _I,
                                                     _F, _I, _P, _SZ, _P, _P]),
    "pkv_decode_schedule_bytes": (_SZ, [_I, _I]),
    "pkv_decode_schedule": (_I, [_P, _SZ, _P, _I64, _I, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P]),
    "pkv_ipc_export": (_I, [_P, _P, ctypes.POINTER(ctypes.c_uint64)]),
    "pkv_ipc_open": (_I, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "pkv_ipc_close": (_I, [_P]),
    "pkv_copy_blocks_peer": (_I, [_P, _P, _I64, _I, _P, _P, _I64, _I, _I, _P, _I, _I64, _P, _P]),
    "pkv_paged_decode_append_attention_fp8_layers": (_I, [_I, _P, _I64, _I64, _P, _I64, _I64, _P, _P,
                                                          _I64, _I64, _I64, _P, _P, _I64, _P, _P, _I64,
                                                          _I, _P, _I64, _I, _P, _I, _I, _I, _I, _I,
                                                          _F, _I, _P, _SZ, _P, _P, _P]),
    "pkv_paged_decode_append_attention_layers": (_I, [_I, _P, _I64, _I64, _P, _I64, _I64, _P, _P,
                                                      _I64, _I64, _I64, _P, _P, _I64, _I, _P, _I64,
                                                      _I, _P, _I, _I, _I, _I, _I, _F, _I, _P, _SZ,
                                                      _P, _P, _P, _P]),
    "pkv_paged_decode_append_attention_layers_flags": (_I, [_I, _P, _I64, _I64, _P, _I64, _I64, _P,
                                                            _P, _I64, _I64, _I64, _P, _P, _I64, _I, _P,
                                                            _I64, _I, _P, _I, _I, _I, _I, _I, _F, _I,
                                                            _P, _SZ, _P, _P, _P, _P, _I]),
}


# decode entries with a per-step schedule: the same arguments plus the schedule
for _n in ("pkv_paged_decode_attention", "pkv_paged_decode_attention_fp8",
           "pkv_paged_decode_append_attention", "pkv_paged_decode_append_attention_fp8"):
    SIGNATURES[_n + "_scheduled"] = (_I, SIGNATURES[_n][1] + [_P])


class PagedKVUnavailable(RuntimeError):
    """libpagedkv.so is missing or cannot be loaded."""


class PagedKVError(RuntimeError):
    def __init__(self, status: int, where: str):
        self.status = status
        super().__init__(f"{where}: pagedkv status {status}: {status_string(status)}")


_lib: ctypes.CDLL | None = None


def lib_path() -> str:
    """The in-tree build, unless PAGEDKV_LIB names another build of the same ABI."""
    return os.environ.get("PAGEDKV_LIB") or _build.LIB


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not os.path.exists(path):
        raise PagedKVUnavailable(
            f"{path} is not built; run `python -m pagedkv.build` (nvcc, sm_100a) first")
    try:
        L = ctypes.CDLL(path)
    except OSError as e:  # pragma: no cover - depends on the machine
        raise PagedKVUnavailable(f"cannot load {path}: {e}") from e
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def status_string(status: int) -> str:
    return load().pkv_status_string(int(status)).decode()


def check(status: int, where: str) -> None:
    if status != OK:
        raise PagedKVError(status, where)

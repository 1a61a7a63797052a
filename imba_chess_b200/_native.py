"""ctypes binding of the C ABI declared in include/imba_b200.h.

The shared library is built in-tree (``python -m imba_chess_b200.build``) and
loaded from this package's directory.  There is no CPU fallback: importing
this module never fails, but every call that needs the library raises
``NativeLibraryError`` when it is missing.
"""

from __future__ import annotations

import ctypes
import os
import threading

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libimba_b200.so")

IMBA_OK = 0
IMBA_ERR_ARG = 1
IMBA_ERR_RANGE = 2
IMBA_ERR_OOM = 3
IMBA_ERR_TIMEOUT = 4
IMBA_ERR_CUDA = 5
IMBA_ERR_UNSUPPORTED = 6
STATUS_NAMES = {
    IMBA_OK: "IMBA_OK",
    IMBA_ERR_ARG: "IMBA_ERR_ARG",
    IMBA_ERR_RANGE: "IMBA_ERR_RANGE",
    IMBA_ERR_OOM: "IMBA_ERR_OOM",
    IMBA_ERR_TIMEOUT: "IMBA_ERR_TIMEOUT",
    IMBA_ERR_CUDA: "IMBA_ERR_CUDA",
    IMBA_ERR_UNSUPPORTED: "IMBA_ERR_UNSUPPORTED",
}

DTYPE_F32 = 0
DTYPE_BF16 = 1
# imba_model_desc.flags: SIMT test hooks of a bf16 handle (cross-checks only)
FLAG_SIMT_GEMM = 1
FLAG_SIMT_ATTN = 2
FLAG_SIMT_BOARD = 4
SIMT_FLAGS = {"gemm": FLAG_SIMT_GEMM, "attn": FLAG_SIMT_ATTN, "board": FLAG_SIMT_BOARD}
MAX_LAYERS = 32
PAGE_TOKENS = 16
NOALLOC_SCRATCH_BYTES = 8 << 20
CHUNK_ROWS = 64
BOARD_BLOCK_FLOATS = 64 + 64 + 192 * 64 + 64 * 64 + 64 + 64 + 128 * 64 + 128 + 64 * 128 + 64
BOARD_PARAM_FLOATS = 2 * BOARD_BLOCK_FLOATS + 128

EXPORTED_SYMBOLS = (
    "imba_version",
    "imba_abi_size",
    "imba_device_arch",
    "imba_model_create",
    "imba_model_destroy",
    "imba_step_workspace_bytes",
    "imba_step",
    "imba_step_noalloc",
    "imba_profile_event_count",
    "imba_step_profiled",
    "imba_kv_scatter",
    "imba_kv_gather",
    "imba_selftest_wait_timeout",
    "imba_kv_scatter_indexed",
)

_P = ctypes.c_void_p
_I32 = ctypes.c_int32


class NativeLibraryError(RuntimeError):
    """The CUDA extension is missing or failed; there is no fallback path."""


class ImbaError(RuntimeError):
    def __init__(self, code: int, what: str) -> None:
        super().__init__(f"{what} failed with {STATUS_NAMES.get(code, code)}")
        self.code = code


class ModelDesc(ctypes.Structure):
    _fields_ = [
        ("model_dim", _I32),
        ("num_layers", _I32),
        ("num_heads", _I32),
        ("attention_dim", _I32),
        ("linear_dim", _I32),
        ("vocab", _I32),
        ("max_pos", _I32),
        ("halfmove_vocab", _I32),
        ("fullmove_vocab", _I32),
        ("has_value_head", _I32),
        ("dtype", _I32),
        ("flags", _I32),
        ("piece_square", _P),
        ("board_params", _P),
        ("board_out_w", _P),
        ("board_out_b", _P),
        ("emb_seq", _P),
        ("emb_turn", _P),
        ("emb_castle", _P),
        ("emb_ep", _P),
        ("emb_halfmove", _P),
        ("emb_fullmove", _P),
        ("emb_prev_move", _P),
        ("emb_pos", _P),
        ("uvqk_w", _P * MAX_LAYERS),
        ("o_w", _P * MAX_LAYERS),
        ("o_b", _P * MAX_LAYERS),
        ("ps_w", _P * MAX_LAYERS),
        ("final_norm_w", _P),
        ("final_norm_b", _P),
        ("policy_w", _P),
        ("policy_w32", _P),
        ("value0_w", _P),
        ("value0_b", _P),
        ("value2_w", _P),
        ("value2_b", _P),
    ]


class PoolDesc(ctypes.Structure):
    _fields_ = [("base", _P), ("num_pages", ctypes.c_int64)]


STEP_INT_FIELDS = ("num_rows", "num_groups", "num_chunks", "num_legal", "num_extra", "num_group_pages")
STEP_PTR_FIELDS = (
    "piece_ids",
    "side_ids",
    "positions",
    "row_vis",
    "row_extra_off",
    "extra_slot",
    "extra_pos",
    "row_dst_slot",
    "group_page_off",
    "group_pages",
    "chunk_group",
    "chunk_row_off",
    "chunk_nrows",
    "row_perm",
    "legal_off",
    "legal_ids",
    "logits",
    "value_logits",
    "value_stm",
    "legal_logits",
    "legal_logprob",
    "hidden",
    "status",
)


class StepDesc(ctypes.Structure):
    _fields_ = [(n, _I32) for n in STEP_INT_FIELDS] + [(n, _P) for n in STEP_PTR_FIELDS]


_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load (once) and return the library, with argument types declared."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise NativeLibraryError(
                f"{LIB_PATH} is missing: build it with `python -m imba_chess_b200.build` "
                "(the B200 path has no CPU fallback)"
            )
        lib = ctypes.CDLL(LIB_PATH)
        lib.imba_version.restype = _I32
        lib.imba_abi_size.argtypes = [_I32]
        lib.imba_abi_size.restype = _I32
        want = (ctypes.sizeof(ModelDesc), ctypes.sizeof(StepDesc), ctypes.sizeof(PoolDesc))
        got = tuple(int(lib.imba_abi_size(i)) for i in range(3))
        if got != want:
            raise NativeLibraryError(
                f"{LIB_PATH} was built against a different include/imba_b200.h (struct sizes {got}, "
                f"binding expects {want}): rebuild with `python -m imba_chess_b200.build`"
            )
        lib.imba_device_arch.restype = _I32
        lib.imba_model_create.argtypes = [ctypes.POINTER(ModelDesc), ctypes.POINTER(_P)]
        lib.imba_model_create.restype = _I32
        lib.imba_model_destroy.argtypes = [_P]
        lib.imba_model_destroy.restype = None
        lib.imba_step_workspace_bytes.argtypes = [_P, _I32]
        lib.imba_step_workspace_bytes.restype = ctypes.c_size_t
        lib.imba_step.argtypes = [_P, ctypes.POINTER(StepDesc), ctypes.POINTER(PoolDesc), _P, ctypes.c_size_t, _P]
        lib.imba_step.restype = _I32
        lib.imba_step_noalloc.argtypes = [_P, ctypes.POINTER(StepDesc), ctypes.POINTER(PoolDesc), _P]
        lib.imba_step_noalloc.restype = _I32
        lib.imba_profile_event_count.argtypes = [_P]
        lib.imba_profile_event_count.restype = _I32
        lib.imba_step_profiled.argtypes = [_P, ctypes.POINTER(StepDesc), ctypes.POINTER(PoolDesc), _P,
                                           ctypes.c_size_t, _P, ctypes.POINTER(_P), _I32]
        lib.imba_step_profiled.restype = _I32
        for name in ("imba_kv_scatter", "imba_kv_gather"):
            fn = getattr(lib, name)
            fn.argtypes = [_P, ctypes.POINTER(PoolDesc), _I32, _I32, _P, _P, _P, _P, _P]
            fn.restype = _I32
        lib.imba_kv_scatter_indexed.argtypes = [_P, ctypes.POINTER(PoolDesc), _I32, _I32, _P, _P, _P, _P, _P,
                                                ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64), _P,
                                                _P]
        lib.imba_kv_scatter_indexed.restype = _I32
        lib.imba_selftest_wait_timeout.argtypes = [ctypes.c_int64, _P, _P]
        lib.imba_selftest_wait_timeout.restype = _I32
        _lib = lib
        return lib


def check(code: int, what: str) -> None:
    if code != IMBA_OK:
        raise ImbaError(code, what)

"""ctypes binding of ``libffa_b200.so`` (the C ABI declared in include/ffa_b200.h).

There is no fallback: if the library is missing or the tensors are not on a
CUDA device, the call raises.  Every C entry point returns an ``ffa_status``;
a non-zero status becomes a ``RuntimeError`` naming the function and the
library's last error string.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

from .build import LIB_PATH

FFA_OK = 0
FFA_ERR_INVALID_ARG = 1
FFA_ERR_UNSUPPORTED = 2
FFA_ERR_CUDA = 3
FFA_ERR_DEVICE_TIMEOUT = 4
FFA_ERR_WORKSPACE = 5
STATUS_NAMES = {
    0: "FFA_OK",
    1: "FFA_ERR_INVALID_ARG",
    2: "FFA_ERR_UNSUPPORTED",
    3: "FFA_ERR_CUDA",
    4: "FFA_ERR_DEVICE_TIMEOUT",
    5: "FFA_ERR_WORKSPACE",
}

DTYPE_CODE = {torch.float16: 0, torch.bfloat16: 1}
# activation / weight dtypes the MLA projection entry points also accept
IN_DTYPE_CODE = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}

_c_void_p = ctypes.c_void_p
_c_int = ctypes.c_int
_c_float = ctypes.c_float
_c_i64p = ctypes.POINTER(ctypes.c_int64)
_c_size_t = ctypes.c_size_t
_c_u32p = ctypes.c_void_p

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "ffa_version": (_c_int, []),
    "ffa_last_error": (ctypes.c_char_p, []),
    "ffa_read_error": (_c_int, [_c_void_p, ctypes.POINTER(ctypes.c_uint32), _c_void_p]),
    "ffa_set_wait_limit_ns": (None, [ctypes.c_ulonglong]),
    "ffa_fwd": (_c_int, [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,  # q k v o lse
        _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,  # dtype B Hq Hkv Sq Skv D Dv
        _c_i64p, _c_i64p, _c_i64p, _c_i64p,  # strides
        _c_float, _c_int, _c_int, _c_int, _c_float,  # scale causal q_offset window softcap
        _c_void_p, _c_int, _c_int, _c_int, _c_int,  # block_mask n_br n_bc bq bkv
        _c_u32p, _c_void_p,  # err stream
    ]),
    "ffa_bwd_workspace_size": (_c_size_t, [_c_int, _c_int, _c_int]),
    "ffa_bwd": (_c_int, [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,  # dout q k v o lse
        _c_void_p, _c_void_p, _c_void_p,  # dq dk dv
        _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,  # dtype B Hq Hkv Sq Skv D Dv
        _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p,  # strides q k v o do dq dk dv
        _c_float, _c_int, _c_int, _c_int, _c_float,  # scale causal q_offset window softcap
        _c_void_p, _c_size_t, _c_u32p, _c_void_p,  # workspace bytes err stream
    ]),
    "ffa_bwd_masked": (_c_int, [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,  # dout q k v o lse
        _c_void_p, _c_void_p, _c_void_p,  # dq dk dv
        _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,  # dtype B Hq Hkv Sq Skv D Dv
        _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p,  # strides q k v o do dq dk dv
        _c_float, _c_int, _c_int, _c_int, _c_float,  # scale causal q_offset window softcap
        _c_void_p, _c_int, _c_int, _c_int, _c_int,  # block_mask n_br n_bc bq bkv
        _c_void_p, _c_size_t, _c_u32p, _c_void_p,  # workspace bytes err stream
    ]),
    "ffa_bwd_noalloc": (_c_int, [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,  # dout q k v o lse
        _c_void_p, _c_void_p, _c_void_p,  # dq dk dv
        _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,  # dtype B Hq Hkv Sq Skv D
        _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p,  # strides q k v o do dq dk dv
        _c_float, _c_int, _c_int, _c_int, _c_float,  # scale causal q_offset window softcap
        _c_u32p, _c_void_p,  # err stream
    ]),
    "ffa_paged_decode_workspace_size": (_c_size_t, [_c_int, _c_int, _c_int, _c_int, _c_int, _c_int]),
    "ffa_paged_decode": (_c_int, [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,  # q k_pages v_pages block_table ctx_lens
        _c_void_p, _c_void_p,  # out lse
        _c_int, _c_int, _c_int, _c_int, _c_int,  # dtype R Hq Hkv D
        _c_int, _c_int, _c_int,  # num_pages page_size max_pages_per_req
        _c_i64p, _c_i64p, _c_float, _c_float, _c_int,  # q_strides o_strides scale softcap chunks_per_split
        _c_void_p, _c_size_t, _c_u32p, _c_void_p,  # workspace bytes err stream
    ]),
    "ffa_mla_decode_workspace_size": (_c_size_t, [_c_int, _c_int, _c_int, _c_int, _c_int]),
    "ffa_mla_decode": (_c_int, [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,  # q ckv bt lens out lse
        _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,  # dtype R H num_pages page_size max_pages
        _c_i64p, _c_i64p, _c_float, _c_int,  # q_strides o_strides scale chunks_per_split
        _c_void_p, _c_size_t, _c_u32p, _c_void_p,  # workspace bytes err stream
    ]),
    "ffa_merge_partial": (_c_int, [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p,  # o_acc lse_acc o_part lse_part
        _c_int, ctypes.c_int64, _c_int, _c_void_p,  # dtype rows D stream
    ]),
    "ffa_mla_q_absorb": (_c_int, [
        _c_void_p, _c_i64p, _c_void_p, _c_i64p, _c_void_p, _c_i64p,  # q_nope s q_rope s w_uk s
        _c_void_p, _c_void_p, _c_void_p, _c_i64p,  # pos inv_freq out s
        _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_void_p,  # in lat R H d L rope stream
    ]),
    "ffa_mla_o_absorb": (_c_int, [
        _c_void_p, _c_i64p, _c_void_p, _c_i64p, _c_void_p, ctypes.c_int64,  # o_lat s w_uv s out row_stride
        _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_void_p,  # in lat R H d L rope stream
    ]),
    "ffa_mla_latent_append": (_c_int, [
        _c_void_p, ctypes.c_int64, _c_void_p, ctypes.c_int64,  # lat s kr s
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, ctypes.c_int64,  # pos slots inv_freq rows n_slots
        _c_int, _c_int, _c_int, _c_int, _c_int, _c_void_p,  # in lat n L rope stream
    ]),
    "ffa_paged_append": (_c_int, [
        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,  # k_new v_new k_pages v_pages slots
        _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,  # dtype n_tokens Hkv D page_size num_pages
        _c_i64p, _c_void_p,  # new_strides stream
    ]),
}

_LIB: ctypes.CDLL | None = None


def lib_path() -> Path:
    return Path(os.environ.get("FFA_B200_LIB", str(LIB_PATH)))


def load() -> ctypes.CDLL:
    """Load the kernel library (once).  Raises if it is absent."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = lib_path()
    if not path.exists():
        raise RuntimeError(
            f"{path.name} not found at {path}; build it with "
            "`python -m fastest_flash_attention_b200.build` (no CPU fallback exists)")
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def register(name: str, restype, argtypes) -> None:
    SIGNATURES[name] = (restype, argtypes)
    if _LIB is not None:
        fn = getattr(_LIB, name)
        fn.restype = restype
        fn.argtypes = argtypes


def check(status: int, fn: str) -> None:
    if status != FFA_OK:
        msg = load().ffa_last_error().decode(errors="replace")
        raise RuntimeError(f"{fn} failed: {STATUS_NAMES.get(status, status)}" + (f" ({msg})" if msg else ""))


def i64arr(*vals: int):
    return (ctypes.c_int64 * len(vals))(*vals)


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


_ERR_WORDS: dict[int, torch.Tensor] = {}


def err_word(device: torch.device) -> torch.Tensor:
    """Per-device uint32 error word that kernels write on an expired wait."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _ERR_WORDS.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=f"cuda:{idx}")
        _ERR_WORDS[idx] = w
    return w


# Error-word codes that report invalid input data rather than an expired wait.
_DATA_ERRORS = {
    0x1FF: "block mask keeps more key tiles than the forward kernel's tile list holds",
    0x3E0: "paged decode: a context length is negative or exceeds max_pages_per_req * page_size",
    0x3E1: "paged decode: a block-table entry is outside [0, num_pages)",
}


def sync_check_enabled() -> bool:
    """FFA_SYNC_CHECK=1: synchronise after each call and read the error word
    (never while a CUDA graph is being captured, where a synchronisation is
    not allowed; a replayed graph is checked by the caller)."""
    if os.environ.get("FFA_SYNC_CHECK", "0") in ("", "0"):
        return False
    return not torch.cuda.is_current_stream_capturing()


def check_device_errors(device: torch.device | None = None) -> None:
    """Synchronise and raise if any kernel on `device` recorded an expired wait."""
    devs = [device.index] if device is not None else list(_ERR_WORDS)
    for idx in devs:
        w = _ERR_WORDS.get(idx)
        if w is None:
            continue
        code = int(w.item())
        if code != 0:
            w.zero_()
            if code in _DATA_ERRORS:
                raise RuntimeError(f"FFA_ERR_INVALID_ARG: {_DATA_ERRORS[code]} (device code 0x{code:x}) on cuda:{idx}")
            raise RuntimeError(f"FFA_ERR_DEVICE_TIMEOUT: in-kernel wait expired at site 0x{code:x} on cuda:{idx}")


def require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "fastest_flash_attention_b200 runs only on CUDA tensors (sm_100a); got a tensor on "
                f"{t.device}. There is no CPU fallback.")

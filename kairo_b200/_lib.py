"""ctypes binding of libkairo_spmm.so (the C ABI declared in include/kairo_spmm.h).

This module is the only place that talks to the native library.  It builds the
library in-tree when it is missing or stale, declares every entry point's
signature, converts kairo_status codes to Python exceptions and keeps
zero-initialised device workspaces per (device, stream).

There is no fallback: if the library cannot be built or loaded, every operator
raises :class:`KairoLibraryError`.
"""

from __future__ import annotations

import ctypes
import threading
from ctypes import POINTER, Structure, c_char_p, c_int32, c_int64, c_size_t, c_uint32, c_void_p

import torch

from kairo_b200 import _build

# kairo_status
SUCCESS = 0
INVALID_VALUE = 1
NOT_SUPPORTED = 2
CUDA_ERROR = 3
WORKSPACE_TOO_SMALL = 4
DEVICE_ERROR = 5

# kairo_dtype
DTYPE_F32 = 0
DTYPE_F16 = 1
DTYPE_BF16 = 2

# kairo_kernel
KERNEL_AUTO = 0
KERNEL_SIMT = 1
KERNEL_TCGEN05 = 2
KERNEL_SPLIT_BF16 = 3

LAYOUT_STANDARD = 0
LAYOUT_LINEAR = 1

# kairo_schedule
SCHEDULE_AUTO = 0
SCHEDULE_ROWS = 1
SCHEDULE_BANDS = 2
SCHEDULE_GROUPS = 3

ABI_VERSION = 2

# device error codes (low 8 bits of the workspace error word)
DEVERR_NONE = 0
DEVERR_WAIT_TIMEOUT = 1
DEVERR_BAD_INDEX = 2
DEVERR_ROW_TOO_LONG = 3

# wait-site tags of DEVERR_WAIT_TIMEOUT (bits 8..15)
WAIT_SITE_EMPTY = 1
WAIT_SITE_FULL = 2
WAIT_SITE_TMEM_EMPTY = 3
WAIT_SITE_TMEM_FULL = 4
WAIT_SITE_DRAIN = 5

_TORCH_TO_KAIRO = {torch.float32: DTYPE_F32, torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16}


class KairoBsr(Structure):
    _fields_ = [
        ("rows", c_int64),
        ("cols", c_int64),
        ("bm", c_int32),
        ("bk", c_int32),
        ("nbr", c_int32),
        ("reserved0", c_int32),
        ("nnzb", c_int64),
        ("nblocks_stored", c_int64),
        ("row_ptr", c_void_p),
        ("col_idx", c_void_p),
        ("blk_idx", c_void_p),
        ("blocks", c_void_p),
        ("dtype", c_int32),
        ("max_row_blocks", c_int32),
    ]


class KairoSpmmConfig(Structure):
    _fields_ = [
        ("kernel", c_int32),
        ("n_tile", c_int32),
        ("stages", c_int32),
        ("row_cost", c_int32),
        ("num_ctas", c_int32),
        ("group_blocks", c_int32),
        ("schedule", c_int32),
        ("band_rows", c_int32),
        ("wait_kcycles", c_int32),
        ("debug_hold_stage", c_int32),
        ("ctas_per_sm", c_int32),
        ("reserved", c_int32 * 1),
    ]


class KairoSpmmPlan(Structure):
    _fields_ = [
        ("kernel", c_int32),
        ("schedule", c_int32),
        ("launches", c_int32),
        ("grid", c_int32),
        ("n_tile", c_int32),
        ("stages", c_int32),
        ("group_blocks", c_int32),
        ("rows", c_int32),
        ("workspace_bytes", ctypes.c_uint64),
    ]


class KairoBsrStack(Structure):
    """kairo_bsr_stack: row groups of a BSR matrix (kairo_bsr_stack_build)."""

    _fields_ = [
        ("rows_per_group", c_int32),
        ("ngroups", c_int32),
        ("nsuper", c_int64),
        ("group_ptr", c_void_p),
        ("super_col", c_void_p),
        ("super_mask", c_void_p),
        ("super_blk", c_void_p),
        ("row_map", c_void_p),
    ]


class KairoLibraryError(RuntimeError):
    """The native library is missing, failed to build, or failed to load."""


class KairoError(RuntimeError):
    """A kairo_status other than SUCCESS, with the library's message."""

    def __init__(self, status: int, message: str, where: str) -> None:
        self.status = status
        self.message = message
        super().__init__(f"{where}: {message} (kairo status {status})")


class KairoDeviceError(RuntimeError):
    """The device recorded an error in a workspace (bad index, wait timeout)."""

    def __init__(self, code: int) -> None:
        self.code = code
        names = {DEVERR_WAIT_TIMEOUT: "pipeline wait timed out", DEVERR_BAD_INDEX: "block index out of range",
                 DEVERR_ROW_TOO_LONG: "block-row too long for the device sort"}
        super().__init__(f"device error {code & 0xFF} ({names.get(code & 0xFF, 'unknown')}), "
                         f"site {code >> 8}")


_lib: ctypes.CDLL | None = None
_lib_lock = threading.Lock()

# name -> (restype, argtypes)
_SIGNATURES = {
    "kairo_bsr_spmm": (c_int32, [POINTER(KairoBsr), c_void_p, c_int64, c_int32, c_int64, c_void_p, c_int64,
                                 c_int32, POINTER(KairoSpmmConfig), c_void_p, c_size_t, c_void_p]),
    "kairo_bsr_spmm_noalloc": (c_int32, [POINTER(KairoBsr), c_void_p, c_int64, c_int32, c_int64, c_void_p,
                                         c_int64, c_int32, POINTER(KairoSpmmConfig), c_void_p]),
    "kairo_noalloc_error": (c_int32, [c_int32, POINTER(c_uint32), c_void_p]),
    "kairo_bsr_spmm_describe": (c_int32, [POINTER(KairoBsr), c_int32, c_int64, POINTER(KairoSpmmConfig),
                                          POINTER(KairoSpmmPlan)]),
    "kairo_bsr_spmm_workspace_size": (c_int32, [POINTER(KairoBsr), c_int32, c_int64, POINTER(KairoSpmmConfig),
                                                POINTER(c_size_t)]),
    "kairo_bsr_stack_size": (c_int32, [POINTER(KairoBsr), c_int32, POINTER(c_size_t)]),
    "kairo_bsr_stack_build": (c_int32, [POINTER(KairoBsr), c_int32, c_void_p, c_size_t, POINTER(KairoBsrStack),
                                        c_void_p]),
    "kairo_bsr_spmm_stacked_workspace_size": (c_int32, [POINTER(KairoBsr), POINTER(KairoBsrStack), c_int64,
                                                        POINTER(KairoSpmmConfig), POINTER(c_size_t)]),
    "kairo_bsr_spmm_stacked_describe": (c_int32, [POINTER(KairoBsr), POINTER(KairoBsrStack), c_int64,
                                                  POINTER(KairoSpmmConfig), POINTER(KairoSpmmPlan)]),
    "kairo_bsr_spmm_stacked": (c_int32, [POINTER(KairoBsr), POINTER(KairoBsrStack), c_void_p, c_int64, c_int64,
                                         c_void_p, c_int64, POINTER(KairoSpmmConfig), c_void_p, c_size_t,
                                         c_void_p]),
    "kairo_bsr_build": (c_int32, [c_void_p, c_void_p, c_int64, c_int32, c_int32, c_void_p, c_void_p, c_void_p,
                                  POINTER(c_int32), POINTER(c_int32), c_void_p, c_size_t, c_void_p]),
    "kairo_bsr_build_workspace_size": (c_int32, [c_int64, c_int32, POINTER(c_size_t)]),
    "kairo_bsr_transpose": (c_int32, [POINTER(KairoBsr), c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
                                      c_void_p]),
    "kairo_bsr_transpose_workspace_size": (c_int32, [POINTER(KairoBsr), POINTER(c_size_t)]),
    "kairo_bsr_transpose_values": (c_int32, [POINTER(KairoBsr), c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "kairo_bsr_sddmm": (c_int32, [POINTER(KairoBsr), c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p,
                                  c_int64, c_int64, c_void_p, c_int32, c_void_p, c_size_t, c_void_p]),
    "kairo_bsr_sddmm_workspace_size": (c_int32, [POINTER(KairoBsr), POINTER(c_size_t)]),
    "kairo_block_norms": (c_int32, [c_void_p, c_int64, c_int64, c_int64, c_int32, c_int32, c_int32, c_void_p,
                                    c_void_p]),
    "kairo_bsr_block_norms": (c_int32, [POINTER(KairoBsr), c_void_p, c_void_p]),
    "kairo_topk_indices": (c_int32, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_size_t, c_void_p]),
    "kairo_topk_workspace_size": (c_int32, [c_int64, POINTER(c_size_t)]),
    "kairo_coo_sort_rows": (c_int32, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                                      c_void_p, c_void_p, c_size_t, c_void_p]),
    "kairo_coo_sort_rows_workspace_size": (c_int32, [c_int64, c_int64, POINTER(c_size_t)]),
    "kairo_sparse_gather": (c_int32, [c_void_p, c_int64, c_int64, c_int32, c_void_p, c_void_p, c_int64, c_void_p,
                                      c_int64, c_void_p, c_void_p]),
    "kairo_mask_bits": (c_int32, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p]),
    "kairo_sparse_gather_bits": (c_int32, [c_void_p, c_int64, c_int64, c_int32, c_void_p, c_void_p, c_int64,
                                           c_void_p, c_void_p]),
    "kairo_sparse_scatter_grad": (c_int32, [c_void_p, c_int32, c_void_p, c_int64, c_void_p, c_int64, c_int64,
                                            c_int64, c_void_p, c_void_p, c_size_t, c_void_p]),
    "kairo_sparse_scatter_grad_workspace_size": (c_int32, [c_int64, c_int64, POINTER(c_size_t)]),
    "kairo_gather_probe": (c_int32, [c_void_p, c_size_t, c_uint32, c_int32, POINTER(ctypes.c_double), c_void_p]),
    "kairo_dense_to_tiles": (c_int32, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int32,
                                       c_int32, c_void_p, c_void_p]),
    "kairo_acc_spmm_forward": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32,
                                         c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p, c_size_t,
                                         c_void_p]),
    "kairo_acc_spmm_forward_workspace_size": (c_int32, [c_int32, c_int32, c_int32, c_int32, c_int32, c_int32,
                                                        c_int32, POINTER(c_size_t)]),
    "kairo_partition_rows": (c_int32, [POINTER(c_int64), c_int32, c_int32, POINTER(c_int32)]),
    "kairo_workspace_error": (c_int32, [c_void_p, c_int32, POINTER(c_uint32), c_void_p]),
    "kairo_status_string": (c_char_p, [c_int32]),
    "kairo_last_error_message": (c_char_p, []),
    "kairo_abi_version": (c_int32, []),
}

EXPORTED_SYMBOLS = tuple(_SIGNATURES)


def lib() -> ctypes.CDLL:
    """Returns the loaded library, building it in-tree first if needed."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        try:
            path = _build.build()
        except Exception as exc:  # noqa: BLE001 - re-raised with context
            raise KairoLibraryError(f"cannot build libkairo_spmm.so: {exc}") from exc
        try:
            handle = ctypes.CDLL(str(path))
        except OSError as exc:
            raise KairoLibraryError(f"cannot load {path}: {exc}") from exc
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        if handle.kairo_abi_version() != ABI_VERSION:
            raise KairoLibraryError("libkairo_spmm ABI version mismatch")
        _lib = handle
        return handle


def available() -> bool:
    try:
        lib()
        return True
    except KairoLibraryError:
        return False


def check(status: int, where: str) -> None:
    if status != SUCCESS:
        msg = lib().kairo_last_error_message()
        raise KairoError(status, msg.decode() if msg else "", where)


def kairo_dtype(dt: torch.dtype) -> int:
    try:
        return _TORCH_TO_KAIRO[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}; expected float32, float16 or bfloat16") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# ------------------------------------------------------------------ workspaces

_ws_lock = threading.Lock()
_ws_cache: dict[tuple[int, int], torch.Tensor] = {}


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """A zero-initialised device buffer of at least ``nbytes`` bytes for the
    current stream of ``device``.  The library leaves the counters it uses at
    zero, so the buffer is reused across launches on that stream."""
    dev = device.index if device.index is not None else torch.cuda.current_device()
    key = (dev, torch.cuda.current_stream(dev).cuda_stream)
    with _ws_lock:
        buf = _ws_cache.get(key)
        if buf is None or buf.numel() < nbytes:
            size = max(nbytes, 1 << 20)
            buf = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", dev))
            _ws_cache[key] = buf
        return buf


def read_workspace_error(ws: torch.Tensor, clear: bool = True) -> int:
    code = c_uint32(0)
    check(lib().kairo_workspace_error(ws.data_ptr(), 1 if clear else 0, ctypes.byref(code),
                                      stream_handle(ws.device)), "kairo_workspace_error")
    return int(code.value)


def raise_on_device_error(ws: torch.Tensor) -> None:
    code = read_workspace_error(ws, clear=True)
    if code:
        raise KairoDeviceError(code)


class KairoDeviceWarning(RuntimeWarning):
    """A device error that an earlier, unchecked launch left in a workspace."""


def take_pending_error(ws: torch.Tensor, where: str) -> int:
    """Reads and clears the error word of a cached workspace before a launch
    whose own errors the caller asked to see (``check=True``).  An error
    found there was recorded by an earlier launch made with ``check=False``
    on the same stream; it is reported as a :class:`KairoDeviceWarning`
    naming it as such, so that the error read after the checked launch
    belongs to that launch alone.  Returns the earlier code (0 if none)."""
    code = read_workspace_error(ws, clear=True)
    if code:
        import warnings

        warnings.warn(KairoDeviceWarning(f"{where}: an earlier launch with check=False on this stream recorded "
                                         f"{KairoDeviceError(code)}; cleared before this launch"), stacklevel=3)
    return code


def pending_device_error(device: torch.device | int | None = None, clear: bool = True) -> int:
    """The device error word of the cached workspace of ``device``'s current
    stream: what launches made with ``check=False`` there have recorded
    since it was last read (KAIRO_DEVERR_* in the low 8 bits, the wait site
    above them; 0 = none).  Synchronises that stream."""
    if device is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    elif isinstance(device, int):
        dev = torch.device("cuda", device)
    else:
        dev = torch.device(device)
    return read_workspace_error(workspace(0, dev), clear=clear)

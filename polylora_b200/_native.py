"""ctypes binding of libpolylora_b200.so (declared in include/polylora_b200.h).

The library is the only compute path of this package: when it is missing or
fails to load, every kernel wrapper raises :class:`NativeLibraryError`; there
is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from . import build as _build

DTYPE_F32 = 0
DTYPE_F16 = 1
DTYPE_BF16 = 2

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_WORKSPACE = 4
ERR_DEVICE = 5

DEV_WAIT_TIMEOUT = 1
DEV_SLOT_RANGE = 2
DEV_RANK_RANGE = 4
DEV_IMAGE_RANGE = 8
DEV_PADDING = 16
DEV_TOKEN_RANGE = 32

NOALLOC_SCRATCH_BYTES = 8 << 20  # PLORA_NOALLOC_SCRATCH_BYTES

_c_void_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_size = ctypes.c_size_t


class NativeLibraryError(RuntimeError):
    """The CUDA library could not be loaded (no silent fallback exists)."""


class PloraError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, func: str, status: int, detail: str) -> None:
        super().__init__(f"{func} failed with status {status}: {detail}")
        self.func = func
        self.status = status
        self.detail = detail


class SlotModule(ctypes.Structure):
    """plora_slot_module."""

    _fields_ = [
        ("lora_a", _c_void_p),
        ("lora_b", _c_void_p),
        ("ranks", _c_void_p),
        ("scales", _c_void_p),
        ("in_features", _i64),
        ("out_features", _i64),
    ]


class SlotRecord(ctypes.Structure):
    """plora_slot_record."""

    _fields_ = [
        ("a_offset", _i64),
        ("b_offset", _i64),
        ("rank", _i32),
        ("scale", ctypes.c_float),
    ]


# name -> (restype, argtypes)
_SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "plora_version": (ctypes.c_char_p, []),
    "plora_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "plora_last_error": (ctypes.c_char_p, []),
    "plora_device_status": (ctypes.c_int, [ctypes.POINTER(_i32), _i32]),
    "plora_weight_split_tokens_per_sm": (_i64, [_i64]),
    "plora_stream_kernels": (_i32, [_i32]),
    "plora_set_wait_limit_ns": (ctypes.c_int, [ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64)]),
    "plora_peft_pack": (
        ctypes.c_int,
        [ctypes.c_char_p, ctypes.POINTER(ctypes.c_char_p), _i32, ctypes.c_char_p, _i32, ctypes.c_double,
         _c_void_p, _size, ctypes.POINTER(_size), ctypes.POINTER(_i64)],
    ),
    "plora_workspace_size": (_size, [_i64, _i64, _i32]),
    "plora_build_segments": (
        ctypes.c_int,
        [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i32, _c_void_p, _c_void_p, _c_void_p, _size, _c_void_p],
    ),
    "plora_flat_schedule": (
        ctypes.c_int,
        [_c_void_p, _c_void_p, _i64, _i32, _i32, _c_void_p, _c_void_p, _c_void_p],
    ),
    "plora_check_right_padded": (
        ctypes.c_int,
        [_c_void_p, _i32, _i32, _c_void_p, _i64, _i64, _c_void_p],
    ),
    "plora_gather_token_rows": (
        ctypes.c_int,
        [_c_void_p, _c_void_p, _i64, _i64, _c_void_p, _c_void_p, _i32, _c_void_p],
    ),
    "plora_scatter_token_rows": (
        ctypes.c_int,
        [_c_void_p, _c_void_p, _i64, _i64, _c_void_p, _c_void_p, _i32, _c_void_p],
    ),
    "plora_sgmv_a_fwd": (
        ctypes.c_int,
        [
            _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
            _i64, _i64, _i64, _i64, _i32, _i32, _i32, _c_void_p, _size, _c_void_p,
        ],
    ),
    "plora_sgmv_b_fwd": (
        ctypes.c_int,
        [
            _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
            _i64, _i64, _i64, _i64, _i32, _i32, _c_void_p, _size, _c_void_p,
        ],
    ),
    "plora_sgmv_shrink": (
        ctypes.c_int,
        [
            _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
            _i64, _i64, _i64, _i32, _i32, _i32, _c_void_p,
        ],
    ),
    "plora_sgmv_expand": (
        ctypes.c_int,
        [
            _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
            _i64, _i64, _i64, _i32, _i32, _c_void_p,
        ],
    ),
    "plora_sgmv_shrink_expand": (
        ctypes.c_int,
        [
            _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
            _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _i32, _i32, _c_void_p,
        ],
    ),
    "plora_sgmv_a_fwd_noalloc": (
        ctypes.c_int,
        [
            _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
            _i64, _i64, _i64, _i64, _i32, _i32, _i32, _c_void_p,
        ],
    ),
    "plora_slot_fill": (
        ctypes.c_int,
        [_c_void_p, _i32, _i32, _i32, _i64, _i32, _c_void_p, _size, _c_void_p, _size, _c_void_p],
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def library_path() -> Path:
    return _build.LIB_PATH


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Loads (building first if absent and nvcc exists) the C-ABI library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not path.exists() and build_if_missing:
            try:
                _build.build()
            except Exception as exc:  # pragma: no cover - depends on toolchain
                raise NativeLibraryError(f"cannot build {path.name}: {exc}") from exc
        if not path.exists():
            raise NativeLibraryError(f"{path} is missing; run python -m polylora_b200.build")
        try:
            lib = ctypes.CDLL(str(path))
        except OSError as exc:
            raise NativeLibraryError(f"cannot load {path}: {exc}") from exc
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
        return lib


def last_error() -> str:
    return (load().plora_last_error() or b"").decode()


def check(func: str, status: int) -> None:
    if status != OK:
        raise PloraError(func, status, last_error())


def call(func: str, *args: object) -> None:
    """Calls a status-returning entry point and raises on failure."""
    check(func, getattr(load(), func)(*args))


def device_status(clear: bool = True) -> int:
    """Synchronises the current device and returns its status word."""
    out = _i32(0)
    load().plora_device_status(ctypes.byref(out), 1 if clear else 0)
    return int(out.value)


def weight_split_tokens_per_sm(value: int = -1) -> int:
    """Sets (value >= 0) and returns the previous work-split threshold of the
    tensor-core kernels, in tokens per SM (see plora_weight_split_tokens_per_sm)."""
    return int(load().plora_weight_split_tokens_per_sm(value))


def stream_kernels(value: int = -1) -> int:
    """Selects the rank-16 kernel family (2: stream kernels with the combined
    call fused, the default; 1: stream kernels, two launches; 0: windowed) and
    returns the previous setting; -1 only reads (see plora_stream_kernels)."""
    return int(load().plora_stream_kernels(value))


def set_wait_limit_ns(limit_ns: int) -> int:
    """Sets the bounded-wait limit of the current device and returns the
    previous one (see plora_set_wait_limit_ns)."""
    prev = ctypes.c_uint64(0)
    check("plora_set_wait_limit_ns", load().plora_set_wait_limit_ns(int(limit_ns), ctypes.byref(prev)))
    return int(prev.value)


def check_right_padded(mask, seq_lens, stream=None) -> None:
    """Enqueues the device-side right-padding check of a (rows, width) mask
    (see plora_check_right_padded); a violation shows up later as
    DEV_PADDING in device_status().  ``seq_lens`` must be the int64 row sums
    of the same mask, on the same device.  Nothing is read back."""
    import torch

    if mask.dim() != 2:
        raise ValueError("attention_mask must be a 2D batch mask")
    if mask.dtype == torch.bool:
        m = mask.view(torch.uint8)
    else:
        m = mask
    m = m.contiguous()
    lens = seq_lens.to(torch.int64).contiguous()
    is_float = 1 if m.is_floating_point() else 0
    if stream is None:
        stream = torch.cuda.current_stream(m.device).cuda_stream
    check("plora_check_right_padded",
          load().plora_check_right_padded(m.data_ptr(), m.element_size(), is_float, lens.data_ptr(),
                                          m.shape[0], m.shape[1], stream))


def token_rows(host, device, table, to_host: bool, stream=None) -> None:
    """Copies the rows of the table's tokens between a pinned host tensor and
    a device tensor of the same shape (tokens x row elements; see
    plora_gather_token_rows / plora_scatter_token_rows): host -> device, or
    device -> host with ``to_host``.  Other rows are not touched."""
    import torch

    if host.device.type != "cpu" or device.device.type != "cuda":
        raise ValueError("token_rows takes a host tensor and a CUDA tensor")
    if host.shape != device.shape or host.dtype != device.dtype:
        raise ValueError(f"host {tuple(host.shape)} {host.dtype} and device {tuple(device.shape)} {device.dtype} differ")
    if not (host.is_contiguous() and device.is_contiguous()):
        raise ValueError("token_rows needs contiguous tensors")
    if host.numel() == 0:
        return
    if not host.is_pinned():
        raise ValueError("the host tensor must be pinned (page-locked) memory")
    if host.dim() not in (2, 3):
        raise ValueError("token_rows takes (tokens, row) or (rows, seq, row) tensors")
    tokens = host.shape[0] * host.shape[1] if host.dim() == 3 else host.shape[0]
    row_bytes = host.numel() * host.element_size() // max(tokens, 1)
    if stream is None:
        stream = torch.cuda.current_stream(device.device).cuda_stream
    fn = "plora_scatter_token_rows" if to_host else "plora_gather_token_rows"
    args = (device.data_ptr(), host.data_ptr()) if to_host else (host.data_ptr(), device.data_ptr())
    check(fn, getattr(load(), fn)(*args, row_bytes, tokens, table.slot_start.data_ptr(),
                                  table.token_index.data_ptr(), table.num_slots, stream))


def workspace_size(num_rows: int, max_seq: int, num_slots: int) -> int:
    return int(load().plora_workspace_size(num_rows, max_seq, num_slots))


def version() -> str:
    return load().plora_version().decode()

"""ctypes view of libtrring.so (include/trring.h), for callers that reach the C ABI without
the torch binding, and for the tests that exercise the ABI itself.  Pointers are plain
integers (``tensor.data_ptr()``), streams are ``cudaStream_t`` handles as integers."""
from __future__ import annotations

import ctypes
from ctypes import (POINTER, c_char_p, c_double, c_int, c_int32, c_int64, c_size_t,
                    c_uint32, c_void_p)

from ._native import LIBRARY

TR_OK = 0
TR_ERR_INVALID = -1
TR_ERR_UNSUPPORTED = -2
TR_ERR_WORKSPACE = -3
TR_ERR_CUDA = -4
TR_ERR_ALIGN = -5
TR_ERR_TIMEOUT = -6
TR_F32, TR_F16, TR_BF16 = 0, 1, 2
KERNEL_AUTO, KERNEL_GENERIC, KERNEL_MMA, KERNEL_TC05, KERNEL_DECODE, KERNEL_SLAB = 0, 1, 2, 3, 4, 5
TR_EPI_NONE, TR_EPI_ADD, TR_EPI_SILU_MUL = 0, 1, 2


class TrSpec(ctypes.Structure):
    _fields_ = [("input_modes", c_int32 * 3), ("output_modes", c_int32 * 3), ("rank", c_int32)]


class TrTiling(ctypes.Structure):
    _fields_ = [("tokens_per_tile", c_int32), ("cluster", c_int32), ("clusters", c_int32),
                ("kernel", c_int32)]


class TrEpilogue(ctypes.Structure):
    _fields_ = [("kind", c_int32), ("out_dtype", c_int32), ("aux", c_void_p),
                ("aux_dtype", c_int32)]


# name -> (restype, argtypes); every function declared in include/trring.h
PROTOTYPES = {
    "tr_plan_create": (c_int, [POINTER(TrSpec), c_int32, c_int32, POINTER(c_void_p)]),
    "tr_plan_destroy": (None, [c_void_p]),
    "tr_packed_bytes": (c_int, [c_void_p, POINTER(c_size_t)]),
    "tr_pack_cores": (c_int, [c_void_p, POINTER(c_void_p), c_void_p, c_void_p]),
    "tr_workspace_bytes": (c_int, [c_void_p, c_int64, POINTER(c_size_t)]),
    "tr_workspace_bytes_tiled": (c_int, [c_void_p, c_int64, POINTER(TrTiling),
                                         POINTER(c_size_t)]),
    "tr_workspace_clear": (c_int, [c_void_p, c_size_t, c_void_p]),
    "tr_workspace_status": (c_int, [c_void_p, c_size_t, POINTER(c_int32), c_int32, c_void_p]),
    "tr_plan_set_wait_limit": (c_int, [c_void_p, c_uint32]),
    "tr_forward": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_size_t,
                           c_void_p]),
    "tr_forward_tiled": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p,
                                 c_size_t, POINTER(TrTiling), c_void_p]),
    "tr_forward_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p]),
    "tr_forward_host": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p,
                                c_void_p, c_void_p, c_size_t, c_void_p]),
    "tr_forward_epilogue": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p,
                                    POINTER(TrEpilogue), c_void_p, c_size_t, POINTER(TrTiling),
                                    c_void_p]),
    "tr_consume_silu_mul": (c_int, [c_void_p, c_void_p, c_void_p, c_int32, c_int64, c_void_p]),
    "tr_consume_add": (c_int, [c_void_p, c_void_p, c_void_p, c_int32, c_int64, c_void_p]),
    "tr_plan_tiling": (c_int, [c_void_p, c_int64, POINTER(TrTiling)]),
    "tr_plan_describe": (c_int, [c_void_p, c_char_p, c_size_t]),
    "tr_plan_flops_per_token": (c_int, [c_void_p, POINTER(c_double)]),
    "tr_status_string": (c_char_p, [c_int]),
    "tr_last_error": (c_char_p, []),
    "tr_empty_launch": (c_int, [c_void_p]),
}

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            raise RuntimeError(f"{LIBRARY} is not built; run `python -m kernel_task_b200.build`")
        handle = ctypes.CDLL(str(LIBRARY))
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


class AbiError(RuntimeError):
    def __init__(self, status: int, what: str):
        L = lib()
        super().__init__(f"{what}: {L.tr_status_string(status).decode()} "
                         f"({L.tr_last_error().decode()})")
        self.status = status


def check(status: int, what: str) -> None:
    if status != TR_OK:
        raise AbiError(status, what)


def workspace_status(ws_ptr: int, ws_bytes: int, reset: bool = True, stream: int = 0) -> int:
    """The device status word of a workspace (TR_OK or TR_ERR_TIMEOUT); synchronises `stream`."""
    st = c_int32()
    check(lib().tr_workspace_status(c_void_p(ws_ptr or None), ws_bytes, ctypes.byref(st),
                                    1 if reset else 0, c_void_p(stream)), "tr_workspace_status")
    return st.value


class Plan:
    """Owner of one tr_plan handle."""

    def __init__(self, input_modes, output_modes, rank: int, dtype: int, device: int = 0):
        spec = TrSpec((c_int32 * 3)(*input_modes), (c_int32 * 3)(*output_modes), rank)
        handle = c_void_p()
        check(lib().tr_plan_create(ctypes.byref(spec), dtype, device, ctypes.byref(handle)),
              "tr_plan_create")
        self.handle = handle

    def __del__(self):
        if getattr(self, "handle", None) and _lib is not None:
            _lib.tr_plan_destroy(self.handle)
            self.handle = None

    def packed_bytes(self) -> int:
        n = c_size_t()
        check(lib().tr_packed_bytes(self.handle, ctypes.byref(n)), "tr_packed_bytes")
        return n.value

    def workspace_bytes(self, tokens: int, tiling: TrTiling | None = None) -> int:
        n = c_size_t()
        check(lib().tr_workspace_bytes_tiled(self.handle, tokens,
                                             ctypes.byref(tiling) if tiling else None,
                                             ctypes.byref(n)), "tr_workspace_bytes")
        return n.value

    def pack(self, core_ptrs, packed_ptr: int, stream: int = 0) -> None:
        arr = (c_void_p * 3)(*core_ptrs)
        check(lib().tr_pack_cores(self.handle, arr, c_void_p(packed_ptr), c_void_p(stream)),
              "tr_pack_cores")

    def forward(self, packed_ptr: int, x_ptr: int, tokens: int, y_ptr: int, ws_ptr: int = 0,
                ws_bytes: int = 0, stream: int = 0, tiling: TrTiling | None = None) -> int:
        return lib().tr_forward_tiled(self.handle, c_void_p(packed_ptr), c_void_p(x_ptr), tokens,
                                      c_void_p(y_ptr), c_void_p(ws_ptr or None), ws_bytes,
                                      ctypes.byref(tiling) if tiling else None, c_void_p(stream))

    def forward_host(self, packed_ptr: int, x_host_ptr: int, tokens: int, y_host_ptr: int,
                     x_dev_ptr: int, y_dev_ptr: int, ws_ptr: int = 0, ws_bytes: int = 0,
                     stream: int = 0) -> int:
        """tr_forward on host buffers through caller-owned device staging (three stream-ordered
        operations; synchronise before reading y)."""
        return lib().tr_forward_host(self.handle, c_void_p(packed_ptr), c_void_p(x_host_ptr),
                                     tokens, c_void_p(y_host_ptr), c_void_p(x_dev_ptr),
                                     c_void_p(y_dev_ptr), c_void_p(ws_ptr or None), ws_bytes,
                                     c_void_p(stream))

    def forward_noalloc(self, packed_ptr: int, x_ptr: int, tokens: int, y_ptr: int,
                        stream: int = 0) -> int:
        """tr_forward with the library's built-in scratch (no caller workspace)."""
        return lib().tr_forward_noalloc(self.handle, c_void_p(packed_ptr), c_void_p(x_ptr),
                                        tokens, c_void_p(y_ptr), c_void_p(stream))

    def forward_epilogue(self, packed_ptr: int, x_ptr: int, tokens: int, y_ptr: int,
                         epilogue: TrEpilogue | None, ws_ptr: int = 0, ws_bytes: int = 0,
                         stream: int = 0, tiling: TrTiling | None = None) -> int:
        return lib().tr_forward_epilogue(
            self.handle, c_void_p(packed_ptr), c_void_p(x_ptr), tokens, c_void_p(y_ptr),
            ctypes.byref(epilogue) if epilogue else None, c_void_p(ws_ptr or None), ws_bytes,
            ctypes.byref(tiling) if tiling else None, c_void_p(stream))

    def set_wait_limit(self, polls: int) -> None:
        """Polls of a bounded device-side wait before it gives up (0 = built-in limit)."""
        check(lib().tr_plan_set_wait_limit(self.handle, polls), "tr_plan_set_wait_limit")

    def tiling(self, tokens: int) -> TrTiling:
        t = TrTiling()
        check(lib().tr_plan_tiling(self.handle, tokens, ctypes.byref(t)), "tr_plan_tiling")
        return t

    def describe(self) -> str:
        buf = ctypes.create_string_buffer(1024)
        check(lib().tr_plan_describe(self.handle, buf, len(buf)), "tr_plan_describe")
        return buf.value.decode()

    def flops_per_token(self) -> float:
        f = c_double()
        check(lib().tr_plan_flops_per_token(self.handle, ctypes.byref(f)), "flops")
        return f.value

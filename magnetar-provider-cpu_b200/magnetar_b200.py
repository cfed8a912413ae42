"""Python mirror of the B200 Provider's C ABI (include/magnetar_b200.h).

`B200Provider` follows the reference's `NativeCpuProvider` /
`NativeCpuExecutor` API (src/native/mod.rs): `write_packed_weight_tensor`
returns "Stored" or "Declined", `read_tensor` returns the dequantised
values, `submit_kernel` returns a handle that `complete_kernel` consumes
once.  The low-level functions (`qmatmul`, `dequantize`, ...) take device
pointers (ints) and a CUDA stream handle.

The library must have been built (magnetar-provider-cpu_b200/build.py); there
is no fallback: `lib()` raises when libmagnetar_b200.so is missing.
"""

from __future__ import annotations

import ctypes
import pathlib
from dataclasses import dataclass

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "libmagnetar_b200.so"
HEADER = HERE.parent / "include" / "magnetar_b200.h"

OK, DECLINED, EXECUTION_FAILED, DTYPE_UNSUPPORTED, ATTRIBUTE_UNSUPPORTED = 0, 1, 2, 3, 4
KERNEL_NOT_FOUND, TIMEOUT, MEMORY_DENIED, UNKNOWN_HANDLE, NOT_FOUND = 5, 6, 7, 8, 9
INVALID_ARGUMENT, CUDA_ERROR, NCCL_ERROR, UNSUPPORTED = 10, 11, 12, 13

Q8_0, Q4_K, Q6_K, IQ4_NL, Q5_K, Q4_0 = 0, 1, 2, 5, 12, 13
FORMATS = {"q8_0": Q8_0, "q4_k": Q4_K, "q5_k": Q5_K, "q6_k": Q6_K, "iq4_nl": IQ4_NL, "q4_0": Q4_0}
BLOCK = {Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210), IQ4_NL: (32, 18),
         Q4_0: (32, 18)}
KERNEL_AUTO, KERNEL_GEMV, KERNEL_GEMM = 0, 1, 2
MAX_RANK = 8


class MgbError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{status_name(status)}: {message}")
        self.status = status


class Settings(ctypes.Structure):
    _fields_ = [("packed_weights", ctypes.c_int32), ("int8_activations", ctypes.c_int32),
                ("device", ctypes.c_int32), ("profile", ctypes.c_int32),
                ("kernel", ctypes.c_int32)]


class Metadata(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("version", ctypes.c_char_p),
                ("vendor", ctypes.c_char_p), ("description", ctypes.c_char_p)]


class DeviceDescriptor(ctypes.Structure):
    _fields_ = [("id", ctypes.c_char * 64), ("name", ctypes.c_char * 128),
                ("architecture", ctypes.c_char * 32), ("compute_units", ctypes.c_uint32),
                ("memory_bytes", ctypes.c_uint64), ("max_concurrent_operations", ctypes.c_uint32),
                ("max_workspace_bytes", ctypes.c_uint64)]


class Advertisement(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("operator_family", ctypes.c_char_p),
                ("rank", ctypes.c_int32), ("input_dtype", ctypes.c_int32),
                ("output_dtype", ctypes.c_int32), ("cancellation", ctypes.c_int32)]


class KernelAttrs(ctypes.Structure):
    _fields_ = [("transpose_a", ctypes.c_int32), ("transpose_b", ctypes.c_int32),
                ("accumulation_dtype", ctypes.c_int32), ("deadline_ms", ctypes.c_int64),
                ("has_scale", ctypes.c_int32), ("scale", ctypes.c_float)]


class KernelResult(ctypes.Structure):
    _fields_ = [("status", ctypes.c_int32), ("reason", ctypes.c_char * 256)]


class Observation(ctypes.Structure):
    _fields_ = [("sequence", ctypes.c_uint64), ("kind", ctypes.c_int32),
                ("kernel", ctypes.c_char * 48), ("detail", ctypes.c_char * 112)]


MAX_TP = 8
TP_SYNC_BYTES = 256
TP_COUNTER_OFFSET = 128
TP_EPOCH_OFFSET = 132  # device epochs: the rank's epoch word
IPC_HANDLE_BYTES = 64


class TpOut(ctypes.Structure):
    """`mgb_tp_out`: where one rank's tensor-parallel call writes."""
    _fields_ = [("y", ctypes.c_void_p * MAX_TP), ("done", ctypes.c_void_p * MAX_TP),
                ("cta_counter", ctypes.c_void_p), ("ldy", ctypes.c_uint64),
                ("col0", ctypes.c_uint64), ("epoch", ctypes.c_uint32), ("world", ctypes.c_int32),
                ("rank", ctypes.c_int32), ("wait_done", ctypes.c_void_p),
                ("wait_epoch", ctypes.c_uint32), ("wait_world", ctypes.c_int32),
                ("wait_timeout_ms", ctypes.c_uint32)]


_lib = None
_vp, _u64, _i32, _cp = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int32, ctypes.c_char_p
_u64p = ctypes.POINTER(ctypes.c_uint64)
_i32p = ctypes.POINTER(ctypes.c_int32)

_SIGNATURES = {
    "mgb_last_error": ([], _cp),
    "mgb_status_name": ([_i32], _cp),
    "mgb_abi_version": ([], _i32),
    "mgb_provider_get_metadata": ([ctypes.POINTER(Metadata)], None),
    "mgb_settings_from_env": ([ctypes.POINTER(Settings)], _i32),
    "mgb_provider_create": ([ctypes.POINTER(Settings), ctypes.POINTER(_vp)], _i32),
    "mgb_provider_destroy": ([_vp], None),
    "mgb_provider_initialize": ([_vp], _i32),
    "mgb_provider_shutdown": ([_vp], _i32),
    "mgb_provider_health": ([_vp], _i32),
    "mgb_provider_device": ([_vp, ctypes.POINTER(DeviceDescriptor)], _i32),
    "mgb_kernel_advertisement_count": ([], ctypes.c_size_t),
    "mgb_kernel_advertisement_get": ([ctypes.c_size_t, ctypes.POINTER(Advertisement)], _i32),
    "mgb_write_tensor": ([_vp, _cp, _u64p, _i32, _vp], _i32),
    "mgb_write_packed_weight": ([_vp, _cp, _i32, _u64, _u64, _i32, _vp, _u64, _i32p], _i32),
    "mgb_read_tensor": ([_vp, _cp, _vp, _u64, _u64p, _i32p], _i32),
    "mgb_resident_shape": ([_vp, _cp, _u64p, _i32p], _i32),
    "mgb_release_tensor": ([_vp, _cp, _i32p], _i32),
    "mgb_is_packed": ([_vp, _cp], _i32),
    "mgb_read_tensor_value": ([_vp, _cp, _i32p], _i32),
    "mgb_write_tensor_value_opaque": ([_vp, _cp], _i32),
    "mgb_copy_tensor": ([_vp, _cp, _cp], _i32),
    "mgb_device_memory": ([_vp, _u64p, _u64p], _i32),
    "mgb_materialization_count": ([_vp], _u64),
    "mgb_submit_kernel": ([_vp, _cp, ctypes.POINTER(KernelAttrs), ctypes.POINTER(_cp), _i32, _cp,
                           _u64p], _i32),
    "mgb_complete_kernel": ([_vp, _u64, ctypes.POINTER(KernelResult)], _i32),
    "mgb_observation_count": ([_vp], ctypes.c_size_t),
    "mgb_observations": ([_vp, ctypes.POINTER(Observation), ctypes.c_size_t,
                          ctypes.POINTER(ctypes.c_size_t)], _i32),
    "mgb_packed_bytes": ([_i32, _u64, _u64], _u64),
    "mgb_repack": ([_i32, _vp, _u64, _u64, _vp, _vp], _i32),
    "mgb_qmatmul_workspace_bytes": ([_i32, _u64, _u64, _u64], _u64),
    "mgb_qmatmul_min_workspace_bytes": ([_i32, _u64, _u64, _u64], _u64),
    "mgb_qmatmul": ([_i32, _vp, _u64, _u64, _vp, _u64, _vp, _vp, _u64, _vp, _u64, _vp], _i32),
    "mgb_qmatmul_static_scratch": ([_i32, _vp, _u64, _u64, _vp, _u64, _vp, _vp, _u64, _vp],
                                   _i32),
    "mgb_qmatmul_bf16": ([_i32, _vp, _u64, _u64, _vp, _u64, _vp, _vp, _u64, _vp], _i32),
    "mgb_dequantize": ([_i32, _vp, _u64, _u64, _vp, _vp], _i32),
    "mgb_qmatmul_input_major": ([_i32, _vp, _u64, _u64, _vp, _u64, _vp, _vp], _i32),
    "mgb_matmul_f32": ([_vp, _u64, _u64, _vp, _u64, _u64, _i32, _i32, _vp, _vp], _i32),
    "mgb_quantize_rows": ([_vp, _u64, _vp, _vp, _vp, _vp], _i32),
    "mgb_take_device_error": ([_i32, _i32p], _i32),
    "mgb_embedding": ([_i32, _vp, _u64, _u64, _i32, _vp, _u64, _i32, ctypes.c_float, _vp, _vp, _vp],
                      _i32),
    "mgb_device_alloc": ([_u64, ctypes.POINTER(_vp)], _i32),
    "mgb_device_free": ([_vp], _i32),
    "mgb_ipc_handle": ([_vp, _vp], _i32),
    "mgb_ipc_open": ([_vp, ctypes.POINTER(_vp)], _i32),
    "mgb_ipc_close": ([_vp], _i32),
    "mgb_qmatmul_tp": ([_i32, _vp, _u64, _u64, _vp, _u64, ctypes.POINTER(TpOut), _vp, _u64, _vp,
                        _u64, _vp], _i32),
    "mgb_tp_wait": ([_vp, _i32, ctypes.c_uint32, ctypes.c_uint32, _vp], _i32),
}


def header_functions() -> list[str]:
    """Every function the C header declares (for the export check)."""
    import re

    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z0-9_]+\s*\*?\s*(mgb_[a-z0-9_]+)\s*\(",
                                 text, flags=re.M)))


def lib() -> ctypes.CDLL:
    """Loads libmagnetar_b200.so (raises when it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run magnetar-provider-cpu_b200/build.py")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (args, res) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def status_name(status: int) -> str:
    return lib().mgb_status_name(status).decode()


def last_error() -> str:
    return lib().mgb_last_error().decode()


def check(status: int) -> None:
    if status != OK:
        raise MgbError(status, last_error())


def packed_bytes(fmt: int, rows: int, cols: int) -> int:
    return int(lib().mgb_packed_bytes(fmt, rows, cols))


# ---- low-level device entry points (device pointers as ints) -------------------------


def repack(fmt: int, ggml_ptr: int, rows: int, cols: int, out_ptr: int, stream: int = 0) -> None:
    check(lib().mgb_repack(fmt, ggml_ptr, rows, cols, out_ptr, stream))


def qmatmul_workspace_bytes(fmt: int, m: int, n: int, k: int) -> int:
    return int(lib().mgb_qmatmul_workspace_bytes(fmt, m, n, k))


def qmatmul_min_workspace_bytes(fmt: int, m: int, n: int, k: int) -> int:
    return int(lib().mgb_qmatmul_min_workspace_bytes(fmt, m, n, k))


def qmatmul(fmt: int, w_ptr: int, n: int, k: int, x_ptr: int, m: int, y_ptr: int,
            addend_ptr: int = 0, addend_len: int = 0, workspace_ptr: int = 0,
            workspace_bytes: int = 0, stream: int = 0) -> None:
    check(lib().mgb_qmatmul(fmt, w_ptr, n, k, x_ptr, m, y_ptr, addend_ptr or None, addend_len,
                            workspace_ptr or None, workspace_bytes, stream or None))


def qmatmul_bf16(fmt: int, w_ptr: int, n: int, k: int, xb_ptr: int, m: int, y_ptr: int,
                 addend_ptr: int = 0, addend_len: int = 0, stream: int = 0) -> None:
    check(lib().mgb_qmatmul_bf16(fmt, w_ptr, n, k, xb_ptr, m, y_ptr, addend_ptr or None,
                                 addend_len, stream or None))


def dequantize(fmt: int, w_ptr: int, rows: int, cols: int, out_ptr: int, stream: int = 0) -> None:
    check(lib().mgb_dequantize(fmt, w_ptr, rows, cols, out_ptr, stream or None))


def qmatmul_input_major(fmt: int, w_ptr: int, rows: int, cols: int, x_ptr: int, m: int,
                        y_ptr: int, stream: int = 0) -> None:
    check(lib().mgb_qmatmul_input_major(fmt, w_ptr, rows, cols, x_ptr, m, y_ptr, stream or None))


def embedding(fmt: int, w_ptr: int, stored_rows: int, stored_cols: int, transposed: bool,
              ids_ptr: int, count: int, out_ptr: int, scale: float | None = None, bad_ptr: int = 0,
              stream: int = 0) -> None:
    check(lib().mgb_embedding(fmt, w_ptr, stored_rows, stored_cols, int(transposed), ids_ptr,
                              count, int(scale is not None), 1.0 if scale is None else scale,
                              out_ptr, bad_ptr or None, stream or None))


def take_device_error(device: int = 0) -> int:
    code = ctypes.c_int32(0)
    check(lib().mgb_take_device_error(device, ctypes.byref(code)))
    return code.value


# ---- tensor parallelism (device pointers as ints) -------------------------------------


def device_alloc(nbytes: int) -> int:
    """A whole zero-filled cudaMalloc allocation on the current device."""
    p = ctypes.c_void_p()
    check(lib().mgb_device_alloc(nbytes, ctypes.byref(p)))
    return int(p.value)


def device_free(ptr: int) -> None:
    check(lib().mgb_device_free(ptr or None))


def ipc_handle(ptr: int) -> bytes:
    buf = (ctypes.c_uint8 * IPC_HANDLE_BYTES)()
    check(lib().mgb_ipc_handle(ptr, buf))
    return bytes(buf)


def ipc_open(handle: bytes) -> int:
    if len(handle) != IPC_HANDLE_BYTES:
        raise ValueError(f"an IPC handle has {IPC_HANDLE_BYTES} bytes, not {len(handle)}")
    buf = (ctypes.c_uint8 * IPC_HANDLE_BYTES).from_buffer_copy(handle)
    p = ctypes.c_void_p()
    check(lib().mgb_ipc_open(buf, ctypes.byref(p)))
    return int(p.value)


def ipc_close(ptr: int) -> None:
    check(lib().mgb_ipc_close(ptr or None))


def tp_out(y: list[int], done: list[int], cta_counter: int, ldy: int, col0: int, epoch: int,
           rank: int, wait_done: int = 0, wait_epoch: int = 0, wait_world: int = 0,
           wait_timeout_ms: int = 0) -> TpOut:
    """`mgb_tp_out`; wait_done (this rank's synchronisation words of an earlier
    fused call) makes the call wait for that call's epoch before reading x."""
    world = len(y)
    if len(done) != world:
        raise ValueError("one done pointer per rank")
    o = TpOut()
    for r in range(world):
        o.y[r] = y[r]
        o.done[r] = done[r]
    o.cta_counter = cta_counter
    o.ldy, o.col0, o.epoch, o.world, o.rank = ldy, col0, epoch & 0xFFFFFFFF, world, rank
    o.wait_done = wait_done or None
    o.wait_epoch, o.wait_world, o.wait_timeout_ms = wait_epoch & 0xFFFFFFFF, wait_world, wait_timeout_ms
    return o


def qmatmul_tp(fmt: int, w_ptr: int, n: int, k: int, x_ptr: int, m: int, out: TpOut,
               addend_ptr: int = 0, addend_len: int = 0, workspace_ptr: int = 0,
               workspace_bytes: int = 0, stream: int = 0) -> None:
    check(lib().mgb_qmatmul_tp(fmt, w_ptr, n, k, x_ptr, m, ctypes.byref(out), addend_ptr or None,
                               addend_len, workspace_ptr or None, workspace_bytes, stream or None))


def tp_wait(done_ptr: int, world: int, epoch: int, timeout_ms: int = 0, stream: int = 0) -> None:
    check(lib().mgb_tp_wait(done_ptr or None, world, epoch & 0xFFFFFFFF, timeout_ms,
                            stream or None))


# ---- the Provider ---------------------------------------------------------------------


@dataclass
class KernelOutcome:
    status: int
    reason: str

    @property
    def ok(self) -> bool:
        return self.status == OK


def settings_from_env() -> Settings:
    s = Settings()
    check(lib().mgb_settings_from_env(ctypes.byref(s)))
    return s


def metadata() -> dict:
    m = Metadata()
    lib().mgb_provider_get_metadata(ctypes.byref(m))
    return {"name": m.name.decode(), "version": m.version.decode(), "vendor": m.vendor.decode(),
            "description": m.description.decode()}


def kernel_advertisements() -> list[dict]:
    out = []
    for i in range(lib().mgb_kernel_advertisement_count()):
        a = Advertisement()
        check(lib().mgb_kernel_advertisement_get(i, ctypes.byref(a)))
        out.append({"name": a.name.decode(), "operator_family": a.operator_family.decode(),
                    "rank": a.rank, "input_dtype": a.input_dtype, "output_dtype": a.output_dtype,
                    "cancellation": a.cancellation})
    return out


class B200Provider:
    """The Provider (`NativeCpuProvider` + `NativeCpuExecutor` counterpart)."""

    def __init__(self, packed_weights: bool = True, int8_activations: bool = False,
                 device: int = 0, profile: bool = False, kernel: int = KERNEL_AUTO,
                 from_env: bool = False):
        s = settings_from_env() if from_env else Settings(int(packed_weights),
                                                          int(int8_activations), device,
                                                          int(profile), kernel)
        h = _vp()
        check(lib().mgb_provider_create(ctypes.byref(s), ctypes.byref(h)))
        self._h = h
        self.settings = s

    def close(self) -> None:
        if self._h:
            lib().mgb_provider_destroy(self._h)
            self._h = _vp()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    # identity / lifecycle
    def initialize(self) -> None:
        check(lib().mgb_provider_initialize(self._h))

    def shutdown(self) -> None:
        check(lib().mgb_provider_shutdown(self._h))

    def health(self) -> int:
        return lib().mgb_provider_health(self._h)

    def device(self) -> dict:
        d = DeviceDescriptor()
        check(lib().mgb_provider_device(self._h, ctypes.byref(d)))
        return {"id": d.id.decode(), "name": d.name.decode(),
                "architecture": d.architecture.decode(), "compute_units": d.compute_units,
                "memory_bytes": d.memory_bytes}

    # storage
    def write_tensor(self, id: str, tensor: np.ndarray) -> None:
        a = np.ascontiguousarray(tensor, dtype=np.float32)
        shape = (ctypes.c_uint64 * max(1, a.ndim))(*a.shape)
        check(lib().mgb_write_tensor(self._h, id.encode(), shape, a.ndim,
                                     a.ctypes.data if a.size else None))

    def write_tensor_ptr(self, id: str, shape: tuple[int, ...], host_ptr: int) -> None:
        """`write_tensor` from a raw host pointer (e.g. a pinned buffer)."""
        sh = (ctypes.c_uint64 * max(1, len(shape)))(*shape)
        check(lib().mgb_write_tensor(self._h, id.encode(), sh, len(shape), host_ptr))

    def read_tensor_into(self, id: str, host_ptr: int, capacity: int) -> list[int]:
        """`read_tensor` into a raw host pointer of `capacity` floats; returns the shape."""
        sh = (ctypes.c_uint64 * MAX_RANK)()
        rank = ctypes.c_int32(0)
        check(lib().mgb_read_tensor(self._h, id.encode(), host_ptr, capacity, sh,
                                    ctypes.byref(rank)))
        return [int(sh[i]) for i in range(rank.value)]

    def write_packed_weight_tensor(self, id: str, fmt: int, stored_rows: int, stored_cols: int,
                                   transposed: bool, data: np.ndarray) -> str:
        b = np.ascontiguousarray(data, dtype=np.uint8)
        stored = ctypes.c_int32(0)
        check(lib().mgb_write_packed_weight(self._h, id.encode(), fmt, stored_rows, stored_cols,
                                            int(transposed), b.ctypes.data if b.size else None,
                                            b.size, ctypes.byref(stored)))
        return "Stored" if stored.value else "Declined"

    def resident_shape(self, id: str) -> list[int] | None:
        shape = (ctypes.c_uint64 * MAX_RANK)()
        rank = ctypes.c_int32(0)
        s = lib().mgb_resident_shape(self._h, id.encode(), shape, ctypes.byref(rank))
        if s == NOT_FOUND:
            return None
        check(s)
        return [int(shape[i]) for i in range(rank.value)]

    def read_tensor(self, id: str) -> np.ndarray | None:
        shape = self.resident_shape(id)
        if shape is None:
            return None
        out = np.empty(shape, dtype=np.float32)
        sh = (ctypes.c_uint64 * MAX_RANK)()
        rank = ctypes.c_int32(0)
        check(lib().mgb_read_tensor(self._h, id.encode(), out.ctypes.data, out.size, sh,
                                    ctypes.byref(rank)))
        return out

    def release_tensor(self, id: str) -> bool:
        was = ctypes.c_int32(0)
        check(lib().mgb_release_tensor(self._h, id.encode(), ctypes.byref(was)))
        return bool(was.value)

    def is_packed(self, id: str) -> bool:
        return bool(lib().mgb_is_packed(self._h, id.encode()))

    def read_tensor_value(self, id: str) -> str | None:
        kind = ctypes.c_int32(0)
        check(lib().mgb_read_tensor_value(self._h, id.encode(), ctypes.byref(kind)))
        return "Opaque" if kind.value else None

    def write_tensor_value_opaque(self, id: str) -> None:
        check(lib().mgb_write_tensor_value_opaque(self._h, id.encode()))

    def copy_tensor(self, src: str, dst: str) -> None:
        check(lib().mgb_copy_tensor(self._h, src.encode(), dst.encode()))

    def device_memory(self) -> tuple[int, int]:
        f, t = ctypes.c_uint64(0), ctypes.c_uint64(0)
        check(lib().mgb_device_memory(self._h, ctypes.byref(f), ctypes.byref(t)))
        return f.value, t.value

    def materializations(self) -> int:
        return int(lib().mgb_materialization_count(self._h))

    # execution
    def submit_kernel(self, kernel: str, inputs: list[str], output: str,
                      transpose_a: bool = False, transpose_b: bool = False,
                      accumulation_dtype: int = 0, deadline_ms: int | None = None,
                      scale: float | None = None) -> int:
        attrs = KernelAttrs(int(transpose_a), int(transpose_b), accumulation_dtype,
                            -1 if deadline_ms is None else deadline_ms, int(scale is not None),
                            1.0 if scale is None else scale)
        arr = (ctypes.c_char_p * max(1, len(inputs)))(*[i.encode() for i in inputs])
        handle = ctypes.c_uint64(0)
        check(lib().mgb_submit_kernel(self._h, kernel.encode(), ctypes.byref(attrs), arr,
                                      len(inputs), output.encode(), ctypes.byref(handle)))
        return handle.value

    def complete_kernel(self, handle: int) -> KernelOutcome:
        r = KernelResult()
        check(lib().mgb_complete_kernel(self._h, handle, ctypes.byref(r)))
        return KernelOutcome(r.status, r.reason.decode())

    def observations(self) -> list[dict]:
        n = lib().mgb_observation_count(self._h)
        arr = (Observation * max(1, n))()
        written = ctypes.c_size_t(0)
        check(lib().mgb_observations(self._h, arr, n, ctypes.byref(written)))
        return [{"sequence": arr[i].sequence, "kind": arr[i].kind,
                 "kernel": arr[i].kernel.decode(), "detail": arr[i].detail.decode()}
                for i in range(written.value)]

    def embedding(self, ids: np.ndarray, table_id: str, output: str = "__e",
                  scale: float | None = None) -> np.ndarray:
        """write the ids (f32), submit `embedding`, complete, read [count, dim]."""
        self.write_tensor("__ids", np.asarray(ids, dtype=np.float32).reshape(-1))
        h = self.submit_kernel("embedding", [table_id, "__ids"], output, scale=scale)
        outcome = self.complete_kernel(h)
        if not outcome.ok:
            raise MgbError(outcome.status, outcome.reason)
        return self.read_tensor(output)

    def matmul(self, x: np.ndarray, weight_id: str, output: str = "__y", **attrs) -> np.ndarray:
        """write x, submit `matmul`, complete, read y (a convenience for tests)."""
        self.write_tensor("__x", x)
        h = self.submit_kernel("matmul", ["__x", weight_id], output, **attrs)
        outcome = self.complete_kernel(h)
        if not outcome.ok:
            raise MgbError(outcome.status, outcome.reason)
        return self.read_tensor(output)

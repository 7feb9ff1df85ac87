"""Python mirror of the reference's backend plugin interface, over the library's C ABI.

Names, argument meaning and error behaviour follow the C# contract the reference's callers use:
  IShorokooInferenceSessionFactory  src/Shorokoo/Core/Inference/Abstractions/IShorokooInferenceSessionFactory.cs:5-24
  IShorokooInferenceSession         src/Shorokoo/Core/Inference/Abstractions/IShorokooInferenceSession.cs:3-13
  IShorokooTensorValue              src/Shorokoo/Core/Inference/Abstractions/IShorokooTensorValue.cs:8-31
The ORT implementation being replaced is src/Backend/OnnxRuntime/Shorokoo.OnnxRuntime/*.cs; this
factory takes the Shorokoo.LinuxGPU slot (LinuxGpuInferenceFactory.cs:5-8). Exceptions map the
library status codes the way the C# shim does: invalid argument / shape -> ValueError
(ArgumentException), unsupported -> NotImplementedError (NotSupportedException), CUDA / internal ->
RuntimeError (InvalidOperationException), out of memory -> MemoryError.
"""
from __future__ import annotations

import ctypes as C
from enum import IntEnum
from typing import Dict, List, Mapping, Optional, Sequence

import numpy as np

from . import _native


class ShorokooTensorElementType(IntEnum):   # ShorokooTensorElementType.cs:6-31
    Float = 1
    UInt8 = 2
    Int8 = 3
    UInt16 = 4
    Int16 = 5
    Int32 = 6
    Int64 = 7
    String = 8
    Bool = 9
    Float16 = 10
    Double = 11
    UInt32 = 12
    UInt64 = 13
    BFloat16 = 16


class ShorokooGraphOptimization(IntEnum):   # ShorokooGraphOptimization.cs
    DisableAll = 0
    EnableBasic = 1
    EnableExtended = 2
    EnableAll = 99


class ShorokooLogSeverity(IntEnum):   # ShorokooLogSeverity.cs
    Verbose = 0
    Info = 1
    Warning = 2
    Error = 3
    Fatal = 4


class ShorokooOnnxValueType(IntEnum):   # ShorokooOnnxValueType.cs
    Unknown = 0
    Tensor = 1
    Sequence = 2


NP_TO_ELEM = {
    np.dtype(np.float32): ShorokooTensorElementType.Float, np.dtype(np.uint8): ShorokooTensorElementType.UInt8,
    np.dtype(np.int8): ShorokooTensorElementType.Int8, np.dtype(np.uint16): ShorokooTensorElementType.UInt16,
    np.dtype(np.int16): ShorokooTensorElementType.Int16, np.dtype(np.int32): ShorokooTensorElementType.Int32,
    np.dtype(np.int64): ShorokooTensorElementType.Int64, np.dtype(np.bool_): ShorokooTensorElementType.Bool,
    np.dtype(np.float16): ShorokooTensorElementType.Float16, np.dtype(np.float64): ShorokooTensorElementType.Double,
    np.dtype(np.uint32): ShorokooTensorElementType.UInt32, np.dtype(np.uint64): ShorokooTensorElementType.UInt64,
}
ELEM_TO_NP = {int(v): k for k, v in NP_TO_ELEM.items()}
ELEM_TO_NP[int(ShorokooTensorElementType.BFloat16)] = np.dtype(np.uint16)   # raw bf16 bit patterns

STATUS_NAMES = {1: "invalid argument", 2: "unsupported", 3: "shape error", 4: "CUDA error", 5: "out of memory",
                6: "internal error"}


class ShorokooB200Error(Exception):
    status: int = 0


class B200ArgumentError(ShorokooB200Error, ValueError):
    pass


class B200NotSupportedError(ShorokooB200Error, NotImplementedError):
    pass


class B200InvalidOperationError(ShorokooB200Error, RuntimeError):
    pass


class B200OutOfMemoryError(ShorokooB200Error, MemoryError):
    pass


def _check(status: int) -> None:
    if status == 0:
        return
    msg = _native.lib().sb_last_error().decode("utf-8", "replace")
    cls = {1: B200ArgumentError, 2: B200NotSupportedError, 3: B200ArgumentError, 5: B200OutOfMemoryError}.get(
        status, B200InvalidOperationError)
    err = cls(f"{STATUS_NAMES.get(status, 'error')}: {msg}")
    err.status = status
    raise err


def _shape_arr(shape: Sequence[int]):
    arr = (C.c_int64 * max(len(shape), 1))(*[int(d) for d in shape])
    return arr, len(shape)


class B200TensorValue:
    """IShorokooTensorValue over a library-owned host value (OrtTensorValue.cs:11-56)."""

    def __init__(self, handle: int):
        self._h = C.c_void_p(handle)

    # -- IShorokooTensorValue ---------------------------------------------------------------
    @property
    def ValueType(self) -> ShorokooOnnxValueType:
        return ShorokooOnnxValueType(_native.lib().sb_value_type(self._h))

    @property
    def ElementType(self) -> ShorokooTensorElementType:
        return ShorokooTensorElementType(_native.lib().sb_value_elem_type(self._h))

    @property
    def Shape(self) -> List[int]:
        L = _native.lib()
        r = L.sb_value_rank(self._h)
        p = L.sb_value_shape(self._h)
        return [int(p[i]) for i in range(r)]

    def _array(self, writable: bool) -> np.ndarray:
        L = _native.lib()
        et = int(self.ElementType)
        if et == ShorokooTensorElementType.String:
            raise B200ArgumentError("string tensor: use GetStringTensorData")
        dt = ELEM_TO_NP[et]
        n = L.sb_value_nbytes(self._h)
        shape = self.Shape
        if n == 0:
            return np.zeros(shape, dt)
        addr = L.sb_value_data(self._h)
        if not addr:
            raise B200InvalidOperationError(L.sb_last_error().decode())
        buf = (C.c_uint8 * n).from_address(addr)
        a = np.frombuffer(buf, dtype=dt).reshape(shape)
        if not writable:
            a.flags.writeable = False
        return a

    def GetTensorDataAsSpan(self) -> np.ndarray:
        """Read-only numpy view of the host data (valid while this value is alive)."""
        return self._array(False)

    def GetTensorMutableDataAsSpan(self) -> np.ndarray:
        return self._array(True)

    def GetStringTensorData(self) -> List[str]:
        L = _native.lib()
        return [L.sb_value_string_at(self._h, i).decode() for i in range(L.sb_value_string_count(self._h))]

    def GetValueCount(self) -> int:
        return _native.lib().sb_value_count(self._h)

    def GetValue(self, index: int) -> "B200TensorValue":
        out = C.c_void_p()
        _check(_native.lib().sb_value_at(self._h, index, C.byref(out)))
        return B200TensorValue(out.value)

    def GetSequenceElementType(self) -> ShorokooTensorElementType:
        return ShorokooTensorElementType(_native.lib().sb_value_sequence_elem_type(self._h))

    def Dispose(self) -> None:
        if self._h:
            _native.lib().sb_value_release(self._h)
            self._h = C.c_void_p()

    @property
    def DevicePointer(self):
        """(device address, device) of a device-resident value, (None, -1) for host values."""
        p, d = C.c_void_p(), C.c_int32()
        _check(_native.lib().sb_value_device_ptr(self._h, C.byref(p), C.byref(d)))
        return p.value, d.value

    # -- conveniences -----------------------------------------------------------------------
    def numpy(self) -> np.ndarray:
        return self._array(False).copy()

    def __del__(self):
        try:
            self.Dispose()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.Dispose()


class B200InferenceSession:
    """IShorokooInferenceSession (OrtInferenceSession.cs:6-39)."""

    def __init__(self, handle: int):
        self._h = C.c_void_p(handle)
        L = _native.lib()
        self._inputs = [L.sb_session_input_name(self._h, i).decode() for i in range(L.sb_session_input_count(self._h))]
        self._outputs = [L.sb_session_output_name(self._h, i).decode() for i in range(L.sb_session_output_count(self._h))]

    @property
    def InputNames(self) -> List[str]:
        return list(self._inputs)

    @property
    def OutputNames(self) -> List[str]:
        return list(self._outputs)

    def _marshal_inputs(self, inputs: Mapping[str, B200TensorValue]):
        names = list(inputs.keys())
        n = len(names)
        carr = (C.c_char_p * max(n, 1))(*[s.encode() for s in names])
        varr = (C.c_void_p * max(n, 1))(*[inputs[s]._h.value for s in names])
        return n, carr, varr

    def Run(self, inputs: Mapping[str, B200TensorValue], outputNames: Optional[Sequence[str]] = None
            ) -> List[B200TensorValue]:
        outs = list(outputNames) if outputNames is not None else self.OutputNames
        n, carr, varr = self._marshal_inputs(inputs)
        m = len(outs)
        onames = (C.c_char_p * max(m, 1))(*[s.encode() for s in outs])
        ovals = (C.c_void_p * max(m, 1))()
        _check(_native.lib().sb_session_run(self._h, n, carr, varr, m, onames, ovals))
        return [B200TensorValue(ovals[i]) for i in range(m)]

    def RunOnDevice(self, inputs: Mapping[str, B200TensorValue], outputNames: Optional[Sequence[str]] = None
                    ) -> List[B200TensorValue]:
        """Run whose outputs stay in device memory (sb_session_run_device): for chaining into another
        Run without host copies; reading a value's data copies it to the host on first use. No
        counterpart in the reference interface."""
        outs = list(outputNames) if outputNames is not None else self.OutputNames
        n, carr, varr = self._marshal_inputs(inputs)
        m = len(outs)
        onames = (C.c_char_p * max(m, 1))(*[s.encode() for s in outs])
        ovals = (C.c_void_p * max(m, 1))()
        _check(_native.lib().sb_session_run_device(self._h, n, carr, varr, m, onames, ovals))
        return [B200TensorValue(ovals[i]) for i in range(m)]

    # -- measurement (no counterpart in the reference interface) --------------------------------
    def time_device(self, inputs: Mapping[str, B200TensorValue], warmup: int = 3, iters: int = 10) -> List[float]:
        n, carr, varr = self._marshal_inputs(inputs)
        ms = (C.c_double * 64)()
        nd = C.c_int32()
        _check(_native.lib().sb_session_time_device(self._h, n, carr, varr, warmup, iters, ms, 64, C.byref(nd)))
        return [ms[i] for i in range(nd.value)]

    def profile(self, inputs: Mapping[str, B200TensorValue], iters: int = 5):
        n, carr, varr = self._marshal_inputs(inputs)
        cap = 8192
        kinds = (C.c_char_p * cap)()
        ms = (C.c_double * cap)()
        ns = C.c_int32()
        _check(_native.lib().sb_session_profile(self._h, n, carr, varr, iters, kinds, ms, cap, C.byref(ns)))
        return [(kinds[i].decode(), ms[i]) for i in range(min(ns.value, cap))]

    def stats(self, inputs: Mapping[str, B200TensorValue]) -> Dict[str, float]:
        n, carr, varr = self._marshal_inputs(inputs)
        la, tc, db = C.c_int64(), C.c_int64(), C.c_int64()
        macs = C.c_double()
        dev = C.c_int32()
        _check(_native.lib().sb_session_stats(self._h, n, carr, varr, C.byref(la), C.byref(tc), C.byref(macs),
                                              C.byref(db), C.byref(dev)))
        return {"launches": la.value, "tc_launches": tc.value, "macs": macs.value, "device_bytes": db.value,
                "devices": dev.value}

    def transfer_bytes(self, inputs: Mapping[str, B200TensorValue]):
        """(host->device, device->host) bytes a Run of these inputs copies."""
        n, carr, varr = self._marshal_inputs(inputs)
        h, d = C.c_int64(), C.c_int64()
        _check(_native.lib().sb_session_transfer_bytes(self._h, n, carr, varr, C.byref(h), C.byref(d)))
        return h.value, d.value

    def Dispose(self) -> None:
        if self._h:
            _native.lib().sb_session_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.Dispose()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.Dispose()


class B200InferenceSessionFactory:
    """IShorokooInferenceSessionFactory for the Shorokoo.LinuxGPU slot (OrtSessionFactory.cs:14-106).

    ``num_devices`` = 0 uses SHOROKOO_B200_DEVICES or every visible GPU; batches shard across them.
    ``precision``: "bf16" (throughput mode), "tf32" (fp32 operands read as TF32), "tf32x3"
    (error-compensated TF32, close to fp32) or None for SHOROKOO_B200_PRECISION (default bf16)."""

    _PRECISIONS = {None: -1, "bf16": 0, "tf32": 1, "tf32x3": 2}

    def __init__(self, num_devices: int = 0, first_device: int = 0, precision: Optional[str] = None):
        if precision not in self._PRECISIONS:
            raise ValueError(f"precision must be 'bf16', 'tf32', 'tf32x3' or None, got {precision!r}")
        self.num_devices = num_devices
        self.first_device = first_device
        self.precision = precision

    @staticmethod
    def ClearSessionCache() -> int:
        """Releases the sessions the library keeps cached by model content (so a new session on the
        same model bytes reuses its plans); returns how many were cached."""
        return int(_native.lib().sb_session_cache_clear())

    def CreateSession(self, modelBytes: bytes,
                      graphOptimization: ShorokooGraphOptimization = ShorokooGraphOptimization.EnableAll,
                      logSeverity: ShorokooLogSeverity = ShorokooLogSeverity.Fatal) -> B200InferenceSession:
        out = C.c_void_p()
        b = bytes(modelBytes)
        _check(_native.lib().sb_session_create_ex(b, len(b), int(graphOptimization), int(logSeverity),
                                                  self.num_devices, self.first_device,
                                                  self._PRECISIONS[self.precision], C.byref(out)))
        return B200InferenceSession(out.value)

    def CreateTensor(self, data, shape: Optional[Sequence[int]] = None) -> B200TensorValue:
        """CreateTensor<T>(T[] data, long[] shape): copies the array into library host memory."""
        a = np.asarray(data)
        if not a.flags.c_contiguous:
            a = a.copy(order="C")   # (np.ascontiguousarray would turn 0-d scalars into 1-d arrays)
        if a.dtype not in NP_TO_ELEM:
            raise B200NotSupportedError(f"element type {a.dtype} is not supported")
        shp = list(a.shape) if shape is None else [int(s) for s in shape]
        if int(np.prod(shp, dtype=np.int64)) != a.size:
            raise B200ArgumentError(f"shape {shp} does not match {a.size} elements")
        return self._create(int(NP_TO_ELEM[a.dtype]), shp, a.ctypes.data, a.nbytes)

    def WrapTensor(self, data) -> B200TensorValue:
        """A tensor value over the caller's C-contiguous array without a copy (sb_value_wrap_tensor),
        the way the reference's CreateTensor<T> aliases a managed array (OrtSessionFactory.cs:56).
        The array must not change while the value is alive; the value keeps a reference to it."""
        a = np.asarray(data)
        if not a.flags.c_contiguous:
            raise B200ArgumentError("WrapTensor needs a C-contiguous array")
        if a.dtype not in NP_TO_ELEM:
            raise B200NotSupportedError(f"element type {a.dtype} is not supported")
        arr, r = _shape_arr(list(a.shape))
        out = C.c_void_p()
        _check(_native.lib().sb_value_wrap_tensor(int(NP_TO_ELEM[a.dtype]), arr, r, C.c_void_p(a.ctypes.data),
                                                  a.nbytes, C.byref(out)))
        v = B200TensorValue(out.value)
        v._keep = a   # the wrapped memory lives as long as the value
        return v

    def CreateTensorFromRawBytes(self, elementType: ShorokooTensorElementType, data: bytes,
                                 shape: Sequence[int]) -> B200TensorValue:
        if int(elementType) == ShorokooTensorElementType.String:
            raise B200NotSupportedError(
                "String tensors are variable-length and not byte-stride; use CreateStringTensor instead.")
        b = bytes(data)
        buf = C.create_string_buffer(b, len(b))
        return self._create(int(elementType), list(shape), C.addressof(buf), len(b))

    def _create(self, et: int, shape, ptr: int, nbytes: int) -> B200TensorValue:
        arr, r = _shape_arr(shape)
        out = C.c_void_p()
        _check(_native.lib().sb_value_create_tensor(et, arr, r, C.c_void_p(ptr), nbytes, C.byref(out)))
        return B200TensorValue(out.value)

    def CreateStringTensor(self, data: Sequence[str], shape: Sequence[int]) -> B200TensorValue:
        arr, r = _shape_arr(shape)
        strs = (C.c_char_p * max(len(data), 1))(*[s.encode() for s in data])
        out = C.c_void_p()
        _check(_native.lib().sb_value_create_string_tensor(strs, len(data), arr, r, C.byref(out)))
        return B200TensorValue(out.value)

    def CreateSequence(self, values: Sequence[B200TensorValue]) -> B200TensorValue:
        arr = (C.c_void_p * max(len(values), 1))(*[v._h.value for v in values])
        out = C.c_void_p()
        _check(_native.lib().sb_value_create_sequence(arr, len(values), C.byref(out)))
        return B200TensorValue(out.value)

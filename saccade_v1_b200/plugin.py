"""ctypes front end of the plugin surface (include/sacc_scan_plugin.h).

Mirrors the reference's TensorRT plugins (src/scan_trt_plugin.cpp) without
TensorRT: `ScanPlugin.create(name, version, fields)` behaves like the
registered IPluginCreatorV3One, and the methods like the IPluginV3 ones, with
the reference's messages.  Errors raise PluginError (the reference returns
-1 and reports the message to TensorRT's error recorder).
"""
from __future__ import annotations

import ctypes

from . import _lib

FIELD_INT32, FIELD_OTHER = 1, 0
TENSOR_FLOAT, TENSOR_HALF, TENSOR_INT32, TENSOR_BF16, TENSOR_OTHER = 0, 1, 3, 7, 99
FORMAT_LINEAR, FORMAT_OTHER = 0, 99
SCAN, EXPAND, MERGE = ("SelectiveScan", "2"), ("CrossScanExpand", "1"), ("CrossScanMerge", "1")
SCAN_F16 = ("SelectiveScan", "3")  # FP16 u, delta, B, C, y; FP32 A, D
BLOCK = ("MambaBlock", "1")         # the head Mamba block; fields dt_rank, residual
LEVEL = ("CrossScanMambaBlock", "1")  # a head level: expand -> block -> merge on FP32 maps; fields dt_rank, residual


class PluginError(ValueError):
    pass


class Field(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("data", ctypes.c_void_p), ("type", ctypes.c_int32), ("length", ctypes.c_int32)]


class TensorDesc(ctypes.Structure):
    _fields_ = [("nb_dims", ctypes.c_int32), ("dims", ctypes.c_int64 * 8), ("type", ctypes.c_int32),
                ("format", ctypes.c_int32)]

    @staticmethod
    def of(dims, type=TENSOR_FLOAT, format=FORMAT_LINEAR):
        d = TensorDesc()
        d.nb_dims = len(dims)
        for i, v in enumerate(dims):
            d.dims[i] = v
        d.type, d.format = type, format
        return d

    def shape(self):
        return tuple(self.dims[i] for i in range(self.nb_dims))


_bound = False


def _lib_plugin():
    global _bound
    L = _lib.load()
    if not _bound:
        vp, i, i32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int32
        P = ctypes.c_void_p
        L.sacc_plugin_create.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(Field), i32, ctypes.POINTER(P)]
        L.sacc_plugin_create.restype = i
        L.sacc_plugin_destroy.argtypes = [P]
        L.sacc_plugin_destroy.restype = None
        L.sacc_plugin_clone.argtypes = [P, ctypes.POINTER(P)]
        L.sacc_plugin_clone.restype = i
        L.sacc_plugin_fields.argtypes = [P] + [ctypes.POINTER(i32)] * 3
        L.sacc_plugin_fields.restype = i
        L.sacc_plugin_output_types.argtypes = [P, ctypes.POINTER(i32), i32, ctypes.POINTER(i32), i32]
        L.sacc_plugin_output_types.restype = i
        L.sacc_plugin_output_shapes.argtypes = [P, ctypes.POINTER(TensorDesc), i32, ctypes.POINTER(TensorDesc), i32]
        L.sacc_plugin_output_shapes.restype = i
        L.sacc_plugin_supports_format.argtypes = [P, i32, ctypes.POINTER(TensorDesc), i32, i32]
        L.sacc_plugin_supports_format.restype = i
        L.sacc_plugin_workspace_size.argtypes = [P]
        L.sacc_plugin_workspace_size.restype = ctypes.c_size_t
        L.sacc_plugin_bind.argtypes = [P]
        L.sacc_plugin_bind.restype = i
        L.sacc_plugin_enqueue.argtypes = [P, ctypes.POINTER(TensorDesc), ctypes.POINTER(TensorDesc), ctypes.POINTER(vp),
                                          ctypes.POINTER(vp), vp]
        L.sacc_plugin_enqueue.restype = i
        L.sacc_plugin_workspace_bytes.argtypes = [P, ctypes.POINTER(TensorDesc), i32, ctypes.POINTER(ctypes.c_size_t)]
        L.sacc_plugin_workspace_bytes.restype = i
        L.sacc_plugin_block_fields.argtypes = [P, ctypes.POINTER(i32), ctypes.POINTER(i32)]
        L.sacc_plugin_block_fields.restype = i
        L.sacc_plugin_enqueue_ws.argtypes = [P, ctypes.POINTER(TensorDesc), ctypes.POINTER(TensorDesc), ctypes.POINTER(vp),
                                             ctypes.POINTER(vp), vp, ctypes.c_size_t, vp]
        L.sacc_plugin_enqueue_ws.restype = i
        L.sacc_plugin_last_error.argtypes = []
        L.sacc_plugin_last_error.restype = ctypes.c_char_p
        _bound = True
    return L


def _check(rc):
    if rc != _lib.SACC_OK:
        raise PluginError(_lib_plugin().sacc_plugin_last_error().decode())


def int_field(name: str, value: int) -> tuple:
    return (name, int(value))


class ScanPlugin:
    """One plugin instance (creator-made), e.g. ScanPlugin.create(*SCAN, [("has_d", 1)])."""

    def __init__(self, handle):
        self._h = handle

    @classmethod
    def create(cls, name: str, version: str, fields=()):
        """fields: (name, int value) pairs, or raw (name, data_ptr_or_None, type, length) tuples."""
        arr = (Field * max(1, len(fields)))()
        keep = []
        for i, f in enumerate(fields):
            if len(f) == 2:
                v = ctypes.c_int32(f[1])
                keep.append(v)
                arr[i] = Field(f[0].encode() if f[0] is not None else None, ctypes.cast(ctypes.pointer(v), ctypes.c_void_p),
                               FIELD_INT32, 1)
            else:
                n, data, t, length = f
                if isinstance(data, int):
                    v = ctypes.c_int32(data)
                    keep.append(v)
                    data = ctypes.cast(ctypes.pointer(v), ctypes.c_void_p)
                arr[i] = Field(n.encode() if n is not None else None, data, t, length)
        h = ctypes.c_void_p()
        _check(_lib_plugin().sacc_plugin_create(name.encode(), version.encode(), arr, len(fields), ctypes.byref(h)))
        return cls(h)

    def __del__(self):
        if getattr(self, "_h", None):
            _lib_plugin().sacc_plugin_destroy(self._h)
            self._h = None

    def clone(self) -> "ScanPlugin":
        h = ctypes.c_void_p()
        _check(_lib_plugin().sacc_plugin_clone(self._h, ctypes.byref(h)))
        return ScanPlugin(h)

    def fields(self):
        v = [ctypes.c_int32() for _ in range(3)]
        _check(_lib_plugin().sacc_plugin_fields(self._h, *[ctypes.byref(x) for x in v]))
        return {k: x.value for k, x in zip(("has_d", "height", "width"), v) if x.value >= 0}

    def output_types(self, in_types, nb_out=2):
        arr = (ctypes.c_int32 * len(in_types))(*in_types)
        out = (ctypes.c_int32 * nb_out)()
        _check(_lib_plugin().sacc_plugin_output_types(self._h, arr, len(in_types), out, nb_out))
        return list(out)

    def output_shapes(self, in_dims, nb_out=2, in_types=None):
        types = in_types or [TENSOR_FLOAT] * len(in_dims)
        ins = (TensorDesc * len(in_dims))(*[TensorDesc.of(d, t) for d, t in zip(in_dims, types)])
        outs = (TensorDesc * nb_out)()
        _check(_lib_plugin().sacc_plugin_output_shapes(self._h, ins, len(in_dims), outs, nb_out))
        return [outs[k].shape() for k in range(nb_out)]

    def block_fields(self):
        v = [ctypes.c_int32() for _ in range(2)]
        _check(_lib_plugin().sacc_plugin_block_fields(self._h, *[ctypes.byref(x) for x in v]))
        return {"dt_rank": v[0].value, "residual": v[1].value}

    def workspace_bytes(self, in_descs) -> int:
        arr = (TensorDesc * len(in_descs))(*in_descs)
        n = ctypes.c_size_t()
        _check(_lib_plugin().sacc_plugin_workspace_bytes(self._h, arr, len(in_descs), ctypes.byref(n)))
        return n.value

    def supports_format(self, pos, descs, nb_in):
        arr = (TensorDesc * len(descs))(*descs)
        return bool(_lib_plugin().sacc_plugin_supports_format(self._h, pos, arr, nb_in, len(descs) - nb_in))

    def workspace_size(self) -> int:
        return _lib_plugin().sacc_plugin_workspace_size(self._h)

    def bind(self):
        _check(_lib_plugin().sacc_plugin_bind(self._h))

    def enqueue(self, in_descs, out_descs, inputs, outputs, stream, workspace=None, workspace_bytes=0):
        ind = (TensorDesc * len(in_descs))(*in_descs)
        outd = (TensorDesc * len(out_descs))(*out_descs)
        inp = (ctypes.c_void_p * len(inputs))(*inputs)
        outp = (ctypes.c_void_p * len(outputs))(*outputs)
        h = stream if isinstance(stream, int) else stream.cuda_stream
        if workspace is None:
            _check(_lib_plugin().sacc_plugin_enqueue(self._h, ind, outd, inp, outp, h))
        else:
            _check(_lib_plugin().sacc_plugin_enqueue_ws(self._h, ind, outd, inp, outp, workspace, workspace_bytes, h))

"""GGUF model files for the expert path (libtsb_moe.so's tsb_gguf_*): metadata, tensors, and a layer's experts
repacked into the native expert blobs (the reference's blob build, src/qwen35/q36_engine.cu:1144-1167, 1196-1200),
moved to the device for MoELayer / PrefillLayer / DecodeStack."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import ExpertLayout, GgufTensorInfo, _check, lib


TensorInfo = GgufTensorInfo


class GGUFFile:
    """A memory-mapped GGUF file (read-only)."""

    def __init__(self, path: str):
        self.L = lib()
        self.h = C.c_void_p()
        _check(self.L.tsb_gguf_open(path.encode(), C.byref(self.h)), "gguf_open")

    def close(self):
        if self.h:
            self.L.tsb_gguf_close(self.h)
            self.h = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def tensor_names(self) -> list[str]:
        buf = C.create_string_buffer(512)
        out = []
        for i in range(self.L.tsb_gguf_tensor_count(self.h)):
            _check(self.L.tsb_gguf_tensor_name(self.h, i, buf, 512), "gguf_tensor_name")
            out.append(buf.value.decode())
        return out

    def tensor(self, name: str) -> TensorInfo:
        t = TensorInfo()
        _check(self.L.tsb_gguf_tensor(self.h, name.encode(), C.byref(t)), "gguf_tensor")
        return t

    def tensor_bytes(self, name: str) -> np.ndarray:
        """The tensor's raw bytes (a copy out of the mapping)."""
        t = self.tensor(name)
        return np.ctypeslib.as_array((C.c_uint8 * t.bytes).from_address(t.data)).copy()

    def tensor_f32(self, name: str) -> np.ndarray:
        """An F32 tensor as numpy, shape in row-major order (the file's ne reversed)."""
        t = self.tensor(name)
        if t.type != 0:
            raise ValueError(f"{name}: type {t.type}, not F32")
        shape = tuple(int(t.ne[d]) for d in reversed(range(t.n_dims)))
        return self.tensor_bytes(name).view(np.float32).reshape(shape)

    def kv_int(self, key: str) -> int:
        v = C.c_int64()
        _check(self.L.tsb_gguf_kv_int(self.h, key.encode(), C.byref(v)), "gguf_kv_int")
        return v.value

    def kv_float(self, key: str) -> float:
        v = C.c_double()
        _check(self.L.tsb_gguf_kv_float(self.h, key.encode(), C.byref(v)), "gguf_kv_float")
        return v.value

    def kv_str(self, key: str) -> str:
        buf = C.create_string_buffer(4096)
        _check(self.L.tsb_gguf_kv_str(self.h, key.encode(), buf, 4096), "gguf_kv_str")
        return buf.value.decode()

    def expert_layer(self, prefix: str):
        """(layout, blob stride, expert count) of the layer whose tensor names start with prefix ("blk.3.")."""
        L = ExpertLayout()
        stride, n = C.c_uint64(), C.c_int32()
        _check(self.L.tsb_gguf_expert_layer(self.h, prefix.encode(), C.byref(L), C.byref(stride), C.byref(n)),
               "gguf_expert_layer")
        return L, int(stride.value), int(n.value)

    def repack_experts(self, prefix: str, first: int = 0, count: int | None = None) -> np.ndarray:
        """Experts [first, first + count) as native expert blobs: uint8 [count, stride] (host)."""
        L, stride, n = self.expert_layer(prefix)
        count = n - first if count is None else count
        out = np.empty((count, stride), np.uint8)
        _check(self.L.tsb_gguf_repack_experts(self.h, prefix.encode(), first, count, out.ctypes.data_as(C.c_void_p),
                                              out.nbytes), "gguf_repack_experts")
        return out

    def device_layer(self, prefix: str, device, first: int = 0, count: int | None = None):
        """The layer's expert blobs [count, stride] (device), its router (fp32 [E (+1), n_embd], with the shared-expert
        gate row appended as the reference's engine does, q36_engine.cu:1139-1142, when the file has one) and its
        layout."""
        import torch
        L, stride, n = self.expert_layer(prefix)
        blobs = torch.from_numpy(self.repack_experts(prefix, first, count)).to(device)
        router = self.tensor_f32(prefix + "ffn_gate_inp.weight")
        names = set(self.tensor_names())
        if prefix + "ffn_gate_inp_shexp.weight" in names:
            router = np.concatenate([router, self.tensor_f32(prefix + "ffn_gate_inp_shexp.weight").reshape(1, -1)])
        return blobs, torch.from_numpy(np.ascontiguousarray(router)).to(device), L

"""ctypes face of oracle/_ref/libtsb_ref_gpu.so: TinyStrata's own decode CUDA kernels compiled for sm_100a from the
reference sources (oracle/Makefile `ref-gpu`, oracle/ref_gpu_shim.cu).  GPU parity tests run them beside the product
kernels on the same device buffers.  Test infrastructure only."""
import ctypes as C
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PATH = os.path.join(ROOT, "oracle", "_ref", "libtsb_ref_gpu.so")
_lib = None
_p, _i64, _i32 = C.c_void_p, C.c_int64, C.c_int32


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(PATH):
            return None
        L = C.CDLL(PATH)
        L.ref_native_router_topk.restype = C.c_int
        L.ref_native_router_topk.argtypes = [_p, _p, _p, C.c_int, C.c_int, C.c_int, _p]
        L.ref_quantize_q8_1_rows.argtypes = [_p, _i64, _i64, _p, _p]
        L.ref_iq_mmvq.argtypes = [C.c_int, _p, _p, _p, C.c_int, C.c_int, C.c_int, _p]
        L.ref_native_expert_bytes.restype = C.c_size_t
        L.ref_native_expert_bytes.argtypes = [C.c_int, C.c_int, _i64, _i64]
        L.ref_native_expert_scratch_bytes.restype = C.c_size_t
        L.ref_native_expert_scratch_bytes.argtypes = [_i64, _i64]
        L.ref_native_expert_grouped.argtypes = [C.c_int, C.c_int, _i64, _i64, _p, _p, _p, _p, _p, _i64, _i64, _p, _p,
                                                _p, _p]
        L.ref_moe_out_small.argtypes = [_p, _p, _p, _p, C.c_int, _p, _p, C.c_int, _p, _p, C.c_int, C.c_float, _p,
                                        C.c_int, _p]
        L.ref_last_cuda_error.restype = C.c_int
        L.ref_route_rows.restype = C.c_int
        L.ref_route_rows.argtypes = [_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, _p, _p, C.c_int, C.c_float, _p,
                                     _p, _p]
        L.ref_moe_sum.argtypes = [_p, _p, _p, C.c_int, C.c_int, C.c_int, _p]
        L.ref_add_scaled.restype = C.c_int
        L.ref_add_scaled.argtypes = [_p, _p, _p, C.c_int, C.c_int, _p]
        _lib = L
    return _lib


def ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def stream():
    import torch
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)

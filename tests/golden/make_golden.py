"""Generate tests/golden/ref_cpu_rows.npz: outputs of TinyStrata's OWN compiled CPU expert kernels (oracle/_ref,
built from the reference sources by oracle/Makefile) on small seeded inputs.

Per case: weight rows (raw GGUF blocks), fp32 activations, the reference's Q8_K image of them (q8k_quant_avx2,
src/kernels/cpu/iq_avx2.cpp:393) and its row products (iq512_rows / iq256_rows for IQ3_XXS and IQ3_S,
src/kernels/cpu/iq_avx512.cpp:245-262; kq256_rows for Q4_K, src/kernels/cpu/kq_avx2.cpp:216) and the gate/up SwiGLU
rows (iq512_gu_rows / kq256_gu_rows).  The oracle's codebook decode is pinned against these.

Run (needs oracle/_ref built, i.e. the reference tree): python tests/golden/make_golden.py
"""
from __future__ import annotations

import ctypes as C
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from tinystrata_b200 import synth  # noqa: E402

Q8K_BYTES = 4 + 256 + 32   # float d, 256 int8, 16 int16 bsums


def ref_rows(R, t, W, n, x_q8k, rows):
    nt = x_q8k.shape[0]
    out = np.zeros((nt, rows), np.float32)
    acts = (C.c_void_p * nt)(*[x_q8k[i].ctypes.data for i in range(nt)])
    outs = (C.c_void_p * nt)(*[out[i].ctypes.data for i in range(nt)])
    rc = R.ref_rows(t, W.ctypes.data_as(C.c_void_p), O.row_bytes(t, n), n, acts, nt, outs, 0, rows)
    assert rc == 0, rc
    return out


def ref_gu(R, t, blob, n, x_q8k, n_ff):
    nt = x_q8k.shape[0]
    ff = np.zeros((nt, n_ff), np.float32)
    acts = (C.c_void_p * nt)(*[x_q8k[i].ctypes.data for i in range(nt)])
    outs = (C.c_void_p * nt)(*[ff[i].ctypes.data for i in range(nt)])
    gu_row = O.row_bytes(t, n)
    rc = R.ref_gu_rows(t, blob.ctypes.data_as(C.c_void_p), gu_row, gu_row * n_ff, n, acts, nt, outs, 0, n_ff)
    assert rc == 0, rc
    return ff


def q8k(R, x):
    y = np.zeros((x.shape[0], x.shape[1] // 256 * Q8K_BYTES), np.uint8)
    for i in range(x.shape[0]):
        R.ref_q8k_quant(x[i].ctypes.data_as(C.c_void_p), y[i].ctypes.data_as(C.c_void_p), x.shape[1])
    return y


def main():
    R = O.ref_cpu()
    if R is None:
        raise SystemExit("oracle/_ref/libtsb_ref_cpu.so is not built (make -C oracle ref)")
    rng = np.random.default_rng(12345)
    cases = {}
    for t, sd in ((synth.T_IQ3_XXS, 0.02), (synth.T_IQ3_S, 0.02), (synth.T_Q4_K, 0.01)):
        n, rows, nt = 512, 8, 3
        W = synth.gen_matrix(rng, t, rows, n, sd)
        x = rng.normal(0, 1, size=(nt, n)).astype(np.float32)
        xk = q8k(R, x)
        y = ref_rows(R, t, W, n, xk, rows)
        n_ff = 4
        blob = synth.gen_matrix(rng, t, 2 * n_ff, n, sd)
        ff = ref_gu(R, t, blob, n, xk, n_ff)
        cases[f"t{t}_W"] = W
        cases[f"t{t}_x"] = x
        cases[f"t{t}_xq8k"] = xk
        cases[f"t{t}_y"] = y
        cases[f"t{t}_blob"] = blob
        cases[f"t{t}_ff"] = ff
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ref_cpu_rows.npz")
    np.savez_compressed(path, isa=np.int32(R.ref_cpu_isa()), **cases)
    print(path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()

"""The C ABI surface, without a GPU: libtsb_moe.so loads and exports every function include/tsb_moe.h declares, the
host-only calls answer as the reference's (the Qwen expert blob is 1,204,224 bytes), errors come back as status codes
with a message, and the product path fails loudly when the library is missing (no CPU fallback)."""
import ctypes as C
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", f) for f in sorted(os.listdir(os.path.join(ROOT, "include"))) if f.endswith(".h")]


def declared():
    names = []
    for h in HEADERS:
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"^[A-Za-z_][\w \*]*?\b(tsb_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    from tinystrata_b200 import build
    build.build()
    import tinystrata_b200 as T
    return T.lib()


def test_header_declares_functions():
    names = declared()
    assert "tsb_native_expert_grouped" in names and "tsb_native_router_topk" in names
    assert len(names) >= 15


def test_every_declared_symbol_is_exported(lib):
    from tinystrata_b200 import LIB_PATH
    out = subprocess.run(["nm", "-D", "--defined-only", LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (tsb_\w+)", out))
    missing = [n for n in declared() if n not in exported]
    assert not missing, missing


def test_python_mirror_binds_every_symbol(lib):
    import tinystrata_b200 as T
    assert sorted(T.SIGNATURES) == declared()


def test_host_calls(lib):
    import tinystrata_b200 as T
    assert lib.tsb_moe_abi_version() == 1
    L = T.native_expert_layout(T.T_IQ3_XXS, T.T_IQ3_XXS, 2048, 512)
    assert (L.gu_row, L.d_row, L.up_off, L.down_off, L.bytes) == (784, 196, 401408, 802816, 1204224)
    L2 = T.native_expert_layout(T.T_Q4_0, T.T_Q4_0, 2816, 704)
    assert (L2.gu_row, L2.d_row) == (1584, 396)
    assert T.row_bytes(T.T_Q6_K, 1792) == 7 * 210 and T.row_bytes(T.T_Q4_K, 2048) == 8 * 144
    assert T.native_expert_supported(T.T_IQ3_XXS, T.T_IQ3_XXS, 2048, 512)
    assert T.native_expert_supported(T.T_Q4_K, T.T_Q6_K, 2048, 1792)
    assert T.native_expert_supported(T.T_IQ3_XXS, T.T_IQ3_S, 2048, 512)
    assert not T.native_expert_supported(99, T.T_IQ3_XXS, 2048, 512)
    assert T.native_expert_scratch_bytes(8, 512) == 8 * 512 * 4


def test_errors_are_status_codes(lib):
    import tinystrata_b200 as T
    L = T.ExpertLayout()
    rc = lib.tsb_native_expert_layout(99, 18, 2048, 512, C.byref(L))
    assert rc == -2 and "99" in T.last_error()
    assert lib.tsb_row_bytes(18, 100) == -1
    with pytest.raises(T.TsbError):
        T.native_expert_layout(18, 18, 2048, 100)


def test_missing_library_fails_loudly(monkeypatch):
    import tinystrata_b200 as T
    monkeypatch.setattr(T, "_lib", None)
    monkeypatch.setattr(T, "LIB_PATH", "/nonexistent/libtsb_moe.so")
    with pytest.raises(T.TsbError, match="no CPU fallback"):
        T.lib()

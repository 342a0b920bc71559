"""The reference-facing C++ shim (shim/tsb_shim.cpp): compiled against the reference's own headers (every signature
of the engines' call sites pinned by the compiler), linked over libtsb_moe.so, and its host-side queries -- expert blob
layouts, row sizes, supported formats, MMQ activation sizes and fits, the router's argument error -- checked on CPU
against the synthetic layouts, the reference's own layout functions (oracle/_ref) and the C ABI.  Skipped where the
reference tree is absent (the GPU box)."""
import json
import os
import subprocess

import pytest

from oracle.oracle import reference_dir
from tinystrata_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def shim_lines():
    ref = reference_dir()
    if not os.path.isdir(os.path.join(ref, "include", "strata")):
        pytest.skip("the reference tree (its headers) is not here")
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "shim"), f"REF={ref}"], check=True)
    out = subprocess.run([os.path.join(ROOT, "shim", "_build", "shim_check")], check=True, capture_output=True,
                         text=True).stdout
    return [json.loads(line) for line in out.splitlines() if line.strip()]


def test_shim_layouts_match_the_synthetic_blobs_and_the_reference(shim_lines):
    layouts = [r for r in shim_lines if r["kind"] == "layout"]
    assert len(layouts) == 6
    from tests import refgpu
    R = refgpu.lib()
    for r in layouts:
        cfg = dict(gu_type=r["gu"], d_type=r["d"], n_embd=r["n_embd"], n_ff=r["n_ff"])
        want = synth.blob_layout(cfg)
        for k in ("gu_row", "d_row", "up_off", "down_off", "bytes"):
            assert r[k] == want[k], (r, k, want[k])
        assert r["supported"] == 1
        if R is not None:   # the reference's own native_expert_layout (iq_kernels.cu), compiled from its sources
            assert R.ref_native_expert_bytes(r["gu"], r["d"], r["n_embd"], r["n_ff"]) == r["bytes"]


def test_shim_formats_and_mmq_queries(shim_lines):
    import tinystrata_b200 as T
    types = {r["t"]: r for r in shim_lines if r["kind"] == "type"}
    for t in (2, 8, 12, 14, 18, 21):
        assert types[t]["iq_supported"] == 1 and types[t]["mmq_supported"] == 1
        assert types[t]["row_bytes_2048"] == synth.row_bytes(t, 2048)
    assert types[1]["iq_supported"] == 0 and types[1]["row_bytes_2048"] == 0
    m = [r for r in shim_lines if r["kind"] == "mmq"][0]
    assert m["q8_bytes"] == T.lib().tsb_mmq_act_bytes(300, 2048)
    assert m["gemma_q8_bytes"] == T.lib().tsb_mmq_act_bytes(300, 2816)
    assert m["fits"] == 1 and m["gemma_fits"] == 1
    assert m["scratch"] == T.native_expert_scratch_bytes(64, 512)
    from tests import refgpu
    if refgpu.lib() is not None:
        # the B200 kernels need less scratch than the reference's (fp32 hidden rows only): a buffer the engine sized
        # by either query serves them
        assert m["scratch"] <= refgpu.lib().ref_native_expert_scratch_bytes(64, 512)
    assert m["router_256_8"] == 1 and m["router_33_8"] == 0


def test_shim_turns_a_refused_call_into_the_reference_exception(shim_lines):
    assert [r for r in shim_lines if r["kind"] == "router_error"][0]["threw"] == 1


def test_shim_slot_products_report_their_formats(shim_lines):
    m = [r for r in shim_lines if r["kind"] == "mmvq"][0]
    assert m["ids_q4_0"] == 1 and m["ids_iq3_xxs"] == 1
    assert m["ids_q5_0"] == 0 and m["slots_q5_0"] == 0   # the reference's "no kernel for it": false, nothing launched

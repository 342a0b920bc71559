"""Host-side argument checks of the one-launch Gemma / LFM decode block and of the host-staged experts: every refusal
is decided before any CUDA call, so these run on CPU (fake, never dereferenced device addresses)."""
import ctypes as C

import numpy as np
import pytest

import tinystrata_b200 as T
from tinystrata_b200 import synth

ARG, UNSUP, ALIGN, WS = -1, -2, -4, -5
A = 1 << 20   # a 16-byte aligned fake device address


def act_call(desc, ws_bytes=1 << 30, router=A, h=A, hq=A, blobs=A, stride=3345408, sh=A, out=A, sh_out=A, ws=A):
    return T.lib().tsb_moe_decode_act(C.byref(desc), C.c_void_p(router), None, None, C.c_void_p(h), C.c_void_p(hq),
                                      C.c_void_p(blobs), stride, C.c_void_p(sh), C.c_void_p(out), 1,
                                      C.c_void_p(sh_out), None, None, C.c_void_p(ws), ws_bytes, None)


def test_decode_act_workspace_grows_with_tokens():
    sizes = [int(T.lib().tsb_moe_decode_act_workspace_bytes(C.byref(T.decode_act_desc(synth.GEMMA, t, True))))
             for t in (1, 4, 16)]
    assert 0 < sizes[0] < sizes[1] < sizes[2]
    d = T.decode_act_desc(synth.GEMMA, 1, True)
    d.struct_size = 8
    assert T.lib().tsb_moe_decode_act_workspace_bytes(C.byref(d)) == 0


def test_decode_act_refusals():
    g = T.decode_act_desc(synth.GEMMA, 1, True)
    assert act_call(g, ws_bytes=16) == WS
    bad = T.decode_act_desc(synth.GEMMA, 1, True)
    bad.struct_size = 12
    assert act_call(bad) == ARG
    assert act_call(T.decode_act_desc(synth.GEMMA, 17, True)) == UNSUP          # more than 16 tokens
    assert act_call(T.decode_act_desc(synth.QWEN, 1, True)) == UNSUP           # IQ3_XXS experts
    d = T.decode_act_desc(synth.GEMMA, 1, True)
    d.gate = 2
    assert act_call(d) == ARG
    d = T.decode_act_desc(synth.GEMMA, 1, True)
    d.n_expert = 100                                                          # not a multiple of 32
    assert act_call(d) == UNSUP
    assert act_call(g, router=0) == ARG
    assert act_call(g, sh=0) == ARG                                           # shared MLP without its blob
    assert act_call(g, h=A + 4) == ALIGN
    assert act_call(g, ws=A + 128) == ALIGN
    lfm = T.decode_act_desc(synth.LFM, 1, False)
    assert act_call(lfm, ws_bytes=16, stride=7139328, sh=0, sh_out=0) == WS    # LFM: no shared MLP needed
    assert "decode_act" in T.last_error()


def staged_call(n_ent=8, K=8, E=64, n_slots=16, stride=1204224, stage_cap=8, slot_of=A, host=A, stage=A, slots=A):
    return T.lib().tsb_moe_group_staged(C.c_void_p(A), n_ent, K, E, C.c_void_p(slot_of), n_slots, C.c_void_p(slots),
                                        C.c_void_p(host), stride, C.c_void_p(stage), stage_cap, C.c_void_p(A),
                                        C.c_void_p(A), C.c_void_p(A), C.c_void_p(A), C.c_void_p(A), None, None)


def test_group_staged_refusals():
    assert staged_call(stage_cap=7) == WS            # a step may miss min(n_ent, E) = 8 experts
    assert staged_call(stride=1204224 + 8) == ALIGN
    assert staged_call(host=A + 8) == ALIGN
    assert staged_call(slot_of=0) == ARG
    assert staged_call(n_slots=-1) == ARG
    assert staged_call(E=5000) == ARG


def test_stage_layer_and_load_refusals():
    so = np.zeros(8, np.int32)
    assert T.lib().tsb_stage_layer(so.ctypes.data, 8, 4, None, C.c_void_p(A), 64, C.c_void_p(A), 0, None) == ARG
    assert T.lib().tsb_stage_layer(so.ctypes.data, 8, 0, None, None, 64, C.c_void_p(A), 0, None) == ARG
    me, ms = np.array([3], np.int32), np.array([9], np.int32)   # slot 9 of 4
    assert T.lib().tsb_staged_load(C.c_void_p(A), C.c_void_p(A), 64, 64, me.ctypes.data, ms.ctypes.data, 1, 8, 4,
                                   None) == ARG
    assert T.lib().tsb_staged_load(C.c_void_p(A), C.c_void_p(A), 64, 128, me.ctypes.data, ms.ctypes.data, 1, 8, 4,
                                   None) == ARG             # a blob larger than its stride


@pytest.mark.parametrize("cfg", [synth.GEMMA, synth.LFM])
def test_decode_act_desc_mirrors_the_config(cfg):
    d = T.decode_act_desc(cfg, 3, bool(cfg.get("sh_n_ff")))
    assert (d.n_tok, d.n_embd, d.n_ff, d.n_expert, d.n_used) == (3, cfg["n_embd"], cfg["n_ff"], cfg["n_expert"],
                                                                 cfg["n_used"])
    assert d.sh_n_ff == (cfg.get("sh_n_ff") or 0)
    assert d.gate == (1 if cfg["router_mode"] == "sigmoid" else 0)
    assert d.struct_size == C.sizeof(T.DecodeActDesc) == 64

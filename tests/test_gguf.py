"""GGUF files (libtsb_moe.so's tsb_gguf_*): a synthetic model file written by ggml's own gguf-py writer, read back
through the library's mmap reader -- metadata of each value type, the tensor directory, F32 router tensors -- and a
layer's ffn_{gate,up,down}_exps tensors repacked into native expert blobs byte for byte equal to the blobs the
kernels take (the reference's blob build, src/qwen35/q36_engine.cu:1144-1167, 1196-1200), with the reference's
stride rule.  CPU only: nothing is launched."""
import numpy as np
import pytest

from tinystrata_b200 import synth


def _write_model(path, cfg, layers, n_expert):
    import gguf
    from gguf import GGMLQuantizationType as Q
    w = gguf.GGUFWriter(str(path), "qwen35moe")
    w.add_uint32("qwen35moe.block_count", len(layers))
    w.add_uint32("qwen35moe.expert_count", n_expert)
    w.add_float32("qwen35moe.rms_eps", 1e-6)
    w.add_string("general.name", "tsb-synthetic")
    w.add_array("tsb.test_array", [1, 2, 3])
    H, F = cfg["n_embd"], cfg["n_ff"]
    Lg = synth.blob_layout(cfg)
    for l, layer in enumerate(layers):
        blobs = layer["blobs"]
        gu_row, d_row = Lg["gu_row"], Lg["d_row"]
        gate = np.stack([b[:F * gu_row] for b in blobs]).reshape(n_expert, F, gu_row)
        up = np.stack([b[Lg["up_off"]:Lg["up_off"] + F * gu_row] for b in blobs]).reshape(n_expert, F, gu_row)
        down = np.stack([b[Lg["down_off"]:Lg["down_off"] + H * d_row] for b in blobs]).reshape(n_expert, H, d_row)
        w.add_tensor(f"blk.{l}.ffn_gate_exps.weight", gate, raw_dtype=Q(cfg["gu_type"]))
        w.add_tensor(f"blk.{l}.ffn_up_exps.weight", up, raw_dtype=Q(cfg["gu_type"]))
        w.add_tensor(f"blk.{l}.ffn_down_exps.weight", down, raw_dtype=Q(cfg["d_type"]))
        w.add_tensor(f"blk.{l}.ffn_gate_inp.weight", np.ascontiguousarray(layer["router"][:n_expert]))
        if cfg.get("shared_gate"):
            w.add_tensor(f"blk.{l}.ffn_gate_inp_shexp.weight", np.ascontiguousarray(layer["router"][n_expert]))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


@pytest.mark.parametrize("name", ["qwen", "qwen_ep", "gemma", "lfm"])
def test_gguf_repack_equals_the_native_blobs(tmp_path, name):
    pytest.importorskip("gguf")
    from tinystrata_b200.gguf import GGUFFile
    cfg = {"qwen": synth.QWEN, "qwen_ep": synth.QWEN_EP, "gemma": synth.GEMMA, "lfm": synth.LFM}[name]
    E = 4
    layers = [synth.make_layer(cfg, 7 + l, n_expert=E) for l in range(2)]
    path = tmp_path / "m.gguf"
    _write_model(path, cfg, layers, E)
    with GGUFFile(str(path)) as g:
        assert g.kv_int("qwen35moe.block_count") == 2
        assert g.kv_int("qwen35moe.expert_count") == E
        assert abs(g.kv_float("qwen35moe.rms_eps") - 1e-6) < 1e-12
        assert g.kv_str("general.name") == "tsb-synthetic"
        assert g.kv_str("general.architecture") == "qwen35moe"
        names = g.tensor_names()
        assert "blk.1.ffn_down_exps.weight" in names
        for l, layer in enumerate(layers):
            L, stride, n = g.expert_layer(f"blk.{l}.")
            assert n == E
            want = synth.blob_layout(cfg)
            assert (L.gu_row, L.d_row, L.up_off, L.down_off, L.bytes) == (want["gu_row"], want["d_row"],
                                                                          want["up_off"], want["down_off"],
                                                                          want["bytes"])
            assert stride >= L.bytes and stride % 16 == 0
            assert stride % synth.BLOCK[cfg["gu_type"]][1] == 0 and stride % synth.BLOCK[cfg["d_type"]][1] == 0
            blobs = g.repack_experts(f"blk.{l}.")
            assert blobs.shape == (E, stride)
            for e in range(E):
                assert np.array_equal(blobs[e, :L.bytes], layer["blobs"][e]), (l, e)
                assert not blobs[e, L.bytes:].any()
            part = g.repack_experts(f"blk.{l}.", first=1, count=2)
            assert np.array_equal(part, blobs[1:3])
            router = g.tensor_f32(f"blk.{l}.ffn_gate_inp.weight")
            assert np.array_equal(router, layer["router"][:E])


def test_gguf_refuses_what_it_cannot_read(tmp_path):
    from tinystrata_b200 import TsbError
    from tinystrata_b200.gguf import GGUFFile
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOTGGUF" + bytes(64))
    with pytest.raises(TsbError, match="not a GGUF"):
        GGUFFile(str(bad))
    trunc = tmp_path / "trunc.gguf"
    trunc.write_bytes(b"GGUF" + (3).to_bytes(4, "little") + (5).to_bytes(8, "little") + (1).to_bytes(8, "little"))
    with pytest.raises(TsbError):
        GGUFFile(str(trunc))
    with pytest.raises(TsbError, match="cannot open"):
        GGUFFile(str(tmp_path / "missing.gguf"))


@pytest.mark.gpu
def test_gguf_layer_runs_through_the_expert_path(tmp_path, cuda):
    """A layer read from a GGUF file (repacked blobs at the reference's stride, router with the shared-gate row
    appended) through the decode-kernel layer and the tensor-core layer: the same outputs, bit for bit, as the same
    weights handed over directly."""
    pytest.importorskip("gguf")
    import torch
    import tinystrata_b200 as T
    from tinystrata_b200.gguf import GGUFFile
    from tinystrata_b200.layer import MoELayer, PrefillLayer
    cfg = dict(synth.QWEN, n_expert=32)
    layer = synth.make_layer(cfg, 11)
    path = tmp_path / "q.gguf"
    _write_model(path, cfg, [layer], 32)
    sh = torch.from_numpy(layer["sh_blob"]).to(cuda)
    x = torch.from_numpy(synth.rms_normed(np.random.default_rng(11), 64, cfg["n_embd"])).to(cuda)
    with GGUFFile(str(path)) as g:
        blobs, router, L = g.device_layer("blk.0.", cuda)
    direct_b = torch.from_numpy(layer["blobs"]).to(cuda)
    direct_r = torch.from_numpy(layer["router"]).to(cuda)
    assert torch.equal(router, direct_r)
    outs = []
    for b in (blobs, direct_b):
        M = MoELayer(cfg, b[:, :int(L.bytes)] if b.shape[1] != L.bytes else b, router, sh, max_tokens=64)
        xm = torch.zeros_like(x)
        M.forward(xm, x, T.quantize_q8_1_rows(x))
        P = PrefillLayer(cfg, b, router, sh, max_tokens=64)
        xp = torch.zeros_like(x)
        P.forward(xp, x)
        torch.cuda.synchronize()
        outs.append((xm.clone(), xp.clone()))
    assert T.device_error() == 0
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])

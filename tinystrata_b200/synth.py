"""Seeded synthetic MoE layers with the shapes and value distributions of the benchmark configurations.

There are no model files on the build or GPU machines, so every weight is synthetic: raw GGUF blocks with uniform
code bytes and the per-format scale fields drawn from |N(0, sd)| (fp16), routers fp32 N(0, 0.02).  The layouts are
TinyStrata's: one blob per expert, ``[gate rows | up rows | down rows]`` of raw GGUF blocks
(``NativeExpertLayout``, src/kernels/cuda/iq_kernels.cu:2120-2138).

CPU generation (numpy, ``make_layer``) feeds the parity tests; ``device_layers`` fills large stacks straight on the GPU
(torch's generator) for the benchmark, with the same distributions.
"""
from __future__ import annotations

import math

import numpy as np

T_Q4_0, T_Q8_0, T_Q4_K, T_Q6_K, T_IQ3_XXS, T_IQ3_S = 2, 8, 12, 14, 18, 21
BLOCK = {T_Q4_0: (32, 18), T_Q8_0: (32, 34), T_Q4_K: (256, 144), T_Q6_K: (256, 210), T_IQ3_XXS: (256, 98),
         T_IQ3_S: (256, 110)}
# byte offsets of the fp16 scale fields inside a block (drawn from |N(0, sd)|); everything else is uniform bytes
SCALE_FIELDS = {T_Q4_0: (0,), T_Q8_0: (0,), T_Q4_K: (0, 2), T_Q6_K: (208,), T_IQ3_XXS: (0,), T_IQ3_S: (0,)}
ACT_SWIGLU, ACT_GELU_TANH, ACT_SWIGLU_CLAMP = 0, 1, 2

# The benchmark configurations (sizes as in the benchmark definitions; seed per config).
QWEN = dict(name="qwen3.6-35b-a3b", n_embd=2048, n_ff=512, n_expert=256, n_used=8, gu_type=T_IQ3_XXS,
            d_type=T_IQ3_XXS, sh_n_ff=512, sh_gu_type=T_Q8_0, sh_d_type=T_Q8_0, router_mode="softmax",
            shared_gate=True, act=ACT_SWIGLU, w_sd=0.02, sh_sd=0.02, router_sd=0.02)
GEMMA = dict(name="gemma-4-26b-a4b", n_embd=2816, n_ff=704, n_expert=128, n_used=8, gu_type=T_Q4_0, d_type=T_Q4_0,
             sh_n_ff=2112, sh_gu_type=T_Q4_0, sh_d_type=T_Q4_0, router_mode="softmax_scaled", shared_gate=False,
             act=ACT_GELU_TANH, sh_act=ACT_GELU_TANH, w_sd=0.01, sh_sd=0.01, router_sd=0.02,
             in_scale=1.0 / math.sqrt(2816.0))
LFM = dict(name="lfm2.5-24b-a2b", n_embd=2048, n_ff=1792, n_expert=64, n_used=4, gu_type=T_Q4_K, d_type=T_Q6_K,
           sh_n_ff=0, router_mode="sigmoid", shared_gate=False, act=ACT_SWIGLU_CLAMP, limit=float("inf"), w_sd=0.01,
           router_sd=0.02, w_scale=0.0)
QWEN_EP = dict(QWEN, name="qwen3.6-35b-a3b-ep", d_type=T_IQ3_S)


def row_bytes(t: int, n: int) -> int:
    qk, bb = BLOCK[t]
    assert n % qk == 0, (t, n)
    return n // qk * bb


def blob_layout(cfg: dict, shared: bool = False) -> dict:
    H = cfg["n_embd"]
    F = cfg["sh_n_ff"] if shared else cfg["n_ff"]
    gu = cfg["sh_gu_type"] if shared else cfg["gu_type"]
    dt = cfg["sh_d_type"] if shared else cfg["d_type"]
    gu_row, d_row = row_bytes(gu, H), row_bytes(dt, F)
    up_off = F * gu_row
    down_off = 2 * up_off
    return dict(gu_type=gu, d_type=dt, n_embd=H, n_ff=F, gu_row=gu_row, d_row=d_row, up_off=up_off,
                down_off=down_off, bytes=down_off + H * d_row)


def gen_blocks(rng: np.random.Generator, t: int, n_blocks: int, sd: float) -> np.ndarray:
    """n_blocks GGUF blocks of type t: uniform bytes, fp16 scale fields |N(0, sd)|."""
    qk, bb = BLOCK[t]
    b = rng.integers(0, 256, size=(n_blocks, bb), dtype=np.uint8)
    for off in SCALE_FIELDS[t]:
        d = np.abs(rng.normal(0.0, sd, size=n_blocks)).astype(np.float16)
        b[:, off:off + 2] = d.view(np.uint8).reshape(n_blocks, 2)
    return b.reshape(-1)


def gen_matrix(rng, t: int, rows: int, n: int, sd: float) -> np.ndarray:
    qk, _ = BLOCK[t]
    return gen_blocks(rng, t, rows * (n // qk), sd)


def gen_blob(rng, cfg: dict, shared: bool = False) -> np.ndarray:
    L = blob_layout(cfg, shared)
    sd = cfg["sh_sd"] if shared else cfg["w_sd"]
    gate = gen_matrix(rng, L["gu_type"], L["n_ff"], L["n_embd"], sd)
    up = gen_matrix(rng, L["gu_type"], L["n_ff"], L["n_embd"], sd)
    down = gen_matrix(rng, L["d_type"], L["n_embd"], L["n_ff"], sd)
    blob = np.concatenate([gate, up, down])
    assert blob.size == L["bytes"]
    return blob


def make_layer(cfg: dict, seed: int, n_expert: int | None = None) -> dict:
    """One synthetic MoE layer on the host.  n_expert limits how many expert blobs are materialised (tests)."""
    rng = np.random.default_rng(seed)
    E = cfg["n_expert"]
    En = n_expert or E
    H = cfg["n_embd"]
    blobs = np.stack([gen_blob(rng, cfg) for _ in range(En)])
    rows = E + (1 if cfg.get("shared_gate") else 0)
    router = rng.normal(0.0, cfg["router_sd"], size=(rows, H)).astype(np.float32)
    layer = dict(cfg=dict(cfg), blobs=blobs, router=router)
    if cfg.get("sh_n_ff"):
        layer["sh_blob"] = gen_blob(rng, cfg, shared=True)
    if cfg["router_mode"] == "softmax_scaled":
        layer["escale"] = np.ones(E, np.float32)
    if cfg["router_mode"] == "sigmoid":
        layer["bias"] = np.zeros(E, np.float32)
    return layer


def rms_normed(rng, T: int, H: int) -> np.ndarray:
    x = rng.normal(0.0, 1.0, size=(T, H)).astype(np.float32)
    return (x / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=1, keepdims=True))).astype(np.float32)


def disjoint_router_spikes(router: np.ndarray, n_expert: int, n_used: int, T: int, H: int, scale: float = 1.0):
    """Make token t's top-n_used experts the set S_t = {(t*n_used + k) % n_expert} (disjoint across the step's tokens
    while T*n_used <= n_expert) by planting a weight on input dimension d_t in those experts' router rows; the
    matching inputs carry a spike on d_t (``spiked_inputs``).  Returns the spike dimensions."""
    dims = [(7 + 61 * t) % H for t in range(T)]
    for t in range(T):
        for k in range(n_used):
            e = (t * n_used + k) % n_expert
            router[e, dims[t]] = scale * (1.0 + 0.01 * k)
    return dims


def spiked_inputs(rng, T: int, H: int, dims, spike: float = 40.0) -> np.ndarray:
    x = rng.normal(0.0, 1.0, size=(T, H)).astype(np.float32)
    for t, d in enumerate(dims):
        x[t, d] = spike
    return x


def device_layers(cfg: dict, n_layers: int, seed: int, device, n_expert: int | None = None):
    """n_layers layers of expert blobs [L, E, blob_bytes] (uint8), generated on the device with torch's generator
    (uniform bytes, scale fields |N(0, sd)|), plus routers and shared blobs.  For the benchmark stack."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    E = n_expert or cfg["n_expert"]
    L = blob_layout(cfg)

    def fill(nbytes_rows, t, sd, shape):
        qk, bb = BLOCK[t]
        n_blocks = nbytes_rows // bb
        b = torch.randint(0, 256, (n_blocks, bb), generator=g, device=device, dtype=torch.uint8)
        for off in SCALE_FIELDS[t]:
            d = torch.randn(n_blocks, generator=g, device=device).abs_().mul_(sd).to(torch.float16)
            b[:, off:off + 2] = d.view(torch.uint8).view(n_blocks, 2)
        return b.view(shape)

    blobs = torch.empty((n_layers, E, L["bytes"]), dtype=torch.uint8, device=device)
    gu_bytes = L["up_off"]
    for l in range(n_layers):
        blobs[l, :, :gu_bytes] = fill(E * gu_bytes, L["gu_type"], cfg["w_sd"], (E, gu_bytes))
        blobs[l, :, gu_bytes:2 * gu_bytes] = fill(E * gu_bytes, L["gu_type"], cfg["w_sd"], (E, gu_bytes))
        dn = L["bytes"] - L["down_off"]
        blobs[l, :, L["down_off"]:] = fill(E * dn, L["d_type"], cfg["w_sd"], (E, dn))
    out = dict(blobs=blobs, layout=L)
    if cfg.get("sh_n_ff"):
        S = blob_layout(cfg, shared=True)
        sh = torch.empty((n_layers, S["bytes"]), dtype=torch.uint8, device=device)
        for l in range(n_layers):
            sh[l, :S["up_off"]] = fill(S["up_off"], S["gu_type"], cfg["sh_sd"], (S["up_off"],))
            sh[l, S["up_off"]:S["down_off"]] = fill(S["up_off"], S["gu_type"], cfg["sh_sd"], (S["up_off"],))
            dn = S["bytes"] - S["down_off"]
            sh[l, S["down_off"]:] = fill(dn, S["d_type"], cfg["sh_sd"], (dn,))
        out["sh_blobs"] = sh
        out["sh_layout"] = S
    rows = cfg["n_expert"] + (1 if cfg.get("shared_gate") else 0)
    out["routers"] = torch.randn((n_layers, rows, cfg["n_embd"]), generator=g, device=device).mul_(cfg["router_sd"])
    return out

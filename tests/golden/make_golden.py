"""Generates the golden fixtures in this folder from the CPU oracle.

    python tests/golden/make_golden.py

The reference (TypeScript) cannot run where this build runs and its own tests
hold no vectors for this path, so these fixtures are produced by the C
restatement in oracle/ (which is itself checked against independent numpy
closed forms and the WGSL-semantics variant in tests/test_oracle.py).  They pin
the oracle against regressions and give the GPU tests fixed inputs.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402

# rmsEps as the GGUF loader holds it: an f32 value (src/gguf.ts:312,464)
EPS = float(np.float32(1e-6))


def attention_q8_case(rng, S, H, KV, Dh, pos_base, window):
    """The engine's exact sequence for one layer and segment (src/engine.ts
    :1305-1317): append K and V [S, KV, Dh] into Q8_0 caches at pos_base,
    then attention_q8 over rows [.., pos_base + S)."""
    rows = pos_base + S
    k_hist = rng.standard_normal((rows, KV, Dh), dtype=np.float32)
    v_hist = rng.standard_normal((rows, KV, Dh), dtype=np.float32)
    q = rng.standard_normal((S, H, Dh), dtype=np.float32)
    kq = np.zeros((rows, KV, Dh), np.int8)
    ks = np.zeros((rows, KV, Dh // 32), np.float32)
    vq, vs = kq.copy(), ks.copy()
    oracle.append_kv_q8(k_hist, kq, ks, 0)
    oracle.append_kv_q8(v_hist, vq, vs, 0)
    out = oracle.attention(q, kq, vq, pos_base, window, oracle.KV_Q8_0, ks, vs)
    return dict(k=k_hist, v=v_hist, q=q, kq=kq, ks=ks, vq=vq, vs=vs, out=out,
                meta=np.array([S, H, KV, Dh, pos_base, window], np.int64))


def attention_dense_case(rng, fmt, B, H, KV, Dh, lens, S=1, window=0):
    lens = np.asarray(lens, np.int64)
    off = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    total = int(lens.sum())
    q = rng.standard_normal((B, S, H, Dh), dtype=np.float32)
    k = rng.standard_normal((total, KV, Dh), dtype=np.float32)
    v = rng.standard_normal((total, KV, Dh), dtype=np.float32)
    if fmt == oracle.KV_F16:
        k, v = k.astype(np.float16).view(np.uint16), v.astype(np.float16).view(np.uint16)
    elif fmt == oracle.KV_BF16:
        k = (k.view(np.uint32) >> 16).astype(np.uint16)  # truncation is fine for inputs
        v = (v.view(np.uint32) >> 16).astype(np.uint16)
    pos = (lens - S).astype(np.int32)
    out = oracle.attention_batch(q, k, v, pos, off, window, fmt)
    return dict(q=q, k=k, v=v, lens=lens, off=off, pos=pos, out=out,
                meta=np.array([fmt, B, S, H, KV, Dh, window], np.int64))


def gdn_case(rng, S, NK, NV, D, load_state):
    conv_dim = 2 * NK * D + NV * D
    qkv = rng.standard_normal((S, conv_dim), dtype=np.float32)
    a = rng.standard_normal((S, NV), dtype=np.float32)
    b = rng.standard_normal((S, NV), dtype=np.float32)
    a_neg = -np.exp(rng.standard_normal(NV, dtype=np.float32) * np.float32(0.5))
    dt_bias = (rng.standard_normal(NV, dtype=np.float32) * np.float32(0.5)).astype(np.float32)
    state = (rng.standard_normal((NV, D, D), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    gbeta = oracle.deltanet_gbeta(a, b, a_neg.astype(np.float32), dt_bias)
    core, new_state = oracle.deltanet_recur(qkv, gbeta, state, NK, NV, load_state)
    return dict(qkv=qkv, a=a, b=b, a_neg=a_neg.astype(np.float32), dt_bias=dt_bias, state=state, gbeta=gbeta,
                core=core, new_state=new_state, meta=np.array([S, NK, NV, D, int(load_state)], np.int64))


def conv1d_case(rng, S, C, K, load_state):
    x = rng.standard_normal((S, C), dtype=np.float32)
    w = (rng.standard_normal((C, K), dtype=np.float32) * np.float32(0.5)).astype(np.float32)
    state = rng.standard_normal((K - 1, C), dtype=np.float32)
    y, new_state = oracle.conv1d_causal(x, w, state, load_state)
    return dict(x=x, w=w, state=state, y=y, new_state=new_state, meta=np.array([S, C, K, int(load_state)], np.int64))


def norm_gate_case(rng, rows, DV, eps):
    core = rng.standard_normal((rows, DV), dtype=np.float32)
    z = rng.standard_normal((rows, DV), dtype=np.float32)
    gamma = (1 + rng.standard_normal(DV, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    y = oracle.deltanet_norm_gate(core, z, gamma, eps)
    return dict(core=core, z=z, gamma=gamma, y=y, eps=np.array([eps], np.float32),
                meta=np.array([rows, DV], np.int64))


def gdn_layer_case(rng, B, NK, NV, D, K, load_state, eps):
    C = 2 * NK * D + NV * D
    d = dict(
        qkv=rng.standard_normal((B, C), dtype=np.float32),
        conv_w=(rng.standard_normal((C, K), dtype=np.float32) * np.float32(0.5)).astype(np.float32),
        conv_state=rng.standard_normal((B, K - 1, C), dtype=np.float32),
        a=rng.standard_normal((B, NV), dtype=np.float32),
        b=rng.standard_normal((B, NV), dtype=np.float32),
        a_neg=(-np.exp(rng.standard_normal(NV, dtype=np.float32) * np.float32(0.5))).astype(np.float32),
        dt_bias=(rng.standard_normal(NV, dtype=np.float32) * np.float32(0.5)).astype(np.float32),
        z=rng.standard_normal((B, NV * D), dtype=np.float32),
        gamma=(1 + rng.standard_normal(D, dtype=np.float32) * np.float32(0.1)).astype(np.float32),
        state=(rng.standard_normal((B, NV, D, D), dtype=np.float32) * np.float32(0.02)).astype(np.float32),
    )
    if not load_state:  # unused: zeros keep the fixture small
        d["state"][:] = 0
        d["conv_state"][:] = 0
    out, conv_new, st_new = oracle.gdn_layer_step(d["qkv"], d["conv_w"], d["conv_state"], d["a"], d["b"],
                                                  d["a_neg"], d["dt_bias"], d["z"], d["gamma"], eps, d["state"],
                                                  NK, NV, load_state)
    d.update(out=out, new_conv_state=conv_new, new_state=st_new, eps=np.array([eps], np.float32),
             meta=np.array([B, NK, NV, D, K, int(load_state)], np.int64))
    return d


def attn_layer_case(rng, S, H, KV, Dh, rot, pos, split, eps):
    """The full-attention layer step of one sequence (src/wasm-backend.ts
    :1125-1157) on a Q8_0 cache that holds `pos` earlier rows."""
    rows = pos + S
    qg = rng.standard_normal((S, H, 2 * Dh if split else Dh), dtype=np.float32)
    k = rng.standard_normal((S, KV, Dh), dtype=np.float32)
    v = rng.standard_normal((S, KV, Dh), dtype=np.float32)
    qn = (1 + rng.standard_normal(Dh, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    kn = (1 + rng.standard_normal(Dh, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    kq, ks = np.zeros((rows, KV, Dh), np.int8), np.zeros((rows, KV, Dh // 32), np.float32)
    vq, vs = kq.copy(), ks.copy()
    if pos:
        oracle.append_kv_q8(rng.standard_normal((pos, KV, Dh), dtype=np.float32), kq, ks, 0)
        oracle.append_kv_q8(rng.standard_normal((pos, KV, Dh), dtype=np.float32), vq, vs, 0)
    cos, sin = oracle.rope_tables(rot, rows, 1e6)
    d = dict(qg=qg, k=k, v=v, qn=qn, kn=kn, kq0=kq.copy(), ks0=ks.copy(), vq0=vq.copy(), vs0=vs.copy(), cos=cos,
             sin=sin, eps=np.array([eps], np.float32), meta=np.array([S, H, KV, Dh, rot, pos, int(split)], np.int64))
    q = np.ascontiguousarray(qg[..., :Dh]) if split else qg
    gate = np.ascontiguousarray(qg[..., Dh:]) if split else None
    q_out, out = oracle.attn_layer_step(q, k, v, qn, kn, eps, cos, sin, rot, pos, kq, ks, vq, vs, gate=gate)
    d.update(q_out=q_out, out=out, kq=kq, ks=ks, vq=vq, vs=vs)
    return d


def main():
    rng = np.random.default_rng(20240601)
    cases = {
        "attn_q8_decode": attention_q8_case(rng, 1, 4, 2, 128, 77, 0),
        "attn_q8_segment": attention_q8_case(rng, 8, 8, 4, 128, 24, 0),
        "attn_q8_swa": attention_q8_case(rng, 3, 4, 1, 128, 50, 16),
        "attn_q8_dh256": attention_q8_case(rng, 1, 8, 2, 256, 20, 0),
        "attn_f32_batch": attention_dense_case(rng, oracle.KV_F32, 3, 4, 2, 128, [5, 40, 70]),
        "attn_f16_batch": attention_dense_case(rng, oracle.KV_F16, 3, 8, 2, 128, [1, 64, 90]),
        "attn_bf16_batch": attention_dense_case(rng, oracle.KV_BF16, 2, 4, 4, 128, [33, 45]),
        "gdn_decode": gdn_case(rng, 1, 1, 2, 128, True),
        "gdn_segment_fresh": gdn_case(rng, 8, 1, 2, 128, False),
        # the layer's neighbours of the recurrence (conv1d_causal, deltanet_norm_gate, and the fused step)
        "conv1d_segment": conv1d_case(rng, 5, 96, 4, True),
        "conv1d_fresh": conv1d_case(rng, 2, 64, 4, False),
        "norm_gate": norm_gate_case(rng, 6, 128, EPS),
        "gdn_layer_step": gdn_layer_case(rng, 2, 1, 2, 128, 4, True, EPS),
        "gdn_layer_fresh": gdn_layer_case(rng, 1, 1, 3, 128, 4, False, EPS),
        # the full-attention layer's neighbours (q/k RMSNorm, RoPE, Q8_0 append, sigmoid gate)
        "attn_layer_qwen3": attn_layer_case(rng, 2, 8, 4, 128, 128, 40, False, EPS),
        "attn_layer_qwen35": attn_layer_case(rng, 1, 4, 2, 256, 64, 30, True, EPS),
    }
    for name, arrays in cases.items():
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
        print(name, sum(a.nbytes for a in arrays.values()), "bytes")


if __name__ == "__main__":
    main()

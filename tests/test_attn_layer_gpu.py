"""GPU parity of the full-attention layer's neighbours of the KV append and
the attention (src/engine.ts:1408-1458; JS src/wasm-backend.ts:1125-1157)
against the oracle: rmsnorm, rope, split_q_gate and sigmoid_gate through the
reference's op names, the fused prologue (split + per-head q / k RMSNorm + RoPE
+ K / V append), the sigmoid-gate epilogue of the decode kernels, and a whole
layer step (prologue + gated attention) for qwen3 and qwen35 shapes.

Tolerances: the standalone ops and the prologue follow the JS arithmetic (f64,
f32 stores), so q rows agree to relative L2 <= 1e-6 and a Q8_0 cache written by
the prologue is bit-identical to appendKvQ8 of the oracle's rows; attention
outputs (f32 decode) to relative L2 <= 1e-4."""
import numpy as np
import pytest
import torch

import oracle
from hachiue_b200 import KV_F16, KV_Q8_0
from hachiue_b200.backend import KVCache, f32_word
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu
dev = "cuda"
TOL = 1e-4
TIGHT = 1e-6


def T(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def test_standalone_ops_via_dispatch(backend):
    rng = np.random.default_rng(5)
    S, H, Dh, rot, pos = 3, 4, 128, 64, 17
    x = rng.standard_normal((S, H, Dh), dtype=np.float32)
    g = rng.standard_normal(Dh, dtype=np.float32)
    y = torch.zeros((S, H, Dh), device=dev)
    backend.dispatch("rmsnorm", [S * H, Dh, f32_word(1e-6), 0], [T(x), T(g), y])
    torch.cuda.synchronize()
    ref = oracle.rmsnorm(x, g, 1e-6)
    assert rel_l2(y.cpu().numpy(), ref) < TIGHT
    y1 = torch.zeros_like(y)
    backend.dispatch("rmsnorm", [S * H, Dh, f32_word(1e-6), 1], [T(x), T(g), y1])
    torch.cuda.synchronize()
    assert rel_l2(y1.cpu().numpy(), oracle.rmsnorm(x, g, 1e-6, True)) < TIGHT

    cos, sin = oracle.rope_tables(rot, 64, 1e6)
    xr = T(ref)
    backend.dispatch("rope", [S, H, Dh, rot, pos], [T(cos), T(sin), xr])
    torch.cuda.synchronize()
    assert rel_l2(xr.cpu().numpy(), oracle.rope(ref, rot, pos, cos, sin)) < TIGHT

    qg = rng.standard_normal((S, H, 2 * Dh), dtype=np.float32)
    q, gate = torch.zeros((S, H, Dh), device=dev), torch.zeros((S, H, Dh), device=dev)
    backend.dispatch("split_q_gate", [S, H, Dh], [T(qg), q, gate])
    torch.cuda.synchronize()
    np.testing.assert_array_equal(q.cpu().numpy(), qg[..., :Dh])
    np.testing.assert_array_equal(gate.cpu().numpy(), qg[..., Dh:])

    att = T(x)
    backend.dispatch("sigmoid_gate", [x.size], [T(qg[..., Dh:]), att])
    torch.cuda.synchronize()
    assert rel_l2(att.cpu().numpy(), oracle.sigmoid_gate(qg[..., Dh:], x)) < TIGHT


def q8_cache(rows, KV, Dh):
    return (np.zeros((rows, KV, Dh), np.int8), np.zeros((rows, KV, Dh // 32), np.float32),
            np.zeros((rows, KV, Dh), np.int8), np.zeros((rows, KV, Dh // 32), np.float32))


def layer_inputs(rng, S, H, KV, Dh, split):
    return dict(q=rng.standard_normal((S, H, 2 * Dh if split else Dh), dtype=np.float32),
                k=rng.standard_normal((S, KV, Dh), dtype=np.float32),
                v=rng.standard_normal((S, KV, Dh), dtype=np.float32),
                qn=(1 + 0.1 * rng.standard_normal(Dh)).astype(np.float32),
                kn=(1 + 0.1 * rng.standard_normal(Dh)).astype(np.float32))


@pytest.mark.parametrize("S,H,KV,Dh,rot,pos,split", [(1, 16, 8, 128, 128, 300, False),   # qwen3 decode
                                                     (5, 16, 8, 128, 128, 0, False),     # qwen3 prompt segment
                                                     (1, 16, 2, 256, 64, 77, True),      # qwen35 full attention
                                                     (3, 8, 2, 256, 256, 12, True)])
def test_layer_step_q8_against_the_oracle(backend, S, H, KV, Dh, rot, pos, split):
    """Prologue (fused) then attention with the gate epilogue, on a Q8_0 cache
    that already holds `pos` rows, against the oracle's runRmsNorm / applyRope
    / appendKvQ8 / runAttentionQ8 / gate sequence."""
    rng = np.random.default_rng(S * 7 + Dh + pos)
    d = layer_inputs(rng, S, H, KV, Dh, split)
    rows = pos + S + 3
    kq, ks, vq, vs = q8_cache(rows, KV, Dh)
    hist_k = rng.standard_normal((pos, KV, Dh), dtype=np.float32)
    hist_v = rng.standard_normal((pos, KV, Dh), dtype=np.float32)
    if pos:
        oracle.append_kv_q8(hist_k, kq, ks, 0)
        oracle.append_kv_q8(hist_v, vq, vs, 0)
    cos, sin = oracle.rope_tables(rot, rows, 1e6)
    eps = float(np.float32(1e-6))  # GGUF stores rmsEps as f32 (src/gguf.ts:312,464)
    qd = d["q"][..., :Dh] if split else d["q"]
    gate = d["q"][..., Dh:] if split else None
    cache = KVCache(KV_Q8_0, T(kq), T(vq), T(ks), T(vs))
    q_out = torch.zeros((S, H, Dh), device=dev)
    gate_out = torch.zeros((S, H, Dh), device=dev) if split else None
    backend.attn_prologue(T(d["q"]), T(d["k"]), T(d["v"]), T(d["qn"]), T(d["kn"]), T(cos), T(sin), q_out, cache, pos,
                          eps, rot, gate_out=gate_out)
    out = torch.zeros((S, H, Dh), device=dev)
    backend.attention(q_out, cache, out, pos, gate=gate_out)
    torch.cuda.synchronize()
    ref_q, ref_out = oracle.attn_layer_step(np.ascontiguousarray(qd), d["k"], d["v"], d["qn"], d["kn"], eps, cos, sin,
                                            rot, pos, kq, ks, vq, vs, gate=gate)
    assert rel_l2(q_out.cpu().numpy(), ref_q) < TIGHT
    np.testing.assert_array_equal(cache.k.cpu().numpy(), kq)
    np.testing.assert_array_equal(cache.v.cpu().numpy(), vq)
    np.testing.assert_array_equal(cache.k_scale.cpu().numpy(), ks)
    np.testing.assert_array_equal(cache.v_scale.cpu().numpy(), vs)
    if split:
        np.testing.assert_array_equal(gate_out.cpu().numpy(), gate)
    assert rel_l2(out.cpu().numpy(), ref_out) < TOL
    assert backend.device_status() == 0


def test_batched_prologue_and_gated_tensor_core_attention(backend):
    """Eight sequences at different positions in one packed f16 cache: the
    prologue appends each sequence's token at its own row, and the tcgen05
    decode kernel applies the gate."""
    rng = np.random.default_rng(11)
    B, H, KV, Dh, rot = 8, 32, 8, 128, 128
    lens = rng.integers(40, 300, B)
    off = np.concatenate([[0], np.cumsum(lens + 1)[:-1]]).astype(np.int64)
    rows = int(off[-1] + lens[-1] + 1)
    kc = (rng.standard_normal((rows, KV, Dh)).astype(np.float16))
    vc = (rng.standard_normal((rows, KV, Dh)).astype(np.float16))
    q = rng.standard_normal((B, 1, H, 2 * Dh), dtype=np.float32)
    k = rng.standard_normal((B, 1, KV, Dh), dtype=np.float32)
    v = rng.standard_normal((B, 1, KV, Dh), dtype=np.float32)
    qn = (1 + 0.1 * rng.standard_normal(Dh)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(Dh)).astype(np.float32)
    cos, sin = oracle.rope_tables(rot, 400, 1e6)
    cache = KVCache(KV_F16, T(kc), T(vc))
    pos_t = torch.from_numpy(lens.astype(np.int32)).to(dev)
    off_t = torch.from_numpy(off).to(dev)
    q_out = torch.zeros((B, 1, H, Dh), device=dev)
    gate_out = torch.zeros((B, 1, H, Dh), device=dev)
    backend.attn_prologue(T(q), T(k), T(v), T(qn), T(kn), T(cos), T(sin), q_out, cache, pos_t, 1e-6, rot,
                          gate_out=gate_out, kv_row_offset=off_t)
    out = torch.zeros((B, 1, H, Dh), device=dev)
    backend.attention(q_out, cache, out, pos_t, kv_row_offset=off_t, max_context=int(lens.max()) + 1, gate=gate_out)
    torch.cuda.synchronize()
    kc_new, vc_new = cache.k.cpu().numpy(), cache.v.cpu().numpy()
    qo, oo = q_out.cpu().numpy(), out.cpu().numpy()
    for b in range(B):
        p = int(lens[b])
        qr = oracle.rope(oracle.rmsnorm(q[b, :, :, :Dh], qn, 1e-6), rot, p, cos, sin)
        kr = oracle.rope(oracle.rmsnorm(k[b], kn, 1e-6), rot, p, cos, sin)
        assert rel_l2(qo[b], qr) < TIGHT
        np.testing.assert_array_equal(kc_new[off[b] + p], kr[0].astype(np.float16))
        np.testing.assert_array_equal(vc_new[off[b] + p], v[b, 0].astype(np.float16))
        ref = oracle.attention(qr, kc_new[off[b]:off[b] + p + 1], vc_new[off[b]:off[b] + p + 1], p, 0, oracle.KV_F16)
        ref = oracle.sigmoid_gate(q[b, :, :, Dh:], ref)
        assert rel_l2(oo[b], ref) < TOL
    assert backend.device_status() == 0


@pytest.mark.parametrize("name", ["attn_layer_qwen3", "attn_layer_qwen35"])
def test_layer_step_golden(backend, name):
    """The committed fixtures (oracle outputs): fused prologue + gated attention."""
    import os
    d = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", name + ".npz")))
    S, H, KV, Dh, rot, pos, split = (int(x) for x in d["meta"])
    cache = KVCache(KV_Q8_0, T(d["kq0"]), T(d["vq0"]), T(d["ks0"]), T(d["vs0"]))
    q_out = torch.zeros((S, H, Dh), device=dev)
    gate_out = torch.zeros((S, H, Dh), device=dev) if split else None
    backend.attn_prologue(T(d["qg"]), T(d["k"]), T(d["v"]), T(d["qn"]), T(d["kn"]), T(d["cos"]), T(d["sin"]), q_out,
                          cache, pos, float(d["eps"][0]), rot, gate_out=gate_out)
    out = torch.zeros((S, H, Dh), device=dev)
    backend.attention(q_out, cache, out, pos, gate=gate_out)
    torch.cuda.synchronize()
    assert rel_l2(q_out.cpu().numpy(), d["q_out"]) < TIGHT
    for t, key in ((cache.k, "kq"), (cache.k_scale, "ks"), (cache.v, "vq"), (cache.v_scale, "vs")):
        np.testing.assert_array_equal(t.cpu().numpy(), d[key])
    assert rel_l2(out.cpu().numpy(), d["out"]) < TOL

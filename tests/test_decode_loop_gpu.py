"""A decode loop over a small qwen35-style hybrid model through the library:
hachiue_b200.arch picks each layer's kernel and holds its device state (Q8_0
KV cache, ping-ponged GDN recurrent and conv states, cache_pos / ssm_parity as
src/engine.ts:1352-1353 and :1481-1483 keep them), and every step's layer
outputs are compared with the oracle's layer steps.  Layer 0 and 2 are Gated
DeltaNet layers (fused layer step), layer 3 full attention with the doubled
q projection and the sigmoid gate (fused prologue + gated attention)."""
import numpy as np
import pytest
import torch

import oracle
from hachiue_b200 import KV_Q8_0
from hachiue_b200.arch import HybridLayerConfig, LayerStates, ModelArch, hybrid_layer_types
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu
dev = "cuda"
TOL = 1e-4


def T(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def test_hybrid_decode_loop(backend):
    rng = np.random.default_rng(31)
    NK, NV, D, K = 2, 4, 128, 4
    H, KVH, Dh, rot, eps = 4, 2, 128, 64, float(np.float32(1e-6))  # an f32 value, as GGUF stores it
    arch = ModelArch("qwen35", 4, H, KVH, Dh, eps, rot, 64,
                     hybrid=HybridLayerConfig(hybrid_layer_types(4, 4), NK, NV, D, K))
    st = LayerStates(arch, max_seq_len=16, kv_format=KV_Q8_0)
    C = arch.hybrid.conv_dim
    lin = [li for li in range(4) if arch.layer_kind(li) == "linear"]
    full = [li for li in range(4) if arch.layer_kind(li) == "full"]
    assert lin == [0, 1, 2] and full == [3]
    # weights
    conv_w = {li: (0.3 * rng.standard_normal((C, K))).astype(np.float32) for li in lin}
    a_neg = {li: -np.exp(rng.standard_normal(NV)).astype(np.float32) for li in lin}
    dt_bias = {li: rng.standard_normal(NV).astype(np.float32) for li in lin}
    gamma = {li: (1 + 0.1 * rng.standard_normal(D)).astype(np.float32) for li in lin}
    qn_w = (1 + 0.1 * rng.standard_normal(Dh)).astype(np.float32)
    kn_w = (1 + 0.1 * rng.standard_normal(Dh)).astype(np.float32)
    cos, sin = oracle.rope_tables(rot, 16, 1e6)
    # oracle state
    ref_conv = {li: np.zeros((1, K - 1, C), np.float32) for li in lin}
    ref_rec = {li: np.zeros((1, NV, D, D), np.float32) for li in lin}
    kq = np.zeros((16, KVH, Dh), np.int8)
    vq = np.zeros_like(kq)
    ks = np.zeros((16, KVH, Dh // 32), np.float32)
    vs = np.zeros_like(ks)
    cache = st.caches[3]
    for step in range(5):
        pos = st.cache_pos
        for li in lin:
            x = rng.standard_normal((1, C)).astype(np.float32)
            ab = rng.standard_normal((2, 1, NV)).astype(np.float32)
            z = rng.standard_normal((1, NV * D)).astype(np.float32)
            s_in, s_out = st.gdn_states(li)
            c_in, c_out = st.conv_state_pair(li)
            out = torch.zeros((1, NV * D), device=dev)
            backend.gdn_layer_step(T(x), T(conv_w[li]), c_in[None], c_out[None], T(ab[0]), T(ab[1]), T(a_neg[li]),
                                   T(dt_bias[li]), T(z), T(gamma[li]), s_in[None], s_out[None], out, NK, NV, eps,
                                   load_state=st.load_state)
            ref_out, ref_conv[li], ref_rec[li] = oracle.gdn_layer_step(
                x, conv_w[li], ref_conv[li], ab[0], ab[1], a_neg[li], dt_bias[li], z, gamma[li], eps, ref_rec[li],
                NK, NV, load_state=pos > 0)
            torch.cuda.synchronize()
            assert rel_l2(out.cpu().numpy(), ref_out) < TOL, (step, li)
            assert rel_l2(s_out.cpu().numpy(), ref_rec[li][0]) < TOL, (step, li)
        q = rng.standard_normal((1, H, 2 * Dh)).astype(np.float32)
        k = rng.standard_normal((1, KVH, Dh)).astype(np.float32)
        v = rng.standard_normal((1, KVH, Dh)).astype(np.float32)
        q_out = torch.zeros((1, H, Dh), device=dev)
        gate = torch.zeros((1, H, Dh), device=dev)
        backend.attn_prologue(T(q), T(k), T(v), T(qn_w), T(kn_w), T(cos), T(sin), q_out, cache, pos, eps, rot,
                              gate_out=gate)
        out = torch.zeros((1, H, Dh), device=dev)
        backend.attention(q_out, cache, out, pos, arch.attention_window(3), gate=gate)
        _, ref = oracle.attn_layer_step(np.ascontiguousarray(q[..., :Dh]), k, v, qn_w, kn_w, eps, cos, sin, rot, pos,
                                        kq, ks, vq, vs, gate=np.ascontiguousarray(q[..., Dh:]))
        torch.cuda.synchronize()
        assert rel_l2(out.cpu().numpy(), ref) < TOL, step
        st.advance(1)
    np.testing.assert_array_equal(cache.k[:5].cpu().numpy(), kq[:5])
    np.testing.assert_array_equal(cache.v_scale[:5].cpu().numpy(), vs[:5])
    assert st.cache_pos == 5 and st.ssm_parity == 1
    assert backend.device_status() == 0

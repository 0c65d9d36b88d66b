"""A prompt prefilled whole, then decoded token by token: the handoff the
reference makes 8 tokens at a time (PREFILL_CHUNK, src/engine.ts:29), here
from the whole-prompt kernels to the decode kernels.
  * Gated DeltaNet: hcu_deltanet_chunked_prefill's final state feeds
    hcu_deltanet_decode (g / beta fused), against the token-serial recurrence
    over prompt + decode tokens.
  * Sliding-window attention: hcu_swa_prefill over the prompt, the prompt's
    K / V appended to the Q8_0 cache, then windowed decode attention, against
    runAttentionQ8 over the whole sequence.
Prefill tolerance (bf16 operands): relative L2 <= 1e-2; decode after a
bf16-prefilled state inherits it; decode attention reads the exact Q8_0 cache:
relative L2 <= 1e-4."""
import numpy as np
import pytest
import torch

import oracle
from hachiue_b200 import KV_Q8_0
from hachiue_b200.backend import KVCache
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu
dev = "cuda"


def bf16(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16)


def test_gdn_prefill_then_decode(backend):
    rng = np.random.default_rng(41)
    NK, NV, D, T, n_dec = 2, 4, 128, 200, 4
    q = rng.standard_normal((T + n_dec, NK, D)).astype(np.float32)
    k = rng.standard_normal((T + n_dec, NK, D)).astype(np.float32)
    v = rng.standard_normal((T + n_dec, NV, D)).astype(np.float32)
    # the prompt's operands at the prefill's bf16 precision, the oracle's too
    q[:T], k[:T], v[:T] = (bf16(x[:T]).float().numpy() for x in (q, k, v))
    a = rng.standard_normal((T + n_dec, NV)).astype(np.float32)
    b = rng.standard_normal((T + n_dec, NV)).astype(np.float32)
    a_neg = -np.exp(0.5 * rng.standard_normal(NV)).astype(np.float32)
    dt_bias = (0.5 * rng.standard_normal(NV)).astype(np.float32)
    gb = oracle.deltanet_gbeta(a, b, a_neg, dt_bias)
    qkv = np.concatenate([q.reshape(T + n_dec, -1), k.reshape(T + n_dec, -1), v.reshape(T + n_dec, -1)], 1)
    ref_core, ref_state = oracle.deltanet_recur(np.ascontiguousarray(qkv), gb, np.zeros((NV, D, D), np.float32),
                                                NK, NV, False)
    # prefill the prompt
    core = torch.zeros((1, T, NV, D), device=dev)
    s0 = torch.zeros((1, NV, D, D), device=dev)
    backend.deltanet_chunked_prefill(bf16(q[None, :T]).to(dev), bf16(k[None, :T]).to(dev), bf16(v[None, :T]).to(dev),
                                     torch.from_numpy(np.ascontiguousarray(gb[0, :T][None])).to(dev),
                                     torch.from_numpy(np.ascontiguousarray(gb[1, :T][None])).to(dev), core, s0)
    torch.cuda.synchronize()
    assert rel_l2(core[0].cpu().numpy(), ref_core[:T]) < 1e-2
    # decode the rest from the prefilled state (ping-pong)
    s1 = torch.zeros_like(s0)
    states = [s0, s1]
    outs = []
    for i in range(n_dec):
        t = T + i
        c = torch.zeros((1, NV, D), device=dev)
        backend.deltanet_decode(torch.from_numpy(np.ascontiguousarray(qkv[t:t + 1])).to(dev),
                                torch.from_numpy(a[t:t + 1]).to(dev), torch.from_numpy(b[t:t + 1]).to(dev),
                                torch.from_numpy(a_neg).to(dev), torch.from_numpy(dt_bias).to(dev),
                                states[i & 1][0], c, states[(i + 1) & 1][0], NK, NV, load_state=True)
        outs.append(c)
    torch.cuda.synchronize()
    dec = torch.cat(outs).cpu().numpy()
    assert rel_l2(dec, ref_core[T:]) < 1e-2
    assert rel_l2(states[n_dec & 1][0].cpu().numpy(), ref_state) < 1e-2
    assert backend.device_status() == 0


def test_swa_prefill_then_windowed_decode(backend):
    rng = np.random.default_rng(43)
    H, KV, D, T, W, n_dec = 8, 2, 128, 300, 128, 3
    q = bf16(rng.standard_normal((1, T, H, D))).to(dev)
    kp = bf16(rng.standard_normal((1, T, KV, D))).to(dev)
    vp = bf16(rng.standard_normal((1, T, KV, D))).to(dev)
    out = torch.zeros((1, T, H, D), device=dev)
    backend.swa_prefill(q, kp, vp, out, W)
    # the prompt's K / V go into the engine's Q8_0 cache, then decode continues
    cache = KVCache.allocate(T + n_dec, KV, D, KV_Q8_0)
    backend.kv_append(kp[0].float(), cache, "k", 0)
    backend.kv_append(vp[0].float(), cache, "v", 0)
    torch.cuda.synchronize()
    ref_pre = oracle.attention(q[0].float().cpu().numpy(), kp[0].float().cpu().numpy(), vp[0].float().cpu().numpy(),
                               0, W)
    assert rel_l2(out[0].cpu().numpy(), ref_pre) < 1e-2
    for i in range(n_dec):
        pos = T + i
        qd = rng.standard_normal((1, H, D)).astype(np.float32)
        kd = rng.standard_normal((1, KV, D)).astype(np.float32)
        vd = rng.standard_normal((1, KV, D)).astype(np.float32)
        backend.kv_append(torch.from_numpy(kd).to(dev), cache, "k", pos)
        backend.kv_append(torch.from_numpy(vd).to(dev), cache, "v", pos)
        o = torch.zeros((1, H, D), device=dev)
        backend.attention(torch.from_numpy(qd).to(dev), cache, o, pos, W)
        torch.cuda.synchronize()
        n = pos + 1
        ref = oracle.attention(qd, cache.k[:n].cpu().numpy(), cache.v[:n].cpu().numpy(), pos, W, KV_Q8_0,
                               cache.k_scale[:n].cpu().numpy(), cache.v_scale[:n].cpu().numpy())
        assert rel_l2(o.cpu().numpy(), ref) < 1e-4, i
    assert backend.device_status() == 0

"""CPU checks of the oracle (the checker the GPU parity tests trust).

Parity is unpinned by the reference (TypeScript, no runtime here, no golden
vectors for this path), so the oracle is pinned three other ways: against the
committed fixtures, against independent dense numpy f64 closed forms, against
the WGSL-semantics variant of each reference kernel, and against known answers
worked out by hand.
"""
import glob
import os

import numpy as np
import pytest

import oracle
from tests.conftest import rel_l2

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


@pytest.mark.parametrize("name", sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "*.npz"))))
def test_golden_reproduces(name):
    d = load(name)
    if name.startswith("attn_q8"):
        S, H, KV, Dh, pos, W = (int(x) for x in d["meta"])
        kq = np.zeros_like(d["kq"])
        ks = np.zeros_like(d["ks"])
        oracle.append_kv_q8(d["k"], kq, ks, 0)
        np.testing.assert_array_equal(kq, d["kq"])
        np.testing.assert_array_equal(ks, d["ks"])
        out = oracle.attention(d["q"], d["kq"], d["vq"], pos, W, oracle.KV_Q8_0, d["ks"], d["vs"])
        np.testing.assert_array_equal(out, d["out"])
    elif name.startswith("attn_layer"):
        S, H, KV, Dh, rot, pos, split = (int(x) for x in d["meta"])
        kq, ks, vq, vs = d["kq0"].copy(), d["ks0"].copy(), d["vq0"].copy(), d["vs0"].copy()
        q = np.ascontiguousarray(d["qg"][..., :Dh]) if split else d["qg"]
        gate = np.ascontiguousarray(d["qg"][..., Dh:]) if split else None
        q_out, out = oracle.attn_layer_step(q, d["k"], d["v"], d["qn"], d["kn"], float(d["eps"][0]), d["cos"],
                                            d["sin"], rot, pos, kq, ks, vq, vs, gate=gate)
        np.testing.assert_array_equal(q_out, d["q_out"])
        np.testing.assert_array_equal(out, d["out"])
        for a, b in ((kq, "kq"), (ks, "ks"), (vq, "vq"), (vs, "vs")):
            np.testing.assert_array_equal(a, d[b])
    elif name.startswith("attn_"):
        fmt, B, S, H, KV, Dh, W = (int(x) for x in d["meta"])
        out = oracle.attention_batch(d["q"], d["k"], d["v"], d["pos"], d["off"], W, fmt)
        np.testing.assert_array_equal(out, d["out"])
    elif name.startswith("conv1d"):
        S, C, K, ls = (int(x) for x in d["meta"])
        y, st = oracle.conv1d_causal(d["x"], d["w"], d["state"], bool(ls))
        np.testing.assert_array_equal(y, d["y"])
        np.testing.assert_array_equal(st, d["new_state"])
    elif name == "norm_gate":
        y = oracle.deltanet_norm_gate(d["core"], d["z"], d["gamma"], float(d["eps"][0]))
        np.testing.assert_array_equal(y, d["y"])
    elif name.startswith("gdn_layer"):
        B, NK, NV, D, K, ls = (int(x) for x in d["meta"])
        out, conv_new, st_new = oracle.gdn_layer_step(d["qkv"], d["conv_w"], d["conv_state"], d["a"], d["b"],
                                                      d["a_neg"], d["dt_bias"], d["z"], d["gamma"],
                                                      float(d["eps"][0]), d["state"], NK, NV, bool(ls))
        np.testing.assert_array_equal(out, d["out"])
        np.testing.assert_array_equal(conv_new, d["new_conv_state"])
        np.testing.assert_array_equal(st_new, d["new_state"])
    else:
        S, NK, NV, D, ls = (int(x) for x in d["meta"])
        gb = oracle.deltanet_gbeta(d["a"], d["b"], d["a_neg"], d["dt_bias"])
        np.testing.assert_array_equal(gb, d["gbeta"])
        core, st = oracle.deltanet_recur(d["qkv"], d["gbeta"], d["state"], NK, NV, bool(ls))
        np.testing.assert_array_equal(core, d["core"])
        np.testing.assert_array_equal(st, d["new_state"])


@pytest.mark.parametrize("window", [0, 5, 64])
@pytest.mark.parametrize("S", [1, 4])
def test_attention_matches_closed_form(S, window):
    rng = np.random.default_rng(7)
    H, KV, Dh, pos = 8, 2, 128, 60
    q = rng.standard_normal((S, H, Dh), dtype=np.float32)
    k = rng.standard_normal((pos + S, KV, Dh), dtype=np.float32)
    v = rng.standard_normal((pos + S, KV, Dh), dtype=np.float32)
    ref = oracle.closed_form.attention(q, k, v, pos, window)
    assert rel_l2(oracle.attention(q, k, v, pos, window), ref) < 1e-6


def test_attention_f16_bf16_decode_like_f32():
    rng = np.random.default_rng(8)
    H, KV, Dh, pos = 4, 2, 128, 30
    q = rng.standard_normal((1, H, Dh), dtype=np.float32)
    k = rng.standard_normal((pos + 1, KV, Dh), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((pos + 1, KV, Dh), dtype=np.float32).astype(np.float16)
    a16 = oracle.attention(q, k.view(np.uint16), v.view(np.uint16), pos, 0, oracle.KV_F16)
    a32 = oracle.attention(q, k.astype(np.float32), v.astype(np.float32), pos, 0, oracle.KV_F32)
    np.testing.assert_array_equal(a16, a32)
    kb = (k.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    vb = (v.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    abf = oracle.attention(q, kb, vb, pos, 0, oracle.KV_BF16)
    kf = (kb.astype(np.uint32) << 16).view(np.float32)
    vf = (vb.astype(np.uint32) << 16).view(np.float32)
    np.testing.assert_array_equal(abf, oracle.attention(q, kf, vf, pos, 0, oracle.KV_F32))


def test_f16_decode_matches_numpy():
    L = oracle.lib()
    for bits in [0, 1, 0x3ff, 0x400, 0x3c00, 0x7bff, 0x8001, 0xfbff, 0x7c00]:
        assert L.oracle_f16_to_f64(bits) == float(np.array([bits], np.uint16).view(np.float16)[0])


def test_q8_attention_js_and_wgsl_agree():
    rng = np.random.default_rng(9)
    S, H, KV, Dh, pos = 3, 4, 2, 128, 40
    k = rng.standard_normal((pos + S, KV, Dh), dtype=np.float32)
    v = rng.standard_normal((pos + S, KV, Dh), dtype=np.float32)
    q = rng.standard_normal((S, H, Dh), dtype=np.float32)
    kq = np.zeros((pos + S, KV, Dh), np.int8)
    ks = np.zeros((pos + S, KV, Dh // 32), np.float32)
    vq, vs = kq.copy(), ks.copy()
    oracle.append_kv_q8(k, kq, ks, 0)
    oracle.append_kv_q8(v, vq, vs, 0)
    for W in (0, 9):
        js = oracle.attention(q, kq, vq, pos, W, oracle.KV_Q8_0, ks, vs)
        wg = oracle.attention_q8_wgsl(q, kq, (ks * np.float32(127)).astype(np.float32), vq,
                                      (vs * np.float32(127)).astype(np.float32), pos, W)
        assert rel_l2(wg, js) < 1e-6
        kd = (kq.reshape(-1, 32) * ks.reshape(-1, 1).astype(np.float64)).reshape(k.shape)
        vd = (vq.reshape(-1, 32) * vs.reshape(-1, 1).astype(np.float64)).reshape(v.shape)
        assert rel_l2(js, oracle.closed_form.attention(q, kd, vd, pos, W)) < 1e-6


def test_append_q8_known_answers():
    # Math.round ties go toward +infinity: with amax = 127, x = +-2.5 maps to 3 / -2.
    src = np.zeros((1, 1, 32), np.float32)
    src[0, 0, :6] = [127.0, 2.5, -2.5, 0.5, -0.5, -127.0]
    cq = np.zeros((1, 1, 32), np.int8)
    cs = np.zeros((1, 1, 1), np.float32)
    oracle.append_kv_q8(src, cq, cs, 0)
    assert list(cq[0, 0, :6]) == [127, 3, -2, 1, 0, -127]
    assert cs[0, 0, 0] == np.float32(1.0)
    # An all-zero block stores scale 0 and zeros.
    oracle.append_kv_q8(np.zeros((1, 1, 32), np.float32), cq, cs, 0)
    assert cs[0, 0, 0] == 0 and not cq.any()


def test_attention_known_answers():
    Dh = 128
    q = np.zeros((1, 1, Dh), np.float32)
    v = np.arange(3 * Dh, dtype=np.float32).reshape(3, 1, Dh)
    k = np.zeros((3, 1, Dh), np.float32)
    # Equal scores: the mean of the values.
    out = oracle.attention(q, k, v, 2, 0)
    np.testing.assert_allclose(out[0, 0], v[:, 0].mean(0), rtol=1e-6)
    # Window 1: only the query's own key.
    out = oracle.attention(q, k, v, 2, 1)
    np.testing.assert_allclose(out[0, 0], v[2, 0], rtol=1e-6)


def test_deltanet_matches_closed_form_and_wgsl():
    rng = np.random.default_rng(10)
    T, NK, NV, D = 6, 2, 4, 128
    q = rng.standard_normal((T, NK, D), dtype=np.float32)
    k = rng.standard_normal((T, NK, D), dtype=np.float32)
    v = rng.standard_normal((T, NV, D), dtype=np.float32)
    qkv = np.concatenate([q.reshape(T, -1), k.reshape(T, -1), v.reshape(T, -1)], 1).astype(np.float32)
    a = rng.standard_normal((T, NV), dtype=np.float32)
    b = rng.standard_normal((T, NV), dtype=np.float32)
    gb = oracle.deltanet_gbeta(a, b, -np.ones(NV, np.float32), np.zeros(NV, np.float32))
    # alpha = exp(g) = exp(-softplus(a)), beta = sigmoid(b)
    np.testing.assert_allclose(np.exp(gb[0]), np.exp(-np.logaddexp(0, a.astype(np.float64))), rtol=1e-6)
    np.testing.assert_allclose(gb[1], 1 / (1 + np.exp(-b.astype(np.float64))), rtol=1e-6)
    st0 = (0.02 * rng.standard_normal((NV, D, D))).astype(np.float32)
    core, st = oracle.deltanet_recur(qkv, gb, st0, NK, NV, True)
    hmap = np.arange(NV) % NK  # tiled QK-head map (kernels.ts:1511)
    o, stc = oracle.closed_form.deltanet(q[:, hmap], k[:, hmap], v, gb[0], gb[1], st0)
    assert rel_l2(core, o) < 1e-6 and rel_l2(st, stc) < 1e-6
    cw, sw = oracle.deltanet_recur_wgsl(qkv, gb, st0, NK, NV, True)
    assert rel_l2(cw, core) < 1e-5 and rel_l2(sw, st) < 1e-5
    # loadState = 0 ignores the incoming state.
    c0, s0 = oracle.deltanet_recur(qkv, gb, st0, NK, NV, False)
    c1, s1 = oracle.deltanet_recur(qkv, gb, np.zeros_like(st0), NK, NV, True)
    np.testing.assert_array_equal(c0, c1)
    np.testing.assert_array_equal(s0, s1)


def test_deltanet_known_answer_single_step():
    # Zero state, alpha = 1, beta = 1, unit k = q = e0: S = e0 v^T, o = v / sqrt(D).
    D = 128
    qkv = np.zeros((1, 3 * D), np.float32)
    qkv[0, 0] = 1.0
    qkv[0, D] = 1.0
    qkv[0, 2 * D:] = np.arange(D, dtype=np.float32)
    gb = np.zeros((2, 1, 1), np.float32)
    gb[1] = 1.0
    core, st = oracle.deltanet_recur(qkv, gb, np.zeros((1, D, D), np.float32), 1, 1, True)
    kn = 1 / np.sqrt(1 + 1e-6)
    np.testing.assert_allclose(st[0, 0], np.arange(D) * kn, rtol=1e-6)
    np.testing.assert_allclose(core[0, 0], np.arange(D) * kn * kn / np.sqrt(D), rtol=1e-6)


def test_batch_drivers_match_single_calls():
    rng = np.random.default_rng(11)
    lens = np.array([3, 17, 9])
    off = np.concatenate([[0], np.cumsum(lens)[:-1]])
    k = rng.standard_normal((lens.sum(), 2, 128), dtype=np.float32)
    v = rng.standard_normal((lens.sum(), 2, 128), dtype=np.float32)
    q = rng.standard_normal((3, 1, 4, 128), dtype=np.float32)
    out = oracle.attention_batch(q, k, v, lens - 1, off, 0, oracle.KV_F32, threads=3)
    for b in range(3):
        ref = oracle.attention(q[b], k[off[b]:off[b] + lens[b]], v[off[b]:off[b] + lens[b]], lens[b] - 1)
        np.testing.assert_array_equal(out[b], ref)


@pytest.mark.parametrize("load", [True, False])
def test_conv1d_matches_closed_form(load):
    """conv1d_causal against a dense numpy f64 form: the extended sequence is
    the conv state (or zeros) followed by the inputs; each output is the SiLU
    of a K-tap dot; the new state is the last K-1 extended rows."""
    rng = np.random.default_rng(3 + load)
    S, C, K = 6, 40, 4
    x = rng.standard_normal((S, C), dtype=np.float32)
    w = rng.standard_normal((C, K), dtype=np.float32)
    st = rng.standard_normal((K - 1, C), dtype=np.float32)
    y, ns = oracle.conv1d_causal(x, w, st, load)
    ext = np.concatenate([st if load else np.zeros_like(st), x], 0).astype(np.float64)
    acc = np.stack([sum(w[:, j].astype(np.float64) * ext[t + j] for j in range(K)) for t in range(S)])
    np.testing.assert_allclose(y, acc / (1 + np.exp(-acc)), rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(ns, ext[S:].astype(np.float32))
    # a 1-token step shifts the state by one row and appends the token
    y1, ns1 = oracle.conv1d_causal(x[:1], w, st, True)
    np.testing.assert_array_equal(ns1, np.concatenate([st[1:], x[:1]], 0))


def test_norm_gate_matches_closed_form():
    rng = np.random.default_rng(9)
    core = rng.standard_normal((5, 128), dtype=np.float32)
    z = rng.standard_normal((5, 128), dtype=np.float32)
    gamma = rng.standard_normal(128, dtype=np.float32)
    y = oracle.deltanet_norm_gate(core, z, gamma, 1e-6)
    c = core.astype(np.float64)
    ref = gamma * c / np.sqrt((c * c).mean(1, keepdims=True) + np.float64(np.float32(1e-6))) * (z / (1 + np.exp(-z.astype(np.float64))))
    np.testing.assert_allclose(y, ref, rtol=1e-6, atol=1e-6)
    # known answer: a row of equal values normalises to 1 (eps aside), silu(0) = 0
    one = oracle.deltanet_norm_gate(np.full((1, 128), 3.0, np.float32), np.full((1, 128), 20.0, np.float32),
                                    np.ones(128, np.float32), 0.0)
    np.testing.assert_allclose(one, np.full((1, 128), 20.0 / (1 + np.exp(-20.0))), rtol=1e-7)
    zero = oracle.deltanet_norm_gate(core[:1], np.zeros((1, 128), np.float32), gamma, 1e-6)
    np.testing.assert_array_equal(zero, np.zeros((1, 128), np.float32))


def test_rmsnorm_rope_gate_match_closed_forms():
    """rmsnorm, RoPE and the sigmoid gate against dense numpy f64 forms, and
    RoPE's known answers: position 0 is the identity, and a rotation by pos
    then by -pos (the conjugate tables) restores the input."""
    rng = np.random.default_rng(21)
    x = rng.standard_normal((3, 4, 128), dtype=np.float32)
    g = rng.standard_normal(128, dtype=np.float32)
    y = oracle.rmsnorm(x, g, 1e-6)
    x64 = x.astype(np.float64)
    ref = x64 / np.sqrt((x64 * x64).mean(-1, keepdims=True) + np.float64(np.float32(1e-6))) * g
    np.testing.assert_allclose(y, ref, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(oracle.rmsnorm(x, g, 1e-6, True),
                               x64 / np.sqrt((x64 * x64).mean(-1, keepdims=True) + np.float64(np.float32(1e-6)))
                               * (1.0 + g), rtol=1e-6, atol=1e-6)
    for rot in (64, 128):
        cos, sin = oracle.rope_tables(rot, 16, 1e6)
        half = rot // 2
        r = oracle.rope(y, rot, 5, cos, sin)
        c, s_ = cos[5:8][:, None, :].astype(np.float64), sin[5:8][:, None, :].astype(np.float64)
        yy = y.astype(np.float64)
        exp = yy.copy()
        exp[..., :half] = yy[..., :half] * c - yy[..., half:rot] * s_
        exp[..., half:rot] = yy[..., half:rot] * c + yy[..., :half] * s_
        np.testing.assert_allclose(r, exp, rtol=1e-6, atol=1e-6)
        np.testing.assert_array_equal(oracle.rope(y[:1], rot, 0, cos, sin), y[:1])  # position 0: cos 1, sin 0
        back = oracle.rope(r, rot, 5, cos, -sin)
        np.testing.assert_allclose(back, y, rtol=1e-5, atol=1e-5)
    gate = rng.standard_normal(x.shape, dtype=np.float32)
    np.testing.assert_allclose(oracle.sigmoid_gate(gate, x), x64 / (1 + np.exp(-gate.astype(np.float64))),
                               rtol=1e-6, atol=1e-6)


def test_wgsl_q8_append_known_answers():
    """kv_append_q8's WGSL semantics (src/kernels.ts:1318-1333): round() ties
    to even where the JS Math.round goes up; the scale array holds
    (amax/127)*127 in f32; an all-zero block stores scale 0 and zeros."""
    src = np.zeros((1, 2, 32), np.float32)
    src[0, 0, :4] = [2.5, -2.5, 3.5, 127.0]  # amax 127 -> inv 1: the products are the values themselves
    qw, aw = np.zeros((1, 2, 32), np.int8), np.zeros((1, 2, 1), np.float32)
    qj, sj = np.zeros((1, 2, 32), np.int8), np.zeros((1, 2, 1), np.float32)
    oracle.append_kv_q8_wgsl(src, qw, aw, 0)
    oracle.append_kv_q8(src, qj, sj, 0)
    assert list(qw[0, 0, :4]) == [2, -2, 4, 127]
    assert list(qj[0, 0, :4]) == [3, -2, 4, 127]
    assert aw[0, 0, 0] == np.float32(np.float32(127.0) / np.float32(127.0)) * np.float32(127.0)
    assert sj[0, 0, 0] == np.float32(1.0)
    assert (qw[0, 1] == 0).all() and aw[0, 1, 0] == 0


def test_wgsl_and_js_q8_conventions_agree():
    """On random rows both conventions store the same int8 values up to a
    rare tie or last-bit difference, and their attention outputs agree."""
    rng = np.random.default_rng(5)
    rows, KV, Dh, H = 300, 2, 128, 4
    x = rng.standard_normal((rows, KV, Dh), dtype=np.float32)
    qw, aw = np.zeros((rows, KV, Dh), np.int8), np.zeros((rows, KV, Dh // 32), np.float32)
    qj, sj = np.zeros_like(qw), np.zeros_like(aw)
    oracle.append_kv_q8_wgsl(x, qw, aw, 0)
    oracle.append_kv_q8(x, qj, sj, 0)
    diff = np.abs(qw.astype(np.int32) - qj.astype(np.int32))
    assert diff.max() <= 1 and (diff > 0).mean() < 1e-3
    np.testing.assert_allclose(aw / 127.0, sj, rtol=1e-6)
    q = rng.standard_normal((1, H, Dh), dtype=np.float32)
    a = oracle.attention_q8_wgsl(q, qw, aw, qw, aw, rows - 1)
    b = oracle.attention(q, qw, qw, rows - 1, 0, oracle.KV_Q8_0, aw / np.float32(127), aw / np.float32(127))
    assert np.linalg.norm(a - b) / np.linalg.norm(b) < 1e-5

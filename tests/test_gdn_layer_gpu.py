"""GPU parity of the Gated DeltaNet layer's neighbours of the recurrence
against the oracle: conv1d_causal (src/kernels.ts:1431-1466), deltanet_norm_gate
(src/kernels.ts:1578-1611), through the reference's op names and the typed API,
and the fused single-token layer step (conv1d + g / beta + recurrence + gated
RMSNorm, src/engine.ts:1366-1400) at the configuration-4 shape.

Tolerance (fp32): relative L2 <= 1e-4; conv states moved without arithmetic are
bit-exact."""
import os

import numpy as np
import pytest
import torch

import oracle
from hachiue_b200 import _lib
from hachiue_b200.backend import HachiueError, f32_word
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
TOL = 1e-4
dev = "cuda"


def g(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def T(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


@pytest.mark.parametrize("name", ["conv1d_segment", "conv1d_fresh"])
def test_conv1d_golden_via_dispatch(backend, name):
    d = g(name)
    S, C, K, ls = (int(x) for x in d["meta"])
    y = torch.full((S, C), float("nan"), device=dev)
    st_out = torch.full((K - 1, C), float("nan"), device=dev)
    backend.dispatch("conv1d_causal", [S, C, K, ls], [T(d["x"]), T(d["w"]), T(d["state"]), y, st_out])
    torch.cuda.synchronize()
    assert rel_l2(y.cpu().numpy(), d["y"]) < TOL
    np.testing.assert_array_equal(st_out.cpu().numpy(), d["new_state"])
    # in place (the JS backend updates its conv state in place)
    st = T(d["state"])
    y2 = torch.zeros_like(y)
    backend.conv1d_causal(T(d["x"]), T(d["w"]), st, y2, st, bool(ls))
    torch.cuda.synchronize()
    assert rel_l2(y2.cpu().numpy(), d["y"]) < TOL
    np.testing.assert_array_equal(st.cpu().numpy(), d["new_state"])


@pytest.mark.parametrize("S,load", [(1, True), (2, True), (7, False)])
def test_conv1d_batched(backend, S, load):
    """A batch of sequences, S smaller and larger than the state length."""
    rng = np.random.default_rng(S + 100 * load)
    B, C, K = 5, 200, 4
    x = rng.standard_normal((B, S, C), dtype=np.float32)
    w = rng.standard_normal((C, K), dtype=np.float32)
    st = rng.standard_normal((B, K - 1, C), dtype=np.float32)
    y = torch.zeros((B, S, C), device=dev)
    st_out = torch.zeros((B, K - 1, C), device=dev)
    backend.conv1d_causal(T(x), T(w), T(st), y, st_out, load)
    torch.cuda.synchronize()
    for b in range(B):
        ref_y, ref_st = oracle.conv1d_causal(x[b], w, st[b], load)
        assert rel_l2(y[b].cpu().numpy(), ref_y) < TOL
        np.testing.assert_array_equal(st_out[b].cpu().numpy(), ref_st)


def test_norm_gate_golden_via_dispatch(backend):
    d = g("norm_gate")
    rows, DV = (int(x) for x in d["meta"])
    y = torch.full((rows, DV), float("nan"), device=dev)
    backend.dispatch("deltanet_norm_gate", [rows, DV, f32_word(float(d["eps"][0])), 0],
                     [T(d["core"]), T(d["z"]), T(d["gamma"]), y])
    torch.cuda.synchronize()
    assert rel_l2(y.cpu().numpy(), d["y"]) < TOL
    y2 = torch.zeros_like(y)
    backend.deltanet_norm_gate(T(d["core"]), T(d["z"]), T(d["gamma"]), y2, float(d["eps"][0]))
    torch.cuda.synchronize()
    assert rel_l2(y2.cpu().numpy(), d["y"]) < TOL


def run_layer(backend, d, NK, NV, ls, in_place_state=False):
    B = d["qkv"].shape[0]
    conv_out = torch.full(d["conv_state"].shape, float("nan"), device=dev)
    st_in = T(d["state"])
    st_out = st_in if in_place_state else torch.full(d["state"].shape, float("nan"), device=dev)
    out = torch.full((B, NV * 128), float("nan"), device=dev)
    backend.gdn_layer_step(T(d["qkv"]), T(d["conv_w"]), T(d["conv_state"]), conv_out, T(d["a"]), T(d["b"]),
                           T(d["a_neg"]), T(d["dt_bias"]), T(d["z"]), T(d["gamma"]), st_in, st_out, out, NK, NV,
                           float(d["eps"][0]), ls)
    torch.cuda.synchronize()
    return out.cpu().numpy(), conv_out.cpu().numpy(), st_out.cpu().numpy()


@pytest.mark.parametrize("name", ["gdn_layer_step", "gdn_layer_fresh"])
def test_layer_step_golden(backend, name):
    d = g(name)
    B, NK, NV, D, K, ls = (int(x) for x in d["meta"])
    out, conv_new, st_new = run_layer(backend, d, NK, NV, bool(ls))
    assert rel_l2(out, d["out"]) < TOL
    np.testing.assert_array_equal(conv_new, d["new_conv_state"])
    assert rel_l2(st_new, d["new_state"]) < TOL
    assert backend.device_status() == 0


def layer_case(rng, B, NK, NV, load):
    D, K = 128, 4
    C = 2 * NK * D + NV * D
    return dict(qkv=rng.standard_normal((B, C), dtype=np.float32),
                conv_w=(rng.standard_normal((C, K), dtype=np.float32) * np.float32(0.5)).astype(np.float32),
                conv_state=rng.standard_normal((B, K - 1, C), dtype=np.float32),
                a=rng.standard_normal((B, NV), dtype=np.float32), b=rng.standard_normal((B, NV), dtype=np.float32),
                a_neg=-np.ones(NV, np.float32), dt_bias=np.zeros(NV, np.float32),
                z=rng.standard_normal((B, NV * D), dtype=np.float32),
                gamma=(1 + rng.standard_normal(D, dtype=np.float32) * np.float32(0.1)).astype(np.float32),
                state=(rng.standard_normal((B, NV, D, D), dtype=np.float32) * np.float32(0.02)).astype(np.float32),
                eps=np.array([1e-6], np.float32))


@pytest.mark.parametrize("B,NK,NV,in_place", [(64, 16, 32, True), (3, 4, 6, False), (150, 2, 2, True)])
def test_layer_step_against_the_oracle_pipeline(backend, B, NK, NV, in_place):
    """Configuration 4's shape (64 sequences, 16 / 32 heads, states updated in
    place), a head map where some QK heads serve one V head and others two, and
    300 items so that CTAs of the persistent kernel take several."""
    rng = np.random.default_rng(B + NK + NV)
    d = layer_case(rng, B, NK, NV, True)
    out, conv_new, st_new = run_layer(backend, d, NK, NV, True, in_place_state=in_place)
    ref_out, ref_conv, ref_st = oracle.gdn_layer_step(d["qkv"], d["conv_w"], d["conv_state"], d["a"], d["b"],
                                                      d["a_neg"], d["dt_bias"], d["z"], d["gamma"], 1e-6,
                                                      d["state"], NK, NV, True)
    assert rel_l2(out, ref_out) < TOL
    np.testing.assert_array_equal(conv_new, ref_conv)
    assert rel_l2(st_new, ref_st) < TOL
    assert backend.device_status() == 0


def test_layer_step_needs_ping_pong_conv_state(backend):
    rng = np.random.default_rng(1)
    d = layer_case(rng, 2, 1, 2, True)
    conv = T(d["conv_state"])
    st = T(d["state"])
    out = torch.zeros((2, 256), device=dev)
    with pytest.raises(HachiueError, match="ping-pong") as e:
        backend.gdn_layer_step(T(d["qkv"]), T(d["conv_w"]), conv, conv, T(d["a"]), T(d["b"]), T(d["a_neg"]),
                               T(d["dt_bias"]), T(d["z"]), T(d["gamma"]), st, st, out, 1, 2, 1e-6, True)
    assert e.value.status == _lib.HCU_EINVAL

"""GPU parity of the Gated DeltaNet recurrence against the oracle.

Tolerance (fp32 recurrence): relative L2 <= 1e-4 on outputs and states."""
import os

import numpy as np
import pytest
import torch

import oracle
from hachiue_b200 import workloads
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
TOL = 1e-4
dev = "cuda"


def g(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def T(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


@pytest.mark.parametrize("name", ["gdn_decode", "gdn_segment_fresh"])
def test_golden_via_dispatch(backend, name):
    """deltanet_gbeta then deltanet_recur with ping-pong states, as
    forwardSegment dispatches them (src/engine.ts:1377-1396)."""
    d = g(name)
    S, NK, NV, D, ls = (int(x) for x in d["meta"])
    gb = torch.zeros((2, S, NV), device=dev)
    backend.dispatch("deltanet_gbeta", [S, NV, 0, 0], [T(d["a"]), T(d["b"]), T(d["a_neg"]), T(d["dt_bias"]), gb])
    st_in, st_out = T(d["state"]), torch.zeros((NV, D, D), device=dev)
    core = torch.zeros((S, NV, D), device=dev)
    backend.dispatch("deltanet_recur", [S, NV, D, D, NK, ls, 0, 0], [T(d["qkv"]), gb, st_in, core, st_out])
    torch.cuda.synchronize()
    assert rel_l2(gb.cpu().numpy(), d["gbeta"]) < 1e-6
    assert rel_l2(core.cpu().numpy(), d["core"]) < TOL
    assert rel_l2(st_out.cpu().numpy(), d["new_state"]) < TOL
    # the fused g/beta path gives the same answer, in place
    st = T(d["state"])
    core2 = torch.zeros_like(core)
    backend.deltanet_decode(T(d["qkv"]), T(d["a"]), T(d["b"]), T(d["a_neg"]), T(d["dt_bias"]), st, core2, st, NK, NV,
                            bool(ls))
    torch.cuda.synchronize()
    assert rel_l2(core2.cpu().numpy(), d["core"]) < TOL
    assert rel_l2(st.cpu().numpy(), d["new_state"]) < TOL


def test_cfg4_qwen35_gdn_decode_step(backend):
    w = workloads.gdn_decode_cfg4()
    B, NK, NV, D = 64, w["NK"], w["NV"], w["D"]
    st = T(w["state"])
    core = torch.zeros((B, 1, NV, D), device=dev)
    backend.deltanet_decode(T(w["qkv"]), T(w["a"]), T(w["b"]), T(w["a_neg"]), T(w["dt_bias"]), st, core, st, NK, NV)
    torch.cuda.synchronize()
    gb = np.stack([oracle.deltanet_gbeta(w["a"][b], w["b"][b], w["a_neg"], w["dt_bias"]) for b in range(B)])
    ref_core, ref_st = oracle.deltanet_recur_batch(w["qkv"], gb, w["state"], NK, NV, True)
    assert rel_l2(core.cpu().numpy(), ref_core) < TOL
    assert rel_l2(st.cpu().numpy(), ref_st) < TOL


@pytest.mark.parametrize("S,load", [(1, False), (3, True), (17, True)])
def test_segments_batched(backend, S, load):
    rng = np.random.default_rng(S + 10 * load)
    B, NK, NV, D = 3, 2, 4, 128
    conv = 2 * NK * D + NV * D
    qkv = rng.standard_normal((B, S, conv), dtype=np.float32)
    a = rng.standard_normal((B, S, NV), dtype=np.float32)
    b = rng.standard_normal((B, S, NV), dtype=np.float32)
    a_neg = -np.ones(NV, np.float32)
    dtb = np.zeros(NV, np.float32)
    st0 = (0.02 * rng.standard_normal((B, NV, D, D))).astype(np.float32)
    gb = np.stack([oracle.deltanet_gbeta(a[i], b[i], a_neg, dtb) for i in range(B)])
    ref_core, ref_st = oracle.deltanet_recur_batch(qkv, gb, st0, NK, NV, load)
    st_out = torch.zeros((B, NV, D, D), device=dev)
    core = torch.zeros((B, S, NV, D), device=dev)
    backend.deltanet_recur(T(qkv), T(gb), T(st0), core, st_out, NK, NV, load)
    torch.cuda.synchronize()
    assert rel_l2(core.cpu().numpy(), ref_core) < TOL
    assert rel_l2(st_out.cpu().numpy(), ref_st) < TOL


def test_single_token_items_chain(backend):
    """S = 1 runs on the persistent step kernel (two CTAs per SM, the next
    item's state prefetched by bulk copy): 80 sequences x 4 V heads = 320
    items give some CTAs two items, through the non-fused entry point with a
    loaded state."""
    rng = np.random.default_rng(77)
    B, S, NK, NV, D = 80, 1, 2, 4, 128
    conv = 2 * NK * D + NV * D
    qkv = rng.standard_normal((B, S, conv), dtype=np.float32)
    a = rng.standard_normal((B, S, NV), dtype=np.float32)
    b = rng.standard_normal((B, S, NV), dtype=np.float32)
    a_neg = -np.ones(NV, np.float32)
    dtb = np.zeros(NV, np.float32)
    st0 = (0.02 * rng.standard_normal((B, NV, D, D))).astype(np.float32)
    gb = np.stack([oracle.deltanet_gbeta(a[i], b[i], a_neg, dtb) for i in range(B)])
    ref_core, ref_st = oracle.deltanet_recur_batch(qkv, gb, st0, NK, NV, True)
    st_out = torch.zeros((B, NV, D, D), device=dev)
    core = torch.zeros((B, S, NV, D), device=dev)
    backend.deltanet_recur(T(qkv), T(gb), T(st0), core, st_out, NK, NV, True)
    torch.cuda.synchronize()
    assert rel_l2(core.cpu().numpy(), ref_core) < TOL
    assert rel_l2(st_out.cpu().numpy(), ref_st) < TOL
    assert backend.device_status() == 0

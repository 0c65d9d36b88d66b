"""GPU parity of the chunked (WY-form, tensor-core) Gated DeltaNet prefill
against the oracle's token-serial f32 recurrence (src/wasm-backend.ts
:1047-1102 semantics).  Tolerance (bf16 tensor-core path): relative L2 <= 1e-2
and max-abs <= 2e-2 on outputs and final states."""
import numpy as np
import pytest
import torch

import oracle
from hachiue_b200 import workloads
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu
REL, ABS = 1e-2, 2e-2
dev = "cuda"


def bf16_bits(x):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def to_dev_bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(dev).view(torch.bfloat16)


def oracle_head(qb, kb, vb, g, beta, b, h, NK, state0=None):
    """Token-serial oracle for one (sequence, V head): builds the reference's
    qkvConv rows for QK head h % NK and that V head."""
    hk = h % NK
    q = workloads.bf16_bits_to_f32(qb[b, :, hk])
    k = workloads.bf16_bits_to_f32(kb[b, :, hk])
    v = workloads.bf16_bits_to_f32(vb[b, :, h])
    T, D = q.shape
    qkv = np.concatenate([q, k, v], 1).astype(np.float32)
    gb = np.stack([g[b, :, h:h + 1], beta[b, :, h:h + 1]]).astype(np.float32)
    st = np.zeros((1, D, D), np.float32) if state0 is None else state0[b, h:h + 1].copy()
    core, st1 = oracle.deltanet_recur(qkv, gb, st, 1, 1, state0 is not None)
    return core[:, 0], st1[0]


def make_inputs(rng, B, T, NK, NV, decay=1.0):
    q = rng.standard_normal((B, T, NK, 128), dtype=np.float32)
    k = rng.standard_normal((B, T, NK, 128), dtype=np.float32)
    v = rng.standard_normal((B, T, NV, 128), dtype=np.float32)
    a = rng.standard_normal((B, T, NV)).astype(np.float64)
    g = (-decay * (np.maximum(a, 0) + np.log1p(np.exp(-np.abs(a))))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((B, T, NV))))).astype(np.float32)
    return bf16_bits(q), bf16_bits(k), bf16_bits(v), g, beta


@pytest.fixture(params=[64, 128])
def chain_cols(backend, request):
    """Both widths of the recurrence kernel's CTAs (64 or 128 value columns;
    the library picks one by occupancy), forced through HCU_OPT_GDN_CHAIN_COLS."""
    backend.set_option("gdn_chain_cols", request.param)
    yield request.param
    backend.set_option("gdn_chain_cols", 0)


def run(backend, qb, kb, vb, g, beta, state0=None):
    B, T, NK, _ = qb.shape
    NV = vb.shape[2]
    core = torch.full((B, T, NV, 128), float("nan"), device=dev)
    st = torch.zeros((B, NV, 128, 128), device=dev)
    sin = None if state0 is None else torch.from_numpy(state0).to(dev)
    backend.deltanet_chunked_prefill(to_dev_bf16(qb), to_dev_bf16(kb), to_dev_bf16(vb), torch.from_numpy(g).to(dev),
                                     torch.from_numpy(beta).to(dev), core, st, sin)
    torch.cuda.synchronize()
    return core.cpu().numpy(), st.cpu().numpy()


@pytest.mark.parametrize("B,T,NK,NV,decay,load", [(1, 64, 1, 2, 1.0, False), (2, 200, 2, 4, 1.0, True),
                                                  (1, 1000, 1, 2, 1.0, False), (1, 640, 2, 2, 0.02, True),
                                                  (1, 129, 1, 1, 0.0, False), (1, 256, 1, 2, 4.0, True),
                                                  (1, 130, 2, 3, 1.0, False)])
def test_small_shapes(backend, chain_cols, B, T, NK, NV, decay, load):
    """One chunk, a partial last chunk, many chunks, weak decay (the state
    carries across chunks), no decay at all and strong decay (in-chunk decay
    factors far below f32 range); zero or loaded initial state; V heads not a
    multiple of twice the QK heads."""
    rng = np.random.default_rng(B + T + NK + NV + int(100 * decay))
    qb, kb, vb, g, beta = make_inputs(rng, B, T, NK, NV, decay)
    st0 = (0.02 * rng.standard_normal((B, NV, 128, 128))).astype(np.float32) if load else None
    core, st = run(backend, qb, kb, vb, g, beta, st0)
    assert np.isfinite(core).all() and np.isfinite(st).all()
    for b in range(B):
        for h in range(NV):
            rc, rs = oracle_head(qb, kb, vb, g, beta, b, h, NK, st0)
            assert rel_l2(core[b, :, h], rc) < REL, (b, h, rel_l2(core[b, :, h], rc))
            assert np.abs(core[b, :, h] - rc).max() < ABS
            assert rel_l2(st[b, h], rs) < REL
    assert backend.device_status() == 0


def test_agrees_with_recurrent_kernel(backend, chain_cols):
    """Same inputs through the token-serial CUDA kernel (hcu_deltanet_recur)."""
    rng = np.random.default_rng(42)
    B, T, NK, NV = 1, 300, 2, 4
    qb, kb, vb, g, beta = make_inputs(rng, B, T, NK, NV)
    core, st = run(backend, qb, kb, vb, g, beta)
    f = workloads.bf16_bits_to_f32
    qkv = np.concatenate([f(qb).reshape(B, T, -1), f(kb).reshape(B, T, -1), f(vb).reshape(B, T, -1)], 2)
    gb = np.stack([g, beta], 1)  # [B, 2, T, NV]
    core2 = torch.zeros((B, T, NV, 128), device=dev)
    st2 = torch.zeros((B, NV, 128, 128), device=dev)
    backend.deltanet_recur(torch.from_numpy(np.ascontiguousarray(qkv)).to(dev),
                           torch.from_numpy(np.ascontiguousarray(gb)).to(dev), st2, core2, st2, NK, NV, False)
    torch.cuda.synchronize()
    assert rel_l2(core, core2.cpu().numpy()) < REL
    assert rel_l2(st, st2.cpu().numpy()) < REL


@pytest.fixture(scope="module")
def cfg5():
    return workloads.gdn_prefill_cfg5()


def test_cfg5_qwen35_chunked_prefill(backend, cfg5):
    """Full config 5 (8 x 8192, 16 QK / 32 V heads, zero initial state); the
    oracle checks all outputs and final states of four (sequence, head) pairs."""
    w = cfg5
    core, st = run(backend, w["q"], w["k"], w["v"], w["g"], w["beta"])
    assert np.isfinite(core).all() and np.isfinite(st).all()
    for b, h in ((0, 0), (0, 17), (5, 3), (7, 31)):
        rc, rs = oracle_head(w["q"], w["k"], w["v"], w["g"], w["beta"], b, h, 16)
        assert rel_l2(core[b, :, h], rc) < REL, (b, h)
        assert np.abs(core[b, :, h] - rc).max() < ABS
        assert rel_l2(st[b, h], rs) < REL


def test_cfg5_whole_output_against_recurrent_kernel(backend, cfg5):
    """Every output and final state of config 5 (8 sequences x 8192 tokens x
    32 V heads) against the token-serial f32 CUDA kernel (hcu_deltanet_recur,
    itself checked against the oracle at 1e-4) on the same bf16-rounded inputs."""
    w = cfg5
    B, T, NK, NV = 8, 8192, 16, 32
    q, k, v = to_dev_bf16(w["q"]), to_dev_bf16(w["k"]), to_dev_bf16(w["v"])
    g, beta = torch.from_numpy(w["g"]).to(dev), torch.from_numpy(w["beta"]).to(dev)
    core = torch.full((B, T, NV, 128), float("nan"), device=dev)
    st = torch.zeros((B, NV, 128, 128), device=dev)
    backend.deltanet_chunked_prefill(q, k, v, g, beta, core, st)
    qkv = torch.cat([q.float().flatten(2), k.float().flatten(2), v.float().flatten(2)], 2).contiguous()
    gb = torch.stack([g, beta], 1).contiguous()  # [B, 2, T, NV]
    core2 = torch.zeros((B, T, NV, 128), device=dev)
    st2 = torch.zeros((B, NV, 128, 128), device=dev)
    backend.deltanet_recur(qkv, gb, st2, core2, st2, NK, NV, False)
    torch.cuda.synchronize()
    assert bool(torch.isfinite(core).all()) and bool(torch.isfinite(st).all())
    for b in range(B):
        d = core[b] - core2[b]
        assert float(d.norm() / core2[b].norm()) < REL, b
        assert float(d.abs().max()) < ABS, b
        assert float((st[b] - st2[b]).norm() / st2[b].norm()) < REL, b
    assert backend.device_status() == 0


def test_slabs_carry_the_state(backend, chain_cols, request):
    """A scratch budget of 1 MiB splits 64 chunks into slabs (one prep + chain
    launch pair each); the state crosses slab boundaries through state_out."""
    backend.set_option("gdn_scratch_mb", 1)
    request.addfinalizer(lambda: backend.set_option("gdn_scratch_mb", 0))
    rng = np.random.default_rng(7)
    B, T, NK, NV = 1, 4096, 1, 2
    qb, kb, vb, g, beta = make_inputs(rng, B, T, NK, NV, 0.05)
    st0 = (0.02 * rng.standard_normal((B, NV, 128, 128))).astype(np.float32)
    core, st = run(backend, qb, kb, vb, g, beta, st0)
    for h in range(NV):
        rc, rs = oracle_head(qb, kb, vb, g, beta, 0, h, NK, st0)
        assert rel_l2(core[0, :, h], rc) < REL, (h, rel_l2(core[0, :, h], rc))
        assert rel_l2(st[0, h], rs) < REL
    assert backend.device_status() == 0


def test_state_snapshots_for_prefix_reuse(backend, chain_cols):
    """Snapshots every 4 chunks: each equals, bit for bit, the final state of a
    prefill over that prefix; resuming from a snapshot reproduces the rest of
    the full prefill's outputs and its final state bit for bit (the restore
    path that lets a hybrid model keep a diverging prompt's common prefix,
    where the reference resets, src/engine.ts:1580-1584)."""
    rng = np.random.default_rng(77)
    B, T, NK, NV, every = 2, 1000, 2, 4, 4
    qb, kb, vb, g, beta = make_inputs(rng, B, T, NK, NV, 0.5)
    st0 = (0.02 * rng.standard_normal((B, NV, 128, 128))).astype(np.float32)
    q, k, v = to_dev_bf16(qb), to_dev_bf16(kb), to_dev_bf16(vb)
    gd, bd = torch.from_numpy(g).to(dev), torch.from_numpy(beta).to(dev)
    s0 = torch.from_numpy(st0).to(dev)
    n_snap = T // (64 * every)
    assert n_snap == 3
    core = torch.full((B, T, NV, 128), float("nan"), device=dev)
    st = torch.zeros((B, NV, 128, 128), device=dev)
    snaps = torch.full((B, n_snap, NV, 128, 128), float("nan"), device=dev)
    backend.deltanet_chunked_prefill(q, k, v, gd, bd, core, st, s0, snapshots=snaps, snap_every=every)
    # the plain entry point gives the same outputs
    core_plain = torch.empty_like(core)
    st_plain = torch.empty_like(st)
    backend.deltanet_chunked_prefill(q, k, v, gd, bd, core_plain, st_plain, s0)
    torch.cuda.synchronize()
    assert torch.equal(core, core_plain) and torch.equal(st, st_plain)
    for j in range(n_snap):
        Tp = 64 * every * (j + 1)
        c_p = torch.empty((B, Tp, NV, 128), device=dev)
        s_p = torch.empty_like(st)
        backend.deltanet_chunked_prefill(q[:, :Tp], k[:, :Tp], v[:, :Tp], gd[:, :Tp], bd[:, :Tp], c_p, s_p, s0)
        torch.cuda.synchronize()
        assert torch.equal(snaps[:, j], s_p), j
        assert torch.equal(c_p, core[:, :Tp]), j
    # resume after snapshot 1 (token 512) and finish the prompt
    t1 = 64 * every * 2
    c_r = torch.empty((B, T - t1, NV, 128), device=dev)
    s_r = torch.empty_like(st)
    backend.deltanet_chunked_prefill(q[:, t1:], k[:, t1:], v[:, t1:], gd[:, t1:], bd[:, t1:], c_r, s_r,
                                     snaps[:, 1].contiguous())
    torch.cuda.synchronize()
    assert torch.equal(c_r, core[:, t1:])
    assert torch.equal(s_r, st)
    # and against the oracle, one head
    rc, rs = oracle_head(qb, kb, vb, g, beta, 1, 3, NK, st0)
    assert rel_l2(core[1, :, 3].cpu().numpy(), rc) < REL
    assert backend.device_status() == 0


def test_snapshot_arguments_are_checked(backend):
    from hachiue_b200._lib import HachiueError
    rng = np.random.default_rng(5)
    qb, kb, vb, g, beta = make_inputs(rng, 1, 256, 1, 2)
    core = torch.empty((1, 256, 2, 128), device=dev)
    st = torch.empty((1, 2, 128, 128), device=dev)
    with pytest.raises(HachiueError):  # wrong snapshot count for T = 256, every = 2
        backend.deltanet_chunked_prefill(to_dev_bf16(qb), to_dev_bf16(kb), to_dev_bf16(vb),
                                         torch.from_numpy(g).to(dev), torch.from_numpy(beta).to(dev), core, st,
                                         snapshots=torch.empty((1, 3, 2, 128, 128), device=dev), snap_every=2)
    with pytest.raises(HachiueError):  # snap_every 0 with a buffer: refused by the C entry point
        backend.deltanet_chunked_prefill(to_dev_bf16(qb), to_dev_bf16(kb), to_dev_bf16(vb),
                                         torch.from_numpy(g).to(dev), torch.from_numpy(beta).to(dev), core, st,
                                         snapshots=torch.empty((1, 0, 2, 128, 128), device=dev), snap_every=0)


def test_chain_width_option_is_checked(backend):
    from hachiue_b200 import HachiueError
    with pytest.raises(HachiueError, match="HCU_OPT_GDN_CHAIN_COLS"):
        backend.set_option("gdn_chain_cols", 96)

"""GPU parity of the attention path against the oracle (through the C ABI).

Tolerance (fp32 decode paths): relative L2 <= 1e-4.  Q8_0 appends are
bit-exact (int8 values and f32 scales)."""
import os

import numpy as np
import pytest
import torch

import oracle
from hachiue_b200 import KV_BF16, KV_F16, KV_F32, KV_Q8_0, KV_Q8_0_WGSL, HachiueError, workloads
from hachiue_b200.backend import KVCache
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
TOL = 1e-4
dev = "cuda"


def g(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def T(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    return t if dtype is None else t.view(dtype)


@pytest.mark.parametrize("name", ["attn_q8_decode", "attn_q8_segment", "attn_q8_swa", "attn_q8_dh256"])
def test_q8_engine_sequence_via_dispatch(backend, name):
    """kv_append_q8 x2 then attention_q8, as forwardSegment dispatches them
    (src/engine.ts:1305-1317), over several segments of the golden case."""
    d = g(name)
    S, H, KV, Dh, pos, W = (int(x) for x in d["meta"])
    rows = pos + S
    cache = KVCache.allocate(rows, KV, Dh, KV_Q8_0)
    # history rows first (one segment), then the case's own S rows
    kf, vf = T(d["k"]), T(d["v"])
    for lo, hi in ((0, pos), (pos, rows)):
        if hi > lo:
            for src, q8, sc in ((kf, cache.k, cache.k_scale), (vf, cache.v, cache.v_scale)):
                backend.dispatch("kv_append_q8", [hi - lo, KV, Dh, lo], [src[lo:hi].contiguous(), q8, sc])
    out = torch.zeros((S, H, Dh), device=dev)
    backend.dispatch("attention_q8", [S, H, KV, Dh, pos, W, 0, 0],
                     [T(d["q"]), cache.k, cache.k_scale, cache.v, cache.v_scale, out])
    torch.cuda.synchronize()
    np.testing.assert_array_equal(cache.k.cpu().numpy(), d["kq"])
    np.testing.assert_array_equal(cache.k_scale.cpu().numpy(), d["ks"])
    np.testing.assert_array_equal(cache.v.cpu().numpy(), d["vq"])
    np.testing.assert_array_equal(cache.v_scale.cpu().numpy(), d["vs"])
    assert rel_l2(out.cpu().numpy(), d["out"]) < TOL
    assert backend.device_status() == 0


@pytest.mark.parametrize("name,fmt,tdt", [("attn_f32_batch", KV_F32, None), ("attn_f16_batch", KV_F16, torch.float16),
                                          ("attn_bf16_batch", KV_BF16, torch.bfloat16)])
def test_dense_batches_golden(backend, name, fmt, tdt):
    d = g(name)
    _, B, S, H, KV, Dh, W = (int(x) for x in d["meta"])
    k = T(d["k"].view(np.int16) if tdt is not None else d["k"], tdt)
    v = T(d["v"].view(np.int16) if tdt is not None else d["v"], tdt)
    cache = KVCache(fmt, k, v)
    out = torch.zeros((B, S, H, Dh), device=dev)
    backend.attention(T(d["q"]), cache, out, T(d["pos"]), W, kv_row_offset=T(d["off"]),
                      max_context=int(d["lens"].max()))
    torch.cuda.synchronize()
    assert rel_l2(out.cpu().numpy(), d["out"]) < TOL


def test_cfg1_qwen3_1p7b_decode(backend):
    w = workloads.decode_cfg1()
    cache = KVCache(KV_F32, T(w["k"]), T(w["v"]))
    out = torch.zeros((1, 16, 128), device=dev)
    backend.attention(T(w["q"]), cache, out, w["pos_base"])
    ref = oracle.attention(w["q"], w["k"], w["v"], w["pos_base"])
    assert rel_l2(out.cpu().numpy(), ref) < TOL


@pytest.fixture(scope="module")
def cfg2():
    return workloads.decode_cfg2()


def test_cfg2_qwen3_8b_batched_decode(backend, cfg2):
    w = cfg2
    k = T(w["k"].view(np.int16), torch.float16)
    v = T(w["v"].view(np.int16), torch.float16)
    cache = KVCache(KV_F16, k, v)
    out = torch.zeros((64, 1, 32, 128), device=dev)
    run = lambda: backend.attention(T(w["q"]), cache, out, T(w["pos_base"]), 0,  # noqa: E731
                                    kv_row_offset=T(w["row_offset"]), max_context=int(w["lens"].max()))
    run()
    first = out.cpu().numpy()
    out.zero_()
    run()  # second call: the split-merge tickets must have re-armed
    second = out.cpu().numpy()
    np.testing.assert_array_equal(first, second)
    assert np.isfinite(first).all()
    # the oracle on every sequence of the batch (runAttentionQ8's loop over an
    # f16 cache, the sequences on all host threads)
    lens = w["lens"]
    ref = oracle.attention_batch(w["q"], w["k"].view(np.uint16), w["v"].view(np.uint16), w["pos_base"],
                                 w["row_offset"], 0, oracle.KV_F16)
    for b in range(64):
        assert rel_l2(first[b], ref[b]) < TOL, b
    assert rel_l2(first, ref) < TOL


@pytest.mark.parametrize("H,KV,Dh", [(4, 4, 128), (32, 2, 128), (16, 2, 256), (8, 1, 256)])
@pytest.mark.parametrize("fmt", [KV_F32, KV_F16, KV_BF16, KV_Q8_0])
def test_head_layouts_and_formats(backend, H, KV, Dh, fmt):
    rng = np.random.default_rng(H * 100 + KV + Dh + fmt)
    rows = 300
    q = rng.standard_normal((1, H, Dh), dtype=np.float32)
    kf = rng.standard_normal((rows, KV, Dh), dtype=np.float32)
    vf = rng.standard_normal((rows, KV, Dh), dtype=np.float32)
    cache = KVCache.allocate(rows, KV, Dh, fmt)
    backend.kv_append(T(kf), cache, "k", 0)
    backend.kv_append(T(vf), cache, "v", 0)
    out = torch.zeros((1, H, Dh), device=dev)
    pos = rows - 1
    backend.attention(T(q), cache, out, pos)
    torch.cuda.synchronize()
    if fmt == KV_Q8_0:
        kk, vv = cache.k.cpu().numpy(), cache.v.cpu().numpy()
        ref = oracle.attention(q, kk, vv, pos, 0, KV_Q8_0, cache.k_scale.cpu().numpy(), cache.v_scale.cpu().numpy())
    else:
        kk = cache.k.view(torch.int16).cpu().numpy().view(np.uint16) if fmt != KV_F32 else cache.k.cpu().numpy()
        vv = cache.v.view(torch.int16).cpu().numpy().view(np.uint16) if fmt != KV_F32 else cache.v.cpu().numpy()
        if fmt == KV_F16:
            np.testing.assert_array_equal(kk, kf.astype(np.float16).view(np.uint16))
        ref = oracle.attention(q, kk, vv, pos, 0, fmt)
    assert rel_l2(out.cpu().numpy(), ref) < TOL


@pytest.mark.parametrize("S,pos,W", [(1, 0, 0), (5, 0, 0), (16, 100, 0), (12, 700, 64), (40, 250, 33), (3, 2, 1)])
def test_segments_and_windows(backend, S, pos, W):
    """Prefill segments (S > 1), the first token (posBase 0), sliding windows
    smaller than a segment, and window 1."""
    rng = np.random.default_rng(S * 1000 + pos + W)
    H, KV, Dh = 16, 4, 128
    rows = pos + S
    q = rng.standard_normal((S, H, Dh), dtype=np.float32)
    k = rng.standard_normal((rows, KV, Dh), dtype=np.float32)
    v = rng.standard_normal((rows, KV, Dh), dtype=np.float32)
    cache = KVCache(KV_F32, T(k), T(v))
    out = torch.zeros((S, H, Dh), device=dev)
    backend.attention(T(q), cache, out, pos, W)
    ref = oracle.attention(q, k, v, pos, W)
    assert rel_l2(out.cpu().numpy(), ref) < TOL


def test_long_context_many_splits(backend):
    rng = np.random.default_rng(5)
    rows, H, KV, Dh = 20000, 8, 2, 128
    q = rng.standard_normal((1, H, Dh), dtype=np.float32)
    k = rng.standard_normal((rows, KV, Dh), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((rows, KV, Dh), dtype=np.float32).astype(np.float16)
    cache = KVCache(KV_F16, T(k.view(np.int16), torch.float16), T(v.view(np.int16), torch.float16))
    out = torch.zeros((1, H, Dh), device=dev)
    backend.attention(T(q), cache, out, rows - 1)
    ref = oracle.attention(q, k.view(np.uint16), v.view(np.uint16), rows - 1, 0, KV_F16)
    assert rel_l2(out.cpu().numpy(), ref) < TOL


def test_errors_are_reported(backend):
    cache = KVCache.allocate(8, 2, 128, KV_F32)
    out = torch.zeros((1, 4, 128), device=dev)
    with pytest.raises(HachiueError, match="cache holds 8 rows"):
        backend.attention(torch.zeros((1, 4, 128), device=dev), cache, out, 8)
    with pytest.raises(HachiueError, match="Dh=64"):
        backend.attention(torch.zeros((1, 4, 64), device=dev), KVCache.allocate(8, 2, 64, KV_F32),
                          torch.zeros((1, 4, 64), device=dev), 3)
    with pytest.raises(HachiueError, match="missing pipeline"):
        backend.dispatch("gemv_q4_k", [1, 2, 3], [out])
    backend.inject_failure(5, 1)
    with pytest.raises(HachiueError, match="injected"):
        backend.attention(torch.zeros((1, 4, 128), device=dev), cache, out, 3)
    backend.attention(torch.zeros((1, 4, 128), device=dev), cache, out, 3)  # recovers
    torch.cuda.synchronize()


@pytest.mark.parametrize("impl", ["tc", "cuda"])
@pytest.mark.parametrize("fmt", [KV_F16, KV_BF16])
@pytest.mark.parametrize("H,KV,S,pos,W", [(32, 8, 1, 4000, 0), (16, 4, 3, 700, 0), (8, 2, 5, 1000, 300),
                                          (4, 4, 1, 129, 0), (16, 2, 1, 2049, 0), (12, 3, 2, 63, 17)])
def test_tensor_core_and_cuda_core_paths(backend, request, impl, fmt, H, KV, S, pos, W):
    """The tcgen05 kernel (default for f16 / bf16, Dh=128) and the CUDA-core
    kernel (option attn_cuda_cores) against the oracle: GQA groups 1-8, S > 1,
    windows, tile-edge context lengths."""
    backend.set_option("attn_cuda_cores", int(impl == "cuda"))
    request.addfinalizer(lambda: backend.set_option("attn_cuda_cores", 0))
    rng = np.random.default_rng(H + KV + S + pos + W + fmt)
    rows = pos + S
    q = rng.standard_normal((S, H, 128), dtype=np.float32)
    kf = rng.standard_normal((rows, KV, 128), dtype=np.float32)
    vf = rng.standard_normal((rows, KV, 128), dtype=np.float32)
    # capacity past the context holds NaN: masked rows must never reach the output
    cache = KVCache.allocate(rows + 200, KV, 128, fmt)
    cache.k.fill_(float("nan"))
    cache.v.fill_(float("nan"))
    backend.kv_append(T(kf), cache, "k", 0)
    backend.kv_append(T(vf), cache, "v", 0)
    out = torch.zeros((S, H, 128), device=dev)
    backend.attention(T(q), cache, out, pos, W)
    torch.cuda.synchronize()
    kk = cache.k[:rows].view(torch.int16).cpu().numpy().view(np.uint16)
    vv = cache.v[:rows].view(torch.int16).cpu().numpy().view(np.uint16)
    ref = oracle.attention(q, kk, vv, pos, W, fmt)
    assert rel_l2(out.cpu().numpy(), ref) < TOL
    assert backend.device_status() == 0


@pytest.mark.parametrize("H,KV,S,pos,W", [(32, 8, 1, 4000, 0), (16, 4, 3, 700, 0), (8, 2, 5, 1000, 300),
                                          (4, 4, 1, 129, 0), (16, 2, 1, 2049, 0), (12, 3, 2, 63, 17),
                                          (16, 8, 1, 1023, 0)])
def test_q8_cache_rows_past_the_context(backend, H, KV, S, pos, W):
    """Q8_0 caches (the engine's format) against runAttentionQ8 over GQA groups
    1-8, S > 1, windows and tile-edge lengths, with the rows past the context
    holding arbitrary int8 values and NaN scales: they must never reach the
    output."""
    rng = np.random.default_rng(7 * H + KV + S + pos + W)
    rows = pos + S
    q = rng.standard_normal((S, H, 128), dtype=np.float32)
    kf = rng.standard_normal((rows, KV, 128), dtype=np.float32)
    vf = rng.standard_normal((rows, KV, 128), dtype=np.float32)
    cache = KVCache.allocate(rows + 200, KV, 128, KV_Q8_0)
    cache.k.copy_(torch.from_numpy(rng.integers(-127, 128, cache.k.shape, dtype=np.int8)))
    cache.v.copy_(torch.from_numpy(rng.integers(-127, 128, cache.v.shape, dtype=np.int8)))
    cache.k_scale.fill_(float("nan"))
    cache.v_scale.fill_(float("nan"))
    backend.kv_append(T(kf), cache, "k", 0)
    backend.kv_append(T(vf), cache, "v", 0)
    out = torch.zeros((S, H, 128), device=dev)
    backend.attention(T(q), cache, out, pos, W)
    torch.cuda.synchronize()
    kq, vq = cache.k[:rows].cpu().numpy(), cache.v[:rows].cpu().numpy()
    ks, vs = cache.k_scale[:rows].cpu().numpy(), cache.v_scale[:rows].cpu().numpy()
    ref = oracle.attention(q, kq, vq, pos, W, KV_Q8_0, ks, vs)
    assert np.isfinite(out.cpu().numpy()).all()
    assert rel_l2(out.cpu().numpy(), ref) < TOL
    assert backend.device_status() == 0


def test_bounded_wait_reports_a_timeout(backend):
    """A device-side wait that nothing ends gives up after its time limit,
    records the timeout bit in the status word and returns: the host reads
    it, and the next call runs normally (no fault, no hang)."""
    assert backend.device_status() == 0
    backend.selftest_wait_timeout()
    assert backend.device_status() == 1  # HCU_DEVERR_TIMEOUT, cleared by the read
    assert backend.device_status() == 0
    rng = np.random.default_rng(3)
    q = rng.standard_normal((1, 4, 128), dtype=np.float32)
    k = rng.standard_normal((40, 2, 128), dtype=np.float32)
    v = rng.standard_normal((40, 2, 128), dtype=np.float32)
    cache = KVCache(KV_F32, T(k), T(v))
    out = torch.zeros((1, 4, 128), device=dev)
    backend.attention(T(q), cache, out, 39)
    torch.cuda.synchronize()
    assert rel_l2(out.cpu().numpy(), oracle.attention(q, k, v, 39)) < TOL
    assert backend.device_status() == 0


@pytest.mark.parametrize("name", ["attn_q8_decode", "attn_q8_segment", "attn_q8_swa", "attn_q8_dh256"])
def test_q8_wgsl_convention_via_dispatch(backend, request, name):
    """The dispatch seam in the WGSL ops' Q8_0 convention (scale array = amax,
    src/kernels.ts:1287-1335 and :1386-1411): kv_append_q8 writes exactly what
    the WGSL append writes (f32, round() ties-to-even), attention_q8 over that
    cache matches both the WGSL-semantics oracle and runAttentionQ8 on the
    same int8 values, and a cache the reference's WGSL append wrote (here its
    restatement, on the CPU) reads correctly."""
    backend.set_q8_convention(KV_Q8_0_WGSL)
    request.addfinalizer(lambda: backend.set_q8_convention(KV_Q8_0))
    d = g(name)
    S, H, KV, Dh, pos, W = (int(x) for x in d["meta"])
    rows = pos + S
    nb = Dh // 32
    kq_ref, vq_ref = np.zeros((rows, KV, Dh), np.int8), np.zeros((rows, KV, Dh), np.int8)
    ka_ref, va_ref = np.zeros((rows, KV, nb), np.float32), np.zeros((rows, KV, nb), np.float32)
    cache = KVCache.allocate(rows, KV, Dh, KV_Q8_0_WGSL)
    kf, vf = T(d["k"]), T(d["v"])
    for lo, hi in ((0, pos), (pos, rows)):
        if hi > lo:
            for src, q8, sc in ((kf, cache.k, cache.k_scale), (vf, cache.v, cache.v_scale)):
                backend.dispatch("kv_append_q8", [hi - lo, KV, Dh, lo], [src[lo:hi].contiguous(), q8, sc])
            oracle.append_kv_q8_wgsl(np.ascontiguousarray(d["k"][lo:hi]), kq_ref, ka_ref, lo)
            oracle.append_kv_q8_wgsl(np.ascontiguousarray(d["v"][lo:hi]), vq_ref, va_ref, lo)
    out = torch.zeros((S, H, Dh), device=dev)
    q = d["q"]
    backend.dispatch("attention_q8", [S, H, KV, Dh, pos, W, 0, 0],
                     [T(q), cache.k, cache.k_scale, cache.v, cache.v_scale, out])
    torch.cuda.synchronize()
    np.testing.assert_array_equal(cache.k.cpu().numpy(), kq_ref)
    np.testing.assert_array_equal(cache.k_scale.cpu().numpy(), ka_ref)
    np.testing.assert_array_equal(cache.v.cpu().numpy(), vq_ref)
    np.testing.assert_array_equal(cache.v_scale.cpu().numpy(), va_ref)
    ref_wgsl = oracle.attention_q8_wgsl(q, kq_ref, ka_ref, vq_ref, va_ref, pos, W)
    ref_js = oracle.attention(q, kq_ref, vq_ref, pos, W, KV_Q8_0, ka_ref / np.float32(127), va_ref / np.float32(127))
    got = out.cpu().numpy()
    assert rel_l2(got, ref_wgsl) < TOL
    assert rel_l2(got, ref_js) < TOL
    # a cache written by the reference's WGSL append, read through the seam
    oc = KVCache(KV_Q8_0_WGSL, T(kq_ref), T(vq_ref), T(ka_ref), T(va_ref))
    out2 = torch.zeros_like(out)
    backend.dispatch("attention_q8", [S, H, KV, Dh, pos, W, 0, 0], [T(q), oc.k, oc.k_scale, oc.v, oc.v_scale, out2])
    torch.cuda.synchronize()
    assert rel_l2(out2.cpu().numpy(), ref_wgsl) < TOL
    assert backend.device_status() == 0


def test_dirty_tickets_are_rearmed_by_a_status_clear(backend):
    """Split tickets left partly counted, as by a call whose bounded wait gave
    up, keep every split of a unit from merging (its output stays unwritten);
    hcu_device_status(clear) re-arms them and the next call matches the
    oracle."""
    rng = np.random.default_rng(41)
    pos, H, KV = 6000, 8, 2  # one sequence, 2 units of many splits
    q = rng.standard_normal((1, H, 128), dtype=np.float32)
    k = rng.standard_normal((pos + 1, KV, 128), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((pos + 1, KV, 128), dtype=np.float32).astype(np.float16)
    cache = KVCache(KV_F16, T(k.view(np.int16), torch.float16), T(v.view(np.int16), torch.float16))
    assert backend.device_status() == 0
    backend.selftest_dirty_tickets()
    out = torch.full((1, H, 128), float("nan"), device=dev)
    backend.attention(T(q), cache, out, pos)
    torch.cuda.synchronize()
    assert np.isnan(out.cpu().numpy()).all()  # no unit drew its last ticket
    assert backend.device_status(clear=True) == 0  # no timeout was recorded; the clear re-arms the tickets
    out.fill_(float("nan"))
    backend.attention(T(q), cache, out, pos)
    torch.cuda.synchronize()
    ref = oracle.attention(q, k.view(np.uint16), v.view(np.uint16), pos, 0, KV_F16)
    assert rel_l2(out.cpu().numpy(), ref) < TOL
    assert backend.device_status() == 0


@pytest.mark.parametrize("impl", ["tc", "cuda"])
@pytest.mark.parametrize("H,KV,S,pos,W,vscale", [(32, 8, 1, 4000, 0, 1.0), (16, 8, 1, 1023, 0, 1.0),
                                                 (8, 8, 1, 128, 0, 1.0), (16, 4, 3, 700, 0, 1.0),
                                                 (8, 2, 5, 1000, 300, 1.0), (4, 2, 8, 129, 0, 1.0),
                                                 (12, 3, 2, 63, 17, 1.0), (16, 8, 1, 6000, 0, 1e-5),
                                                 (16, 8, 1, 3000, 0, 3e4), (8, 4, 2, 255, 1, 1.0)])
def test_q8_tensor_core_and_cuda_core_paths(backend, request, impl, H, KV, S, pos, W, vscale):
    """Q8_0 caches on the int8 tensor-core kernel (default for GQA groups up to
    4 with Dh 128) and on the CUDA-core kernel, against runAttentionQ8: groups
    1-4, S > 1, windows (1 included), tile-edge and multi-split contexts, and
    rows whose magnitudes (hence block scales) vary by 10^3 within a tile, for
    V values of scale 1e-5 to 3e4."""
    backend.set_option("attn_cuda_cores", int(impl == "cuda"))
    request.addfinalizer(lambda: backend.set_option("attn_cuda_cores", 0))
    rng = np.random.default_rng(H * 7 + KV + S + pos + W)
    rows = pos + S
    q = rng.standard_normal((S, H, 128), dtype=np.float32)
    mag = np.exp(rng.uniform(-3.5, 3.5, (rows, KV, 4))).astype(np.float32).repeat(32, axis=2)
    kf = rng.standard_normal((rows, KV, 128), dtype=np.float32) * mag
    vf = (rng.standard_normal((rows, KV, 128), dtype=np.float32) * mag[:, ::-1] * np.float32(vscale)).astype(np.float32)
    cache = KVCache.allocate(rows, KV, 128, KV_Q8_0)
    backend.kv_append(T(kf), cache, "k", 0)
    backend.kv_append(T(np.ascontiguousarray(vf)), cache, "v", 0)
    out = torch.full((S, H, 128), float("nan"), device=dev)
    backend.attention(T(q), cache, out, pos, W)
    torch.cuda.synchronize()
    kq, vq = cache.k.cpu().numpy(), cache.v.cpu().numpy()
    ks, vs = cache.k_scale.cpu().numpy(), cache.v_scale.cpu().numpy()
    ref = oracle.attention(q, kq, vq, pos, W, KV_Q8_0, ks, vs)
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    assert rel_l2(got, ref) < TOL
    assert backend.device_status() == 0


@pytest.mark.parametrize("impl", ["tc", "cuda"])
def test_q8_batched_ragged_sequences(backend, request, impl):
    """cfg2's layout on a Q8_0 cache: a packed batch of ragged sequences with
    per-sequence positions and row offsets, H = 32, KV = 8."""
    backend.set_option("attn_cuda_cores", int(impl == "cuda"))
    request.addfinalizer(lambda: backend.set_option("attn_cuda_cores", 0))
    rng = np.random.default_rng(77)
    lens = np.array([1, 127, 128, 129, 700, 4096, 8045, 2049])
    off = np.concatenate([[0], np.cumsum(lens)[:-1]])
    B, H, KV = len(lens), 32, 8
    kf = rng.standard_normal((lens.sum(), KV, 128), dtype=np.float32)
    vf = rng.standard_normal((lens.sum(), KV, 128), dtype=np.float32)
    cache = KVCache.allocate(int(lens.sum()), KV, 128, KV_Q8_0)
    backend.kv_append(T(kf), cache, "k", 0)
    backend.kv_append(T(vf), cache, "v", 0)
    q = rng.standard_normal((B, 1, H, 128), dtype=np.float32)
    out = torch.full((B, 1, H, 128), float("nan"), device=dev)
    backend.attention(T(q), cache, out, T((lens - 1).astype(np.int32)), 0, kv_row_offset=T(off.astype(np.int64)),
                      max_context=int(lens.max()))
    torch.cuda.synchronize()
    ref = oracle.attention_batch(q, cache.k.cpu().numpy(), cache.v.cpu().numpy(), lens - 1, off, 0, KV_Q8_0,
                                 cache.k_scale.cpu().numpy(), cache.v_scale.cpu().numpy())
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    assert rel_l2(got, ref) < TOL
    assert backend.device_status() == 0


@pytest.mark.parametrize("fmt,H,KV,lens,W,cuda_cores", [
    (KV_F32, 8, 2, [1, 50, 300, 1000], 0, 0),   # 16 splits of 64 keys; units with 1, 1, 5 and 16 splits
    (KV_F32, 16, 8, [1000, 640], 300, 0),       # a window: 5 splits per unit
    (KV_Q8_0, 32, 4, [900, 1024], 0, 0),        # GQA group 8 on Q8_0: the CUDA-core kernel, 4 splits of 256 keys
    (KV_F16, 16, 8, [1024], 0, 1),              # f16 forced onto the CUDA-core kernel: 8 splits of 128 keys
])
def test_cluster_merge_of_small_launches(backend, request, fmt, H, KV, lens, W, cuda_cores):
    """Small CUDA-core launches (a few sequences, at most 16 key splits per
    unit) merge their splits inside thread-block clusters through distributed
    shared memory; units whose sequence needs fewer splits than the cluster
    holds leave empty partials in the other CTAs."""
    backend.set_option("attn_cuda_cores", cuda_cores)
    request.addfinalizer(lambda: backend.set_option("attn_cuda_cores", 0))
    rng = np.random.default_rng(sum(lens) + H + KV + W)
    lens = np.array(lens)
    off = np.concatenate([[0], np.cumsum(lens)[:-1]])
    B = len(lens)
    kf = rng.standard_normal((lens.sum(), KV, 128), dtype=np.float32)
    vf = rng.standard_normal((lens.sum(), KV, 128), dtype=np.float32)
    q = rng.standard_normal((B, 1, H, 128), dtype=np.float32)
    if fmt == KV_Q8_0:
        cache = KVCache.allocate(int(lens.sum()), KV, 128, KV_Q8_0)
        backend.kv_append(T(kf), cache, "k", 0)
        backend.kv_append(T(vf), cache, "v", 0)
        kref, vref = cache.k.cpu().numpy(), cache.v.cpu().numpy()
        scales = (cache.k_scale.cpu().numpy(), cache.v_scale.cpu().numpy())
    elif fmt == KV_F16:
        kh, vh = kf.astype(np.float16), vf.astype(np.float16)
        cache = KVCache(KV_F16, T(kh.view(np.int16), torch.float16), T(vh.view(np.int16), torch.float16))
        kref, vref, scales = kh.view(np.uint16), vh.view(np.uint16), ()
    else:
        cache = KVCache(KV_F32, T(kf), T(vf))
        kref, vref, scales = kf, vf, ()
    out = torch.full((B, 1, H, 128), float("nan"), device=dev)
    backend.attention(T(q), cache, out, T((lens - 1).astype(np.int32)), W, kv_row_offset=T(off.astype(np.int64)),
                      max_context=int(lens.max()))
    torch.cuda.synchronize()
    ref = oracle.attention_batch(q, kref, vref, lens - 1, off, W, fmt, *scales)
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    assert rel_l2(got, ref) < TOL
    assert backend.device_status() == 0

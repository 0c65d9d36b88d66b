"""GPU parity of the tcgen05 sliding-window prefill against the oracle.

The oracle is runAttentionQ8's loop (src/wasm-backend.ts:826-895) with a bf16
cache, S = T queries at posBase 0 and the window rule of attention_q8
(src/kernels.ts:1373-1377).  Tolerance (bf16 tensor-core path): relative L2
<= 1e-2 and max-abs <= 2e-2."""
import numpy as np
import pytest
import torch

import oracle
from hachiue_b200 import HachiueError, workloads
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu
REL, ABS = 1e-2, 2e-2
dev = "cuda"


def bf16_dev(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(dev).view(torch.bfloat16)


def check_slice(out, qb, kb, vb, b, qs, qe, W):
    """Oracle on queries [qs, qe) of sequence b, all heads."""
    q = workloads.bf16_bits_to_f32(qb[b, qs:qe])
    ref = oracle.attention(np.ascontiguousarray(q), np.ascontiguousarray(kb[b]), np.ascontiguousarray(vb[b]), qs, W,
                           oracle.KV_BF16)
    got = out[b, qs:qe]
    assert rel_l2(got, ref) < REL, (b, qs, qe, rel_l2(got, ref))
    assert np.abs(got - ref).max() < ABS


def rand_bf16(rng, shape):
    x = torch.from_numpy(rng.standard_normal(shape, dtype=np.float32)).to(torch.bfloat16)
    return x.view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("B,T,H,KV,W", [(1, 128, 2, 1, 0), (2, 300, 4, 2, 64), (1, 515, 6, 3, 0), (1, 384, 2, 2, 1),
                                        (2, 700, 8, 2, 1024), (1, 1000, 4, 1, 200), (3, 257, 2, 1, 129)])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_small_shapes(backend, B, T, H, KV, W, out_dtype):
    rng = np.random.default_rng(B * 7 + T + H + W)
    qb, kb, vb = rand_bf16(rng, (B, T, H, 128)), rand_bf16(rng, (B, T, KV, 128)), rand_bf16(rng, (B, T, KV, 128))
    out = torch.full((B, T, H, 128), float("nan"), device=dev, dtype=out_dtype)
    backend.swa_prefill(bf16_dev(qb), bf16_dev(kb), bf16_dev(vb), out, W)
    torch.cuda.synchronize()
    o = out.float().cpu().numpy()
    assert np.isfinite(o).all()
    for b in range(B):
        check_slice(o, qb, kb, vb, b, 0, T, W)
    assert backend.device_status() == 0


@pytest.mark.parametrize("ctas", [1, 3])
@pytest.mark.parametrize("B,T,H,KV,W", [(2, 700, 8, 2, 1024), (1, 515, 6, 3, 0), (3, 257, 2, 1, 129)])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_persistent_item_chains(backend, request, ctas, B, T, H, KV, W, out_dtype):
    """The kernel is persistent (one CTA per SM walks a list of work items);
    capping the grid at 1 or 3 CTAs makes every CTA run a long chain of
    items with different key ranges and head groups, and odd rounds of the
    snake order, on shapes the oracle checks whole.  Each item's output is
    written while the next item runs (bf16 through the staging buffer)."""
    backend.set_option("swa_ctas", ctas)
    request.addfinalizer(lambda: backend.set_option("swa_ctas", 0))
    rng = np.random.default_rng(B * 11 + T + H + W + ctas)
    qb, kb, vb = rand_bf16(rng, (B, T, H, 128)), rand_bf16(rng, (B, T, KV, 128)), rand_bf16(rng, (B, T, KV, 128))
    out = torch.full((B, T, H, 128), float("nan"), device=dev, dtype=out_dtype)
    backend.swa_prefill(bf16_dev(qb), bf16_dev(kb), bf16_dev(vb), out, W)
    torch.cuda.synchronize()
    o = out.float().cpu().numpy()
    assert np.isfinite(o).all()
    for b in range(B):
        check_slice(o, qb, kb, vb, b, 0, T, W)
    assert backend.device_status() == 0


@pytest.fixture(scope="module")
def cfg3():
    return workloads.swa_cfg3()


def test_cfg3_plamo3_swa_prefill(backend, cfg3):
    """Full config 3 (8 x 4096, 16 / 4 heads, W = 1024); the oracle checks the
    first window, the window edge, the middle and the end of two sequences."""
    w = cfg3
    q, k, v = bf16_dev(w["q"]), bf16_dev(w["k"]), bf16_dev(w["v"])
    out = torch.empty((8, 4096, 16, 128), device=dev, dtype=torch.bfloat16)
    backend.swa_prefill(q, k, v, out, w["window"])
    torch.cuda.synchronize()
    o = out.float().cpu().numpy()
    assert np.isfinite(o).all()
    for b in (0, 7):
        for qs, qe in ((0, 130), (1000, 1100), (2047, 2177), (3990, 4096)):
            check_slice(o, w["q"], w["k"], w["v"], b, qs, qe, w["window"])
    # a second call gives bit-identical results
    out2 = torch.empty_like(out)
    backend.swa_prefill(q, k, v, out2, w["window"])
    assert torch.equal(out, out2)


def test_cfg3_whole_output_against_f32_reference(backend, cfg3):
    """Every output of config 3 (8 sequences x 4096 queries x 16 heads)
    against softmax(Q K^T / sqrt(128)) V in f32 on the GPU with the window
    band of attention_q8 (src/kernels.ts:1373-1377): keys max(0, i - 1023) .. i.
    The oracle-checked slices above pin this closed form's semantics; this
    covers the rest of the output."""
    w = cfg3
    q, k, v = bf16_dev(w["q"]), bf16_dev(w["k"]), bf16_dev(w["v"])
    out = torch.empty((8, 4096, 16, 128), device=dev, dtype=torch.bfloat16)
    backend.swa_prefill(q, k, v, out, w["window"])
    torch.cuda.synchronize()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        T, W = 4096, w["window"]
        i = torch.arange(T, device=dev)
        band = (i[None, :] <= i[:, None]) & (i[None, :] > i[:, None] - W)  # [query, key]
        err2 = ref2 = 0.0
        worst = 0.0
        for b in range(8):
            for g in range(4):  # KV head g serves query heads 4g .. 4g + 3
                qh = q[b, :, 4 * g:4 * g + 4].float().permute(1, 0, 2)  # [4, T, 128]
                kh, vh = k[b, :, g].float(), v[b, :, g].float()
                s = torch.matmul(qh, kh.t()) / np.sqrt(128.0)
                s = s.masked_fill(~band, float("-inf"))
                ref = torch.matmul(torch.softmax(s, dim=-1), vh)  # [4, T, 128]
                got = out[b, :, 4 * g:4 * g + 4].float().permute(1, 0, 2)
                d = got - ref
                err2 += float((d.double() ** 2).sum())
                ref2 += float((ref.double() ** 2).sum())
                worst = max(worst, float(d.abs().max()))
                assert float(d.norm() / ref.norm()) < REL, (b, g)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    assert (err2 / ref2) ** 0.5 < REL
    assert worst < ABS


def test_rejects_bad_arguments(backend):
    q = torch.zeros((1, 128, 2, 64), device=dev, dtype=torch.bfloat16)
    with pytest.raises(HachiueError, match="D=64"):
        backend.swa_prefill(q, q[:, :, :1].contiguous(), q[:, :, :1].contiguous(), torch.zeros_like(q))
    with pytest.raises(HachiueError, match="bf16"):
        backend.swa_prefill(q.float(), q, q, q)

"""The precision split of the f16 / bf16 tcgen05 decode kernel
(attention_decode_tc.cu), restated in numpy and checked against the oracle's
runAttentionQ8 loop over the same cache (src/wasm-backend.ts:826-895).  CPU
only.

The tensor cores take 16-bit operands only, so the f32 query row and the f32
probabilities are sent as sums of 16-bit terms in the same type as the cache:
f16 as hi + lo of x * 2^8, bf16 as hi + mid + lo.  Each term meets the cache
in its own MMA column group and the f32 accumulators add them, which keeps the
result at f32 accuracy; a single 16-bit term would not.
"""
import numpy as np
import pytest

import oracle

LOG2E = 1.4426950408889634


def bf16(x):
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).astype(np.float64)


def f16(x):
    return np.asarray(x, dtype=np.float64).astype(np.float16).astype(np.float64)


def terms(x, kind, n):
    """x as n 16-bit terms of type kind (the scaled f16 split uses x * 2^8)."""
    rnd = f16 if kind == "f16" else bf16
    scale = 256.0 if kind == "f16" else 1.0
    r, out = np.asarray(x, np.float64) * scale, []
    for _ in range(n):
        t = rnd(r)
        out.append(t)
        r = r - t
    return out, scale


def tc_decode(q, k, v, kind, n):
    """One query row q [Dh] over the 16-bit cache values k, v [T, Dh]."""
    qt, qs = terms(q.astype(np.float32), kind, n)
    s = sum(k @ t for t in qt) / qs  # f32 accumulation of exact products (f64 here)
    s = s / np.sqrt(q.shape[0]) * LOG2E
    p = np.exp2(s - s.max()).astype(np.float32)
    pt, ps = terms(p, kind, n)
    return sum(v.T @ t for t in pt) / ps / p.astype(np.float64).sum()


@pytest.mark.parametrize("kind,fmt,n,T", [("f16", oracle.KV_F16, 2, 300), ("f16", oracle.KV_F16, 2, 2048),
                                          ("bf16", oracle.KV_BF16, 3, 300), ("bf16", oracle.KV_BF16, 3, 2048)])
def test_split_terms_keep_f32_accuracy(kind, fmt, n, T):
    rng = np.random.default_rng(T + n)
    Dh = 128
    q = rng.standard_normal((1, 1, Dh), dtype=np.float32)
    kf, vf = (rng.standard_normal((T, 1, Dh), dtype=np.float32) for _ in range(2))
    if kind == "f16":
        kb, vb = kf.astype(np.float16), vf.astype(np.float16)
        kv_oracle, kvals, vvals = (kb.view(np.uint16), vb.view(np.uint16)), kb[:, 0].astype(np.float64), \
            vb[:, 0].astype(np.float64)
    else:
        kvals, vvals = bf16(kf[:, 0]), bf16(vf[:, 0])
        bits = lambda x: np.ascontiguousarray((bf16(x).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16))  # noqa: E731
        kv_oracle = (bits(kf), bits(vf))
    ref = oracle.attention(q, kv_oracle[0], kv_oracle[1], T - 1, 0, fmt)[0, 0]
    rel = lambda a, b: np.linalg.norm(a - b) / np.linalg.norm(b)  # noqa: E731
    assert rel(tc_decode(q[0, 0], kvals, vvals, kind, n), ref) < 1e-5
    # one 16-bit term only: visibly worse, which is why the kernel splits
    assert rel(tc_decode(q[0, 0], kvals, vvals, kind, 1), ref) > 1e-4

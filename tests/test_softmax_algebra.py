"""The two softmax schemes of the attention kernels, restated in float64 numpy
and checked against the oracle's runAttentionQ8 (src/wasm-backend.ts:826-895).
CPU only.

* Split-K decode (attention_decode*.cu): each split of a sequence's keys leaves
  a partial (acc = sum_j 2^(s_j - m) v_j, m = its max in the log2 domain, l =
  sum_j 2^(s_j - m)); the merge rescales every partial to the largest m.  Empty
  splits (no keys) leave m = -inf and add nothing.
* Tiled prefill (swa_prefill.cu): one query row walks 128-key tiles with a
  running max; O and l are rescaled only when a tile's max exceeds the running
  max by more than 8 (log2 units), so P = 2^(s - m) stays below 2^8 and the
  final O / l cancels the stale max.
"""
import numpy as np
import pytest

import oracle

LOG2E = 1.4426950408889634


def scores_log2(q, k, scale):
    return (k @ q) * scale * LOG2E


def split_k(q, k, v, scale, splits):
    s = scores_log2(q, k, scale)
    parts = []
    for idx in np.array_split(np.arange(len(s)), splits):
        if len(idx) == 0:
            parts.append((np.zeros(v.shape[1]), -np.inf, 0.0))
            continue
        m = s[idx].max()
        p = np.exp2(s[idx] - m)
        parts.append((p @ v[idx], m, p.sum()))
    M = max(m for _, m, _ in parts)
    acc = sum(a * np.exp2(m - M) for a, m, _ in parts if np.isfinite(m))
    den = sum(l * np.exp2(m - M) for _, m, l in parts if np.isfinite(m))
    return acc / den


def tiled_lazy(q, k, v, scale, tile=128, slack=8.0):
    s = scores_log2(q, k, scale)
    m, l, o = -np.inf, 0.0, np.zeros(v.shape[1])
    rescales = 0
    for t0 in range(0, len(s), tile):
        st = s[t0:t0 + tile]
        mt = st.max()
        if mt > m + slack:
            if np.isfinite(m):
                o *= np.exp2(m - mt)
                l *= np.exp2(m - mt)
                rescales += 1
            m = mt
        p = np.exp2(st - m)
        assert p.max() <= 2.0 ** slack
        o += p @ v[t0:t0 + tile]
        l += p.sum()
    return o / l, rescales


@pytest.mark.parametrize("ctx,splits,shift", [(1, 1, 0.0), (300, 4, 0.0), (1000, 16, 0.0), (5, 16, 0.0),
                                              (2048, 7, 30.0)])
def test_split_k_merge_is_exact_softmax(ctx, splits, shift):
    """More splits than keys (empty splits) and scores far from zero included."""
    rng = np.random.default_rng(ctx + splits)
    Dh, H = 128, 1
    q = rng.standard_normal((1, H, Dh), dtype=np.float32)
    k = rng.standard_normal((ctx, 1, Dh), dtype=np.float32) + np.float32(shift / np.sqrt(Dh))
    v = rng.standard_normal((ctx, 1, Dh), dtype=np.float32)
    ref = oracle.attention(q, k, v, ctx - 1)[0, 0]
    got = split_k(q[0, 0].astype(np.float64), k[:, 0].astype(np.float64), v[:, 0].astype(np.float64),
                  1 / np.sqrt(Dh), splits)
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-5


@pytest.mark.parametrize("ctx,growth", [(128, 0.0), (700, 0.0), (1000, 0.05), (513, 0.5)])
def test_lazy_rescale_is_exact_softmax(ctx, growth):
    """Scores that climb along the keys force rescales; the result is still the
    softmax the oracle computes."""
    rng = np.random.default_rng(ctx)
    Dh = 128
    q = rng.standard_normal((1, 1, Dh), dtype=np.float32)
    ramp = (growth * np.arange(ctx, dtype=np.float32))[:, None, None] * q / np.linalg.norm(q)
    k = (rng.standard_normal((ctx, 1, Dh), dtype=np.float32) + ramp).astype(np.float32)
    v = rng.standard_normal((ctx, 1, Dh), dtype=np.float32)
    ref = oracle.attention(q, k, v, ctx - 1)[0, 0]
    got, rescales = tiled_lazy(q[0, 0].astype(np.float64), k[:, 0].astype(np.float64), v[:, 0].astype(np.float64),
                               1 / np.sqrt(Dh))
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-5
    if growth >= 0.5:
        assert rescales > 0

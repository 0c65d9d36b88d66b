"""The digit scheme of the Q8_0 tcgen05 decode kernel (attention_decode_q8tc.cu),
restated in numpy and checked against the oracle's runAttentionQ8
(src/wasm-backend.ts:826-895) on the engine's own cache.  CPU only.

Scores: q is scaled by 2^20 / max|q|, rounded to an integer of 21 bits, and
split into three balanced base-128 digits in [-64, 64]; each digit row times
the int8 key block is an exact integer dot product (what kind::i8 MMAs
produce), recombined and scaled by the key block's f32 scale.
Output: per 128-key tile and 32-element block, y = p * vs / max(vs) lies in
[0, 1]; it is rounded to 22 bits and split into three unsigned base-256 digits,
each times the int8 value column an exact integer sum, recombined and scaled
back by max(vs) / 2^22.
"""
import numpy as np
import pytest

import oracle

LOG2E = 1.4426950408889634


def balanced_digits(x):
    """Integers |x| <= 2^20 as three base-128 digits, each in [-64, 64]: the
    two low digits balanced in [-64, 63], the top one the remainder."""
    d = []
    for _ in range(2):
        r = ((x + 64) % 128) - 64
        d.append(r)
        x = (x - r) // 128
    d.append(x)
    return d


def q8_decode(q, kq, ks, vq, vs, tile=128):
    """One query row q [Dh] over an int8 cache kq, vq [T, Dh] with f32 block
    scales ks, vs [T, Dh / 32] (the JS convention: value = int8 * scale)."""
    T, Dh = kq.shape
    nb = Dh // 32
    qs = 2.0 ** 20 / np.abs(q).max()
    qi = np.rint(q * qs).astype(np.int64)
    digits = balanced_digits(qi)
    assert all(np.abs(d).max() <= 64 for d in digits)
    s = np.zeros(T)
    for b in range(nb):
        blk = slice(32 * b, 32 * b + 32)
        kb = kq[:, blk].astype(np.int64)
        dots = sum((kb @ d[blk]) * 128 ** i for i, d in enumerate(digits))  # exact integer dot products
        s += ks[:, b] * dots / qs
    s = s / np.sqrt(Dh) * LOG2E
    m = s.max()
    p = np.exp2(s - m)
    out = np.zeros(Dh)
    for t0 in range(0, T, tile):
        tt = slice(t0, min(t0 + tile, T))
        for b in range(nb):
            blk = slice(32 * b, 32 * b + 32)
            vmax = vs[tt, b].max()
            if vmax == 0:
                continue
            y = np.rint(p[tt] * vs[tt, b] / vmax * 2.0 ** 22).astype(np.int64)  # 22 bits, y <= 2^22
            yd = [(y >> (8 * i)) & 255 for i in range(3)]
            vb = vq[tt, blk].astype(np.int64)
            sums = sum((yd[i] @ vb) * 256 ** i for i in range(3))  # exact integer sums
            out[blk] += sums * vmax / 2.0 ** 22
    return out / p.sum()


@pytest.mark.parametrize("T,seed", [(1, 0), (100, 1), (1024, 2), (3000, 3)])
def test_digit_scheme_matches_run_attention_q8(T, seed):
    rng = np.random.default_rng(seed)
    Dh = 128
    kf = rng.standard_normal((T, 1, Dh), dtype=np.float32)
    vf = rng.standard_normal((T, 1, Dh), dtype=np.float32)
    kq, vq = np.zeros((T, 1, Dh), np.int8), np.zeros((T, 1, Dh), np.int8)
    ks, vs = np.zeros((T, 1, Dh // 32), np.float32), np.zeros((T, 1, Dh // 32), np.float32)
    oracle.append_kv_q8(kf, kq, ks, 0)
    oracle.append_kv_q8(vf, vq, vs, 0)
    q = rng.standard_normal((1, 1, Dh), dtype=np.float32)
    ref = oracle.attention(q, kq, vq, T - 1, 0, oracle.KV_Q8_0, ks, vs)[0, 0]
    got = q8_decode(q[0, 0].astype(np.float64), kq[:, 0], ks[:, 0].astype(np.float64), vq[:, 0],
                    vs[:, 0].astype(np.float64))
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-5


def test_balanced_digits_cover_21_bits():
    x = np.array([-(2 ** 20), -(2 ** 20) + 1, -64, -65, 0, 63, 64, 65, 2 ** 20 - 1, 2 ** 20], dtype=np.int64)
    d = balanced_digits(x.copy())
    assert np.array_equal(d[0] + 128 * d[1] + 16384 * d[2], x)
    assert all(np.abs(di).max() <= 64 for di in d)

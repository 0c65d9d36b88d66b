"""The chunked (WY) form of the gated delta rule that the prefill kernels
compute, restated in float64 numpy in the order the kernels use it, against
the oracle's token-serial recurrence (src/wasm-backend.ts:1047-1102).  CPU only.

Per V head and 64-token chunk, with S0 the entering state ([dk][dv]), gamma
the in-chunk cumulative sum of g, ik / iq the key / query norm factors and
K, Q, V the raw chunk rows:

  prep (gdn_prep_kernel):
    A_ij   = beta_i ik_i ik_j exp(gamma_i - gamma_j) k_i.k_j   (j < i)
    T      = (I + A)^-1,  Tb = T diag(beta)
    QKm_ij = iq_i ik_j exp(gamma_i - gamma_j) q_i.k_j          (j <= i)
    W      = [Tb; QKm Tb],  c2 = exp(gamma) ik,  c3 = exp(gamma) iq,
    c4     = ik exp(gamma_last - gamma),  e = exp(gamma_last)
  recurrence (gdn_chain_kernel, state in TMEM):
    [X; QS]     = [K; Q] S0
    R'          = V - diag(c2) X
    [Tb R'; O]  = [0; diag(c3) QS] + W R'     (X zeroed, QS scaled in place)
    S1          = e S0 + K^T diag(c4) (Tb R')   (accumulated onto e S0)

The second test rounds to bf16 where the kernels hold MMA operands (the state
copy, R', W, Dsb) and checks that the result stays inside the GPU tests'
bound; it lands at 1.5e-3 to 3e-3, the error the kernels show on the GPU.
"""
import numpy as np
import pytest

import oracle

C = 64


def bf16(x):
    """Round to bf16 (nearest even), as the kernels store an MMA operand."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).astype(np.float64)


def tf32(x):
    """Round f32 to tf32 as the prep does: add half an ulp of the 10-bit mantissa, truncate."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32)
    return ((u.astype(np.uint64) + 0x1000) & 0xFFFFE000).astype(np.uint32).view(np.float32)


def blocked_inverse(A):
    """(I + A)^-1 of a strictly lower-triangular 64 x 64 f32 A (tf32 values) the
    way gdn_prep_kernel builds it: 16 x 16 diagonal blocks by forward
    substitution in f32 (every element rounded to tf32), the 32 x 32 blocks
    T[2p+1][2p] = -T[2p+1][2p+1] A[2p+1][2p] T[2p][2p] in f32, and the 64 x 64
    block T[1][0] = -T22 (A21 T11) on the tf32 tensor cores (A21 T11 rounded to
    tf32 in between)."""
    f32 = np.float32
    T = np.zeros((64, 64), f32)
    for base in range(0, 64, 16):
        Ab = A[base:base + 16, base:base + 16]
        blk = np.zeros((16, 16), f32)
        for r in range(16):
            acc = np.zeros(16, f32)
            for j in range(r):
                acc = (Ab[r, j].astype(np.float64) * blk[j] + acc).astype(f32)  # fmaf
            blk[r] = tf32(np.where(np.arange(16) == r, f32(1), -acc))
        T[base:base + 16, base:base + 16] = blk
    for p in (0, 1):
        rb, cb = 16 * (2 * p + 1), 32 * p
        X1 = (A[rb:rb + 16, cb:cb + 16].astype(np.float64) @ T[cb:cb + 16, cb:cb + 16]).astype(f32)
        T[rb:rb + 16, cb:cb + 16] = tf32(-(T[rb:rb + 16, rb:rb + 16].astype(np.float64) @ X1).astype(f32))
    X2 = tf32((A[32:64, 0:32].astype(np.float64) @ T[0:32, 0:32]).astype(f32))
    T[32:64, 0:32] = (-(T[32:64, 32:64].astype(np.float64) @ X2)).astype(f32)
    return T.astype(np.float64)


def exact_inverse(A):
    return np.linalg.inv(np.eye(A.shape[0]) + A)


def kernel_inverse(A):
    """The prep's T for a chunk of n <= 64 tokens: A rounded to tf32, padded."""
    n = A.shape[0]
    Ap = np.zeros((64, 64), np.float32)
    Ap[:n, :n] = tf32(A.astype(np.float32))
    return blocked_inverse(Ap)[:n, :n]


def chunked(q, k, v, g, beta, S0, operand=lambda x: x, inverse=exact_inverse):
    """q, k, v [T, D]; g, beta [T]; S0 [D, D].  Returns (out [T, D], S_T).
    ``operand`` rounds what the kernels hold as bf16 MMA operands: the state
    copy, R', W and Dsb (identity: the exact chunked form)."""
    T, D = q.shape
    ik = 1 / np.sqrt((k * k).sum(1) + 1e-6)
    iq = 1 / np.sqrt((q * q).sum(1) + 1e-6) / np.sqrt(D)
    S = S0.copy()
    out = np.zeros((T, D))
    for c0 in range(0, T, C):
        sl = slice(c0, min(c0 + C, T))
        n = sl.stop - sl.start
        K, Q, V, b, ikc, iqc = k[sl], q[sl], v[sl], beta[sl], ik[sl], iq[sl]
        gam = np.cumsum(g[sl])
        i, j = np.indices((n, n))
        dec = np.where(j <= i, np.exp(np.where(j <= i, gam[:, None] - gam[None, :], 0.0)), 0.0)
        A = np.where(j < i, b[:, None] * ikc[:, None] * ikc[None, :] * dec * (K @ K.T), 0.0)
        Tb = inverse(A) * b[None, :]
        QKm = iqc[:, None] * ikc[None, :] * dec * (Q @ K.T)
        W = operand(np.vstack([Tb, QKm @ Tb]))
        c2, c3 = np.exp(gam) * ikc, np.exp(gam) * iqc
        c4, e = ikc * np.exp(gam[-1] - gam), np.exp(gam[-1])
        Sb = operand(S)
        P = np.vstack([K @ Sb, Q @ Sb])
        Rp = operand(V - c2[:, None] * P[:n])
        P = np.vstack([np.zeros((n, D)), c3[:, None] * P[n:]]) + W @ Rp
        out[sl] = P[n:]
        S = e * S + K.T @ operand(c4[:, None] * P[:n])
    return out, S


@pytest.mark.parametrize("T,decay,load", [(64, 1.0, False), (150, 1.0, True), (256, 0.05, True), (200, 4.0, False),
                                          (129, 0.0, True)])
def test_chunked_form_matches_token_serial_oracle(T, decay, load):
    rng = np.random.default_rng(T + int(10 * decay))
    D = 128
    q, k, v = (rng.standard_normal((T, D)) for _ in range(3))
    a = rng.standard_normal(T)
    g = -decay * (np.maximum(a, 0) + np.log1p(np.exp(-np.abs(a))))
    beta = 1 / (1 + np.exp(-rng.standard_normal(T)))
    S0 = 0.05 * rng.standard_normal((D, D)) if load else np.zeros((D, D))
    f32 = lambda x: np.ascontiguousarray(x, dtype=np.float32)  # noqa: E731
    qkv = f32(np.concatenate([q, k, v], 1))
    gb = f32(np.stack([g, beta])[:, :, None])
    ref_out, ref_S = oracle.deltanet_recur(qkv, gb, f32(S0)[None], 1, 1, load)
    # the same f32 inputs in float64
    q, k, v = (qkv[:, i * D:(i + 1) * D].astype(np.float64) for i in range(3))
    out, S = chunked(q, k, v, gb[0, :, 0].astype(np.float64), gb[1, :, 0].astype(np.float64),
                     f32(S0).astype(np.float64))
    rel = lambda a, b: np.linalg.norm(a - b) / np.linalg.norm(b)  # noqa: E731
    assert rel(out, ref_out[:, 0]) < 1e-4
    assert rel(S, ref_S[0]) < 1e-4


@pytest.mark.parametrize("T,decay,load", [(256, 1.0, True), (640, 0.02, True), (200, 4.0, False)])
def test_bf16_operands_stay_inside_the_gpu_tolerance(T, decay, load):
    """With bf16 q / k / v and the kernels' bf16 MMA operands (state copy, R',
    W, Dsb; f32 accumulation and state), the chunked form stays within the
    GPU parity bound (relative L2 1e-2) of the token-serial oracle on the same
    bf16 inputs."""
    rng = np.random.default_rng(3 * T)
    D = 128
    q, k, v = (bf16(rng.standard_normal((T, D))) for _ in range(3))
    a = rng.standard_normal(T)
    g = (-decay * (np.maximum(a, 0) + np.log1p(np.exp(-np.abs(a))))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal(T)))).astype(np.float32)
    S0 = (0.02 * rng.standard_normal((D, D))).astype(np.float32) if load else np.zeros((D, D), np.float32)
    f32 = lambda x: np.ascontiguousarray(x, dtype=np.float32)  # noqa: E731
    ref_out, ref_S = oracle.deltanet_recur(f32(np.concatenate([q, k, v], 1)), f32(np.stack([g, beta])[:, :, None]),
                                           f32(S0)[None], 1, 1, load)
    out, S = chunked(q, k, v, g.astype(np.float64), beta.astype(np.float64), S0.astype(np.float64), operand=bf16)
    rel = lambda a, b: np.linalg.norm(a - b) / np.linalg.norm(b)  # noqa: E731
    assert rel(out, ref_out[:, 0]) < 1e-2
    assert rel(S, ref_S[0]) < 1e-2


def test_blocked_tf32_inverse():
    """The prep's blocked tf32 inverse against the exact one, alone and inside
    the chunked form with bf16 operands (still inside the GPU bound)."""
    rng = np.random.default_rng(11)
    D, T = 128, 256
    k = rng.standard_normal((64, D))
    ik = 1 / np.sqrt((k * k).sum(1) + 1e-6)
    b = 1 / (1 + np.exp(-rng.standard_normal(64)))
    gam = np.cumsum(-np.log1p(np.exp(rng.standard_normal(64))))
    i, j = np.indices((64, 64))
    A = np.where(j < i, b[:, None] * ik[:, None] * ik[None, :] * np.exp(np.where(j < i, gam[:, None] - gam[None, :], 0))
                 * (k @ k.T), 0.0)
    Te, Tk = exact_inverse(A), kernel_inverse(A)
    assert np.linalg.norm(Tk - Te) / np.linalg.norm(Te) < 1e-4  # measured 7.5e-6
    q, kk, v = (bf16(rng.standard_normal((T, D))) for _ in range(3))
    a = rng.standard_normal(T)
    g = (-(np.maximum(a, 0) + np.log1p(np.exp(-np.abs(a))))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal(T)))).astype(np.float32)
    S0 = (0.02 * rng.standard_normal((D, D))).astype(np.float32)
    f32 = lambda x: np.ascontiguousarray(x, dtype=np.float32)  # noqa: E731
    ref_out, ref_S = oracle.deltanet_recur(f32(np.concatenate([q, kk, v], 1)), f32(np.stack([g, beta])[:, :, None]),
                                           f32(S0)[None], 1, 1, True)
    out, S = chunked(q, kk, v, g.astype(np.float64), beta.astype(np.float64), S0.astype(np.float64), operand=bf16,
                     inverse=kernel_inverse)
    rel = lambda a, b: np.linalg.norm(a - b) / np.linalg.norm(b)  # noqa: E731
    assert rel(out, ref_out[:, 0]) < 1e-2
    assert rel(S, ref_S[0]) < 1e-2

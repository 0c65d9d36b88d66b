"""Seeded synthetic inputs with the shapes of the benchmark configurations.

The reference publishes no dataset for this path; every configuration is
synthetic.  Inputs come from ``numpy.random.default_rng(seed)`` (PCG64) drawn in
the order listed, so the oracle, the parity tests and the benchmark see the
same values.  "N(0, 0.02)" is read as standard deviation 0.02.

  cfg1  Qwen3-1.7B GQA decode: 1 seq, H=16, KV=8, Dh=128, T=1024, f32 KV
  cfg2  Qwen3-8B batched GQA decode: 64 seqs, H=32, KV=8, T_b ~ U[512, 8192], f16 KV
  cfg3  PLaMo-3 SWA prefill: 8 x 4096, H=16, KV=4, Dh=128, W=1024, bf16
  cfg4  Qwen3.5 GDN decode step: 64 seqs, NK=16, NV=32, D=128, f32 state
  cfg5  Qwen3.5 GDN chunked prefill: 8 x 8192, NK=16, NV=32, D=128, bf16 in
  cfg6  cfg4 as a whole layer step: conv1d (K=4) + g/beta + recurrence + gated
        RMSNorm around it (not a BASELINE.json configuration: the fused
        neighbours of the recurrence)
  cfg7  cfg1 as a whole attention layer step on the reference's Q8_0 cache:
        q / k RMSNorm + RoPE + K / V append + attention (not a BASELINE.json
        configuration: the fused neighbours of the append and the attention)
"""
from __future__ import annotations

import numpy as np


def _normal(rng, shape, std=1.0, dtype=np.float32):
    x = rng.standard_normal(shape, dtype=np.float32)
    if std != 1.0:
        x *= np.float32(std)
    return x.astype(dtype, copy=False)


def _l2n(x: np.ndarray) -> np.ndarray:
    n = np.sqrt((x.astype(np.float64) ** 2).sum(-1, keepdims=True))
    return (x / n).astype(np.float32)


def decode_cfg1(seed: int = 0, T: int = 1024):
    """q [1, 16, 128] (S=1), K / V caches [T, 8, 128] f32, pos_base T-1."""
    rng = np.random.default_rng(seed)
    q = _normal(rng, (16, 128))
    k = _normal(rng, (8, T, 128))
    v = _normal(rng, (8, T, 128))
    return dict(q=q[None], k=np.ascontiguousarray(k.transpose(1, 0, 2)), v=np.ascontiguousarray(v.transpose(1, 0, 2)),
                pos_base=T - 1, H=16, KV=8, Dh=128)


def decode_cfg2(seed: int = 1, batch: int = 64, lo: int = 512, hi: int = 8193, H: int = 32, KV: int = 8, Dh: int = 128):
    """Packed f16 caches: sequence b's rows are [off[b], off[b] + T_b) of
    K / V [sum(T), KV, Dh]; q [B, 1, H, Dh] f32; pos_base[b] = T_b - 1."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(lo, hi, batch).astype(np.int64)
    q = _normal(rng, (batch, H, Dh))
    total = int(lens.sum())
    k = _normal(rng, (total, KV, Dh), dtype=np.float16)
    v = _normal(rng, (total, KV, Dh), dtype=np.float16)
    off = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    return dict(q=q[:, None], k=k, v=v, lens=lens, row_offset=off, pos_base=(lens - 1).astype(np.int32),
                H=H, KV=KV, Dh=Dh)


def swa_cfg3(seed: int = 2, B: int = 8, T: int = 4096, H: int = 16, KV: int = 4, D: int = 128, window: int = 1024):
    """bf16 Q [B, T, H, D], K / V [B, T, KV, D] (as uint16 bit patterns)."""
    import torch  # bf16 rounding

    rng = np.random.default_rng(seed)
    out = {}
    for name, heads in (("q", H), ("k", KV), ("v", KV)):
        x = torch.from_numpy(_normal(rng, (B, T, heads, D))).to(torch.bfloat16)
        out[name] = x.view(torch.int16).numpy().view(np.uint16)
    out.update(window=window, H=H, KV=KV, D=D)
    return out


def gdn_decode_cfg4(seed: int = 3, batch: int = 64, NK: int = 16, NV: int = 32, D: int = 128):
    """state [B, NV, D, D] f32 (reference [dk][dv] order), qkv_conv
    [B, 1, 2*NK*D + NV*D] f32 (q, k L2-normalised), a / b [B, 1, NV]
    (alpha = exp(-softplus(a)) via aNeg = -1, dtBias = 0; beta = sigmoid(b))."""
    rng = np.random.default_rng(seed)
    state = _normal(rng, (batch, NV, D, D), std=0.02)
    q = _l2n(_normal(rng, (batch, NK, D)))
    k = _l2n(_normal(rng, (batch, NK, D)))
    v = _normal(rng, (batch, NV, D))
    a = _normal(rng, (batch, NV))
    b = _normal(rng, (batch, NV))
    qkv = np.concatenate([q.reshape(batch, -1), k.reshape(batch, -1), v.reshape(batch, -1)], 1)[:, None]
    return dict(state=state, qkv=np.ascontiguousarray(qkv), a=a[:, None].copy(), b=b[:, None].copy(),
                a_neg=-np.ones(NV, np.float32), dt_bias=np.zeros(NV, np.float32), NK=NK, NV=NV, D=D)


def gdn_prefill_cfg5(seed: int = 4, B: int = 8, T: int = 8192, NK: int = 16, NV: int = 32, D: int = 128):
    """q, k [B, T, NK, D] (L2-normalised), v [B, T, NV, D] as bf16 bit
    patterns; g = -softplus(a), beta = sigmoid(b) f32 [B, T, NV]."""
    import torch

    rng = np.random.default_rng(seed)
    q = _l2n(_normal(rng, (B, T, NK, D)))
    k = _l2n(_normal(rng, (B, T, NK, D)))
    v = _normal(rng, (B, T, NV, D))
    a = _normal(rng, (B, T, NV)).astype(np.float64)
    b = _normal(rng, (B, T, NV)).astype(np.float64)
    g = (-(np.maximum(a, 0) + np.log1p(np.exp(-np.abs(a))))).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-b))).astype(np.float32)

    def bf(x):
        return torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)

    return dict(q=bf(q), k=bf(k), v=bf(v), g=g, beta=beta, NK=NK, NV=NV, D=D)


def bf16_bits_to_f32(x: np.ndarray) -> np.ndarray:
    return (x.astype(np.uint32) << 16).view(np.float32)


def f16_bits(x: np.ndarray) -> np.ndarray:
    return x.astype(np.float16).view(np.uint16)


# Algorithmic bytes / flops per call (the roofline numerators).
def cfg2_bytes(lens: np.ndarray, H=32, KV=8, Dh=128) -> int:
    """K and V f16 read once + q read + out written (f32)."""
    return int(lens.sum()) * KV * Dh * 2 * 2 + 2 * len(lens) * H * Dh * 4


def cfg2_q8_bytes(lens: np.ndarray, H=32, KV=8, Dh=128) -> int:
    """cfg2's shapes on the reference's Q8_0 cache: K and V int8 plus one f32
    scale per 32 elements, read once; q read and out written (f32)."""
    return int(lens.sum()) * KV * (Dh + Dh // 32 * 4) * 2 + 2 * len(lens) * H * Dh * 4


def cfg2_lens(seed: int = 1, batch: int = 64, lo: int = 512, hi: int = 8193) -> np.ndarray:
    """The per-sequence context lengths of :func:`decode_cfg2` (its first draw)."""
    return np.random.default_rng(seed).integers(lo, hi, batch).astype(np.int64)


def swa_flops(T=4096, W=1024, B=8, H=16, D=128) -> int:
    """Algorithmic FLOPs of causal sliding-window attention: 4*D per (query,
    key) pair inside the window (QK^T and PV), pairs = sum_i min(i+1, W)."""
    pairs = sum(min(i + 1, W) for i in range(T)) if W > 0 else T * (T + 1) // 2
    return 4 * D * pairs * B * H


def cfg5_flops(B=8, T=8192, NV=32, C=64, D=128) -> int:
    """Canonical chunked (WY) FLOPs of the GDN prefill: per token and V head
    10*C*D + 6*D^2 (full C x C blocks, the C^3 triangular solve excluded)."""
    return B * T * NV * (10 * C * D + 6 * D * D)


def cfg5_bytes(B=8, T=8192, NK=16, NV=32, D=128) -> int:
    """HBM bytes that must move: q, k, v bf16 in, g, beta f32 in, core f32 out,
    final state f32 out."""
    return (2 * B * T * NK * D * 2 + B * T * NV * D * 2 + 2 * B * T * NV * 4 + B * T * NV * D * 4
            + B * NV * D * D * 4)


def cfg1_bytes(T=1024, H=16, KV=8, Dh=128) -> int:
    return 2 * KV * T * Dh * 4 + 2 * H * Dh * 4


def cfg4_bytes(B=64, NK=16, NV=32, D=128) -> int:
    """state read + write, q, k, v, out (f32), a, b (f32)."""
    return 2 * B * NV * D * D * 4 + B * (2 * NK * D + NV * D) * 4 + B * NV * D * 4 + 2 * B * NV * 4


def gdn_layer_cfg6(seed: int = 6, batch: int = 64, NK: int = 16, NV: int = 32, D: int = 128, K: int = 4):
    """Configuration 4's shapes through the layer's neighbours: the pre-conv
    mix qkv_mixed [B, C] (C = 2*NK*D + NV*D), conv weights [C, K] ~ N(0, 0.5),
    conv state [B, K-1, C], a / b [B, NV] (aNeg = -1, dtBias = 0), the gate z
    [B, NV*D], the norm weight gamma [D] ~ 1 + N(0, 0.1), eps 1e-6, state
    [B, NV, D, D] ~ N(0, 0.02)."""
    rng = np.random.default_rng(seed)
    C = 2 * NK * D + NV * D
    return dict(qkv=_normal(rng, (batch, C)), conv_w=_normal(rng, (C, K), std=0.5),
                conv_state=_normal(rng, (batch, K - 1, C)), a=_normal(rng, (batch, NV)), b=_normal(rng, (batch, NV)),
                z=_normal(rng, (batch, NV * D)), gamma=(1 + _normal(rng, (D,), std=0.1)).astype(np.float32),
                state=_normal(rng, (batch, NV, D, D), std=0.02), a_neg=-np.ones(NV, np.float32),
                dt_bias=np.zeros(NV, np.float32), eps=float(np.float32(1e-6)), NK=NK, NV=NV, D=D, K=K)


def cfg6_bytes(B=64, NK=16, NV=32, D=128, K=4) -> int:
    """state read + write, pre-conv mix, conv state read + write, conv
    weights, a / b, gate z, output, norm weight, aNeg / dtBias (f32)."""
    C = 2 * NK * D + NV * D
    return (2 * B * NV * D * D * 4 + B * C * 4 + 2 * B * (K - 1) * C * 4 + C * K * 4 + 2 * B * NV * 4
            + 2 * B * NV * D * 4 + D * 4 + 2 * NV * 4)


def attn_layer_cfg7(seed: int = 7, H: int = 16, KV: int = 8, Dh: int = 128, context: int = 1024, theta: float = 1e6):
    """Configuration 1's shapes as a qwen3 attention layer step: q [1, H, Dh],
    k, v [1, KV, Dh] ~ N(0, 1) (the GEMV outputs), q / k norm weights ~ 1 +
    N(0, 0.1), and a Q8_0 cache whose first context-1 rows hold random int8
    values with scales ~ |N(0, 0.02)|; the step appends row context-1."""
    rng = np.random.default_rng(seed)
    rows = context
    kq = rng.integers(-127, 128, (rows, KV, Dh), dtype=np.int8)
    vq = rng.integers(-127, 128, (rows, KV, Dh), dtype=np.int8)
    ks = np.abs(_normal(rng, (rows, KV, Dh // 32), std=0.02))
    vs = np.abs(_normal(rng, (rows, KV, Dh // 32), std=0.02))
    return dict(q=_normal(rng, (1, H, Dh)), k=_normal(rng, (1, KV, Dh)), v=_normal(rng, (1, KV, Dh)),
                q_norm=(1 + _normal(rng, (Dh,), std=0.1)).astype(np.float32),
                k_norm=(1 + _normal(rng, (Dh,), std=0.1)).astype(np.float32),
                kq=kq, ks=ks, vq=vq, vs=vs, pos=context - 1, rot=Dh, theta=theta, eps=float(np.float32(1e-6)), H=H, KV=KV, Dh=Dh)


def cfg7_bytes(H=16, KV=8, Dh=128, context=1024) -> int:
    """Q8_0 K and V read (int8 + f32 scale per 32), q / k / v in, q_out write
    and read, the appended K / V rows, norm weights, one RoPE row, out."""
    cache = 2 * context * KV * (Dh + Dh // 32 * 4)
    io = (H + 2 * KV) * Dh * 4 + 2 * H * Dh * 4 + 2 * KV * (Dh + Dh // 32 * 4) + 2 * Dh * 4 + Dh * 4 + H * Dh * 4
    return cache + io

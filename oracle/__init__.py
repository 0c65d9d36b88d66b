"""CPU oracle for hachiue's attention hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` may import this package, and only as the checker.  The product path
(``hachiue_b200``) never imports it.

Parity status: **unpinned** by the reference.  hachiue is TypeScript and no JS
runtime exists where this build runs, its WGSL twin needs a WebGPU browser, and
its tests hold no golden vectors for this path.  ``hachiue_oracle.c`` restates
the JS functions line by line (src/wasm-backend.ts:793-895, :1036-1102) with
their number semantics; ``closed_form`` below restates the same maths in dense
numpy f64 as an independent self-check.

All arrays are numpy; the C library is built by ``oracle/Makefile``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "liboracle.so")
_lock = threading.Lock()
_lib = None


def build(force: bool = False) -> str:
    """Compile the C oracle (gcc, no GPU needed).  Returns the .so path."""
    src = os.path.join(_HERE, "hachiue_oracle.c")
    if force or not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        env = dict(os.environ)
        env.setdefault("CC", "gcc")
        subprocess.run(["make", "-s", "-C", _HERE], check=True, env=env)
    return _SO


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = ctypes.CDLL(_SO)
            vp, i32, i64, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_long, ctypes.c_float
            L.oracle_append_kv_q8.argtypes = [vp, vp, vp, i32, i32, i32, i32]
            L.oracle_attention.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, i64]
            L.oracle_attention_batch.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp, vp,
                                                 i32, i32, i32]
            L.oracle_attention_q8_wgsl.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32]
            L.oracle_deltanet_gbeta.argtypes = [vp, vp, vp, vp, vp, i32, i32]
            L.oracle_deltanet_recur.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, i32, i32]
            L.oracle_deltanet_recur_wgsl.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32]
            L.oracle_deltanet_recur_batch.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i64, i64,
                                                      i64, i64, i32]
            L.oracle_f16_to_f64.argtypes = [ctypes.c_uint16]
            L.oracle_conv1d_causal.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32]
            L.oracle_deltanet_norm_gate.argtypes = [vp, vp, vp, vp, i32, i32, ctypes.c_double]
            L.oracle_rmsnorm.argtypes = [vp, vp, vp, i32, i32, ctypes.c_double, i32]
            L.oracle_append_kv_q8_wgsl.argtypes = [vp, vp, vp, i32, i32, i32, i32]
            L.oracle_rope.argtypes = [vp, i32, i32, i32, i32, i32, vp, vp]
            L.oracle_sigmoid_gate.argtypes = [vp, vp, i64]
            L.oracle_f16_to_f64.restype = ctypes.c_double
            _ = f
            _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


KV_F32, KV_F16, KV_BF16, KV_Q8_0, KV_Q8_0_WGSL = 0, 1, 2, 3, 4


def append_kv_q8(src: np.ndarray, cache_q: np.ndarray, cache_s: np.ndarray, pos_base: int) -> None:
    """appendKvQ8 (src/wasm-backend.ts:793-824): src f32 [S, KV, Dh] into the
    int8 cache [rows, KV, Dh] and f32 scales [rows, KV, Dh/32] at row pos_base."""
    S, KV, Dh = src.shape
    assert src.dtype == np.float32 and cache_q.dtype == np.int8 and cache_s.dtype == np.float32
    assert cache_q.shape[0] >= pos_base + S
    lib().oracle_append_kv_q8(_p(src), _p(cache_q), _p(cache_s), S, KV, Dh, pos_base)


def append_kv_q8_wgsl(src: np.ndarray, cache_q: np.ndarray, cache_amax: np.ndarray, pos_base: int) -> None:
    """kv_append_q8 WGSL semantics (src/kernels.ts:1287-1335): like
    :func:`append_kv_q8` in f32 with round() ties-to-even, and the scale array
    receives amax ((amax / 127) * 127 in f32)."""
    S, KV, Dh = src.shape
    assert src.dtype == np.float32 and cache_q.dtype == np.int8 and cache_amax.dtype == np.float32
    assert cache_q.shape[0] >= pos_base + S
    lib().oracle_append_kv_q8_wgsl(_p(src), _p(cache_q), _p(cache_amax), S, KV, Dh, pos_base)


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, pos_base: int, window: int = 0,
              kv_format: int = KV_F32, k_scale: np.ndarray | None = None,
              v_scale: np.ndarray | None = None, row_offset: int = 0) -> np.ndarray:
    """runAttentionQ8 (src/wasm-backend.ts:826-895) for one sequence.

    q f32 [S, H, Dh]; k / v [rows, KV, Dh] as f32, f16 (uint16 bits or float16),
    bf16 (uint16 bits) or int8 (Q8_0, with f32 scales [rows, KV, Dh/32])."""
    S, H, Dh = q.shape
    KV = k.shape[1]
    if kv_format == KV_Q8_0:
        assert k_scale is not None and v_scale is not None
        ks, vs = _p(k_scale), _p(v_scale)
    else:
        ks = vs = None
    k = np.ascontiguousarray(k)
    v = np.ascontiguousarray(v)
    out = np.zeros_like(q)
    lib().oracle_attention(_p(q), _p(k), ks, _p(v), vs, _p(out), S, H, KV, Dh, pos_base, window, kv_format,
                           row_offset)
    return out


def attention_batch(q: np.ndarray, k: np.ndarray, v: np.ndarray, pos_base: np.ndarray,
                    row_offset: np.ndarray, window: int = 0, kv_format: int = KV_F32,
                    k_scale=None, v_scale=None, threads: int = 0) -> np.ndarray:
    """Batched runAttentionQ8: q f32 [B, S, H, Dh]; sequence b reads cache rows
    row_offset[b] + j; runs sequences on `threads` host threads (0 = all)."""
    B, S, H, Dh = q.shape
    KV = k.shape[1]
    pos_base = np.ascontiguousarray(pos_base, dtype=np.int32)
    row_offset = np.ascontiguousarray(row_offset, dtype=np.int64)
    if threads <= 0:
        threads = os.cpu_count() or 1
    out = np.zeros_like(q)
    ks = _p(k_scale) if kv_format == KV_Q8_0 else None
    vs = _p(v_scale) if kv_format == KV_Q8_0 else None
    lib().oracle_attention_batch(_p(q), _p(np.ascontiguousarray(k)), ks, _p(np.ascontiguousarray(v)), vs,
                                 _p(out), B, S, H, KV, Dh, _p(pos_base), _p(row_offset), window, kv_format,
                                 threads)
    return out


def attention_q8_wgsl(q, kq, k_amax, vq, v_amax, pos_base: int, window: int = 0) -> np.ndarray:
    """attention_q8 WGSL semantics (src/kernels.ts:1341-1426), f32 arithmetic;
    the scale arrays hold amax (= the JS scale x 127)."""
    S, H, Dh = q.shape
    KV = kq.shape[1]
    out = np.zeros_like(q)
    lib().oracle_attention_q8_wgsl(_p(q), _p(kq), _p(k_amax), _p(vq), _p(v_amax), _p(out), S, H, KV, Dh,
                                   pos_base, window)
    return out


def deltanet_gbeta(a: np.ndarray, b: np.ndarray, a_neg: np.ndarray, dt_bias: np.ndarray) -> np.ndarray:
    """g / beta (src/wasm-backend.ts:1036-1045): a, b f32 [S, NV] -> [2, S, NV]."""
    S, NV = a.shape
    out = np.zeros((2, S, NV), np.float32)
    lib().oracle_deltanet_gbeta(_p(a), _p(b), _p(a_neg), _p(dt_bias), _p(out), S, NV)
    return out


def conv1d_causal(qkv_mixed: np.ndarray, conv_w: np.ndarray, conv_state: np.ndarray, load_state: bool = True):
    """Causal conv1d + SiLU (src/wasm-backend.ts:1003-1031): qkv_mixed f32
    [S, C], conv_w f32 [C, K], conv_state f32 [K-1, C].  Returns (qkv_conv
    [S, C], new conv_state); the input state is not modified."""
    S, C = qkv_mixed.shape
    K = conv_w.shape[1]
    st = np.array(conv_state, dtype=np.float32, copy=True, order="C")
    out = np.zeros((S, C), np.float32)
    lib().oracle_conv1d_causal(_p(np.ascontiguousarray(qkv_mixed, np.float32)),
                               _p(np.ascontiguousarray(conv_w, np.float32)), _p(st), _p(out), S, C, K,
                               int(load_state))
    return out, st


def deltanet_norm_gate(core: np.ndarray, z: np.ndarray, gamma: np.ndarray, eps: float) -> np.ndarray:
    """Gated RMSNorm (src/wasm-backend.ts:1104-1117): core, z f32 [rows, DV],
    gamma f32 [DV] -> y f32 [rows, DV].  ``eps`` is added as an f64 number, as
    the JS adds arch.rmsEps (which the GGUF loader reads with getFloat32,
    src/gguf.ts:312,464, so it holds an f32 value)."""
    DV = gamma.shape[0]
    c = np.ascontiguousarray(core, np.float32).reshape(-1, DV)
    zz = np.ascontiguousarray(z, np.float32).reshape(-1, DV)
    y = np.zeros_like(c)
    lib().oracle_deltanet_norm_gate(_p(c), _p(zz), _p(np.ascontiguousarray(gamma, np.float32)), _p(y), c.shape[0],
                                    DV, float(eps))
    return y.reshape(core.shape)


def rmsnorm(x: np.ndarray, gamma: np.ndarray, eps: float, add_unit_offset: bool = False) -> np.ndarray:
    """runRmsNorm (src/wasm-backend.ts:427-444) over rows of gamma's length;
    ``eps`` is added as an f64 number, like arch.rmsEps."""
    dim = gamma.shape[0]
    xx = np.ascontiguousarray(x, np.float32).reshape(-1, dim)
    y = np.zeros_like(xx)
    lib().oracle_rmsnorm(_p(xx), _p(np.ascontiguousarray(gamma, np.float32)), _p(y), xx.shape[0], dim, float(eps),
                         int(add_unit_offset))
    return y.reshape(np.shape(x))


def rope(x: np.ndarray, rotary_dim: int, pos_base: int, cos_tab: np.ndarray, sin_tab: np.ndarray) -> np.ndarray:
    """applyRope (src/wasm-backend.ts:767-791) on x [S, heads, head_dim];
    returns the rotated copy."""
    S, nh, hd = x.shape
    y = np.array(x, dtype=np.float32, copy=True, order="C")
    lib().oracle_rope(_p(y), S, nh, hd, rotary_dim, pos_base, _p(np.ascontiguousarray(cos_tab, np.float32)),
                      _p(np.ascontiguousarray(sin_tab, np.float32)))
    return y


def sigmoid_gate(gate: np.ndarray, att: np.ndarray) -> np.ndarray:
    """att * sigmoid(gate) (src/wasm-backend.ts:1152-1157); returns the product."""
    y = np.array(att, dtype=np.float32, copy=True, order="C")
    lib().oracle_sigmoid_gate(_p(np.ascontiguousarray(gate, np.float32)), _p(y), y.size)
    return y


def rope_tables(rotary_dim: int, max_pos: int, theta: float, factor: float = 1.0, orig_max_pos: int = 4096,
                beta_fast: float = 32.0, beta_slow: float = 1.0):
    """cos / sin tables [max_pos, rotary_dim / 2] f32 as buildRopeTables makes
    them (src/engine.ts:261-311): f64 inverse frequencies theta^(-2i/rotary_dim),
    blended toward freq / factor by YaRN's linear ramp when factor > 1, and
    cos / sin of pos * inv_freq scaled by 0.1 ln(factor) + 1."""
    half = rotary_dim >> 1
    mscale = 0.1 * np.log(factor) + 1.0 if factor > 1.0 else 1.0
    i = np.arange(half, dtype=np.float64)
    freq = 1.0 / np.power(float(theta), 2.0 * i / rotary_dim)
    if factor > 1.0:
        def corr_dim(n_rot):
            return rotary_dim * np.log(orig_max_pos / (n_rot * 2.0 * np.pi)) / (2.0 * np.log(theta))
        low = max(0.0, corr_dim(beta_fast))
        high = min(half - 1.0, corr_dim(beta_slow))
        if low == high:
            high += 0.001
        ramp = np.clip((i - low) / (high - low), 0.0, 1.0)
        inv = freq / factor * ramp + freq * (1.0 - ramp)
    else:
        inv = freq
    angle = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None, :]
    return (np.cos(angle) * mscale).astype(np.float32), (np.sin(angle) * mscale).astype(np.float32)


def attn_layer_step(q, k, v, q_norm, k_norm, eps, cos_tab, sin_tab, rotary_dim: int, pos_base: int, kq, ks, vq, vs,
                    gate=None):
    """One full-attention layer step of one sequence between the q / k / v
    GEMVs and attn_output, as src/wasm-backend.ts:1125-1157 (and the engine's
    dispatches, src/engine.ts:1408-1458) run it: per-head q / k RMSNorm, RoPE
    at positions pos_base.., the Q8_0 append of K and V (the caches are updated
    in place), attention_q8, and for qwen35 the sigmoid gate.  q [S, H, Dh];
    k, v [S, KV, Dh]; gate [S, H, Dh] or None.  Returns (q_normed, out)."""
    S, H, Dh = q.shape
    KV = k.shape[1]
    qn = rope(rmsnorm(q, q_norm, eps), rotary_dim, pos_base, cos_tab, sin_tab)
    kn = rope(rmsnorm(k, k_norm, eps), rotary_dim, pos_base, cos_tab, sin_tab)
    append_kv_q8(kn, kq, ks, pos_base)
    append_kv_q8(np.ascontiguousarray(v, np.float32), vq, vs, pos_base)
    out = attention(qn, kq, vq, pos_base, 0, KV_Q8_0, ks, vs)
    if gate is not None:
        out = sigmoid_gate(gate, out)
    return qn, out


def gdn_layer_step(qkv_mixed, conv_w, conv_state, a, b, a_neg, dt_bias, z, gamma, eps, state, NK: int, NV: int,
                   load_state: bool = True):
    """One Gated DeltaNet layer step for one token per sequence, as the engine
    dispatches it between the qkv / gate GEMVs and ssm_out (src/engine.ts
    :1366-1400; JS src/wasm-backend.ts:1003-1117): conv1d_causal, g / beta,
    the recurrence, the gated RMSNorm.  qkv_mixed [B, C]; conv_w [C, K];
    conv_state [B, K-1, C]; a, b [B, NV]; z [B, NV*D]; gamma [D]; state
    [B, NV, D, D].  Returns (out [B, NV*D], new conv_state, new state)."""
    B = qkv_mixed.shape[0]
    D = state.shape[-1]
    out = np.zeros((B, NV * D), np.float32)
    conv_new = np.zeros_like(conv_state, dtype=np.float32)
    st_new = np.zeros_like(state, dtype=np.float32)
    for i in range(B):
        qkv_conv, conv_new[i] = conv1d_causal(qkv_mixed[i][None], conv_w, conv_state[i], load_state)
        gb = deltanet_gbeta(a[i][None], b[i][None], a_neg, dt_bias)
        core, st_new[i] = deltanet_recur(qkv_conv, gb, state[i], NK, NV, load_state)
        out[i] = deltanet_norm_gate(core.reshape(NV, D), z[i].reshape(NV, D), gamma, eps).reshape(-1)
    return out, conv_new, st_new


def deltanet_recur(qkv_conv: np.ndarray, gbeta: np.ndarray, state: np.ndarray, NK: int, NV: int,
                   load_state: bool = True, threads: int = 1):
    """Recurrence (src/wasm-backend.ts:1047-1102).  qkv_conv f32 [S, convDim];
    gbeta f32 [2, S, NV]; state f32 [NV, D, D] ([dk][dv]).  Returns
    (core [S, NV, D], new_state); the input state is not modified."""
    S = qkv_conv.shape[0]
    D = state.shape[-1]
    st = np.array(state, dtype=np.float32, copy=True, order="C")
    core = np.zeros((S, NV, D), np.float32)
    lib().oracle_deltanet_recur(_p(np.ascontiguousarray(qkv_conv)), _p(np.ascontiguousarray(gbeta)), _p(st),
                                _p(core), S, NK, NV, D, int(load_state), threads)
    return core, st


def deltanet_recur_wgsl(qkv_conv, gbeta, state, NK: int, NV: int, load_state: bool = True):
    """deltanet_recur WGSL semantics (src/kernels.ts:1496-1573), f32 arithmetic."""
    S = qkv_conv.shape[0]
    D = state.shape[-1]
    core = np.zeros((S, NV, D), np.float32)
    out = np.zeros_like(state)
    lib().oracle_deltanet_recur_wgsl(_p(qkv_conv), _p(gbeta), _p(np.ascontiguousarray(state)), _p(core),
                                     _p(out), S, NV, D, D, NK, int(load_state))
    return core, out


def deltanet_recur_batch(qkv_conv: np.ndarray, gbeta: np.ndarray, state: np.ndarray, NK: int, NV: int,
                         load_state: bool = True, threads: int = 0):
    """Batched recurrence: qkv_conv [B, S, convDim], gbeta [B, 2, S, NV],
    state [B, NV, D, D]; sequences on `threads` host threads (0 = all)."""
    B, S, _ = qkv_conv.shape
    D = state.shape[-1]
    st = np.array(state, dtype=np.float32, copy=True, order="C")
    core = np.zeros((B, S, NV, D), np.float32)
    if threads <= 0:
        threads = os.cpu_count() or 1
    qkv_conv = np.ascontiguousarray(qkv_conv)
    gbeta = np.ascontiguousarray(gbeta)
    lib().oracle_deltanet_recur_batch(_p(qkv_conv), _p(gbeta), _p(st), _p(core), B, S, NK, NV, D,
                                      int(load_state), qkv_conv[0].size, gbeta[0].size, st[0].size,
                                      core[0].size, threads)
    return core, st


# --------------------------------------------------------------------------
# Independent dense restatements (numpy f64) used to self-check the C oracle.
# --------------------------------------------------------------------------
class closed_form:
    @staticmethod
    def attention(q, k, v, pos_base: int, window: int = 0):
        """softmax(q k^T / sqrt(Dh)) v with the causal sliding-window mask, f64.
        q [S, H, Dh]; k, v [rows, KV, Dh] as float arrays."""
        q = q.astype(np.float64)
        k = k.astype(np.float64)
        v = v.astype(np.float64)
        S, H, Dh = q.shape
        KV = k.shape[1]
        G = H // KV
        out = np.zeros((S, H, Dh))
        for qi in range(S):
            pos = pos_base + qi
            j0 = pos + 1 - window if (window > 0 and pos + 1 > window) else 0
            for h in range(H):
                kk = k[j0:pos + 1, h // G]
                vv = v[j0:pos + 1, h // G]
                s = kk @ q[qi, h] / np.sqrt(Dh)
                p = np.exp(s - s.max())
                out[qi, h] = p @ vv / p.sum()
        return out

    @staticmethod
    def deltanet(q, k, v, g, beta, state0):
        """Gated delta rule in the matrix form S <- a S (I - b k k^T) + b v k^T,
        o = S q / sqrt(D), with q, k L2-normalised (eps 1e-6).  Here S is the
        [dv, dk] matrix (the transpose of the reference's [dk][dv] storage).
        q, k [T, NV, D] (already mapped to V heads), v [T, NV, D], g, beta
        [T, NV]; state0 [NV, D(dk), D(dv)] in the reference order."""
        T, NV, D = v.shape
        S = np.transpose(state0.astype(np.float64), (0, 2, 1)).copy()
        o = np.zeros((T, NV, D))
        for t in range(T):
            for h in range(NV):
                kk = k[t, h].astype(np.float64)
                qq = q[t, h].astype(np.float64)
                kk = kk / np.sqrt(kk @ kk + 1e-6)
                qq = qq / np.sqrt(qq @ qq + 1e-6) / np.sqrt(D)
                a = np.exp(g[t, h])
                b = beta[t, h]
                S[h] = a * S[h] @ (np.eye(D) - b * np.outer(kk, kk)) + b * np.outer(v[t, h], kk)
                o[t, h] = S[h] @ qq
        return o, np.transpose(S, (0, 2, 1))


def threads_available() -> int:
    return os.cpu_count() or 1

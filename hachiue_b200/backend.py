"""The ``cuda`` backend: hachiue's attention-dispatch seam over libhachiue_cuda.

``CudaBackend.dispatch(shader_name, words, buffers)`` mirrors
``HachiueEngine.dispatch(pass, shaderName, uniformBuf, storageBufs, gx)``
(src/engine.ts:1056-1075) with the uniform words of ``mkUniform``
(src/engine.ts:1040-1054): the same op names, the same words, the same buffer
order, and ``HachiueError('hachiue: missing pipeline <name>')`` for an unknown
name.  The typed methods are the same ops with named arguments plus the
batched forms the B200 build adds.

Buffers are CUDA ``torch.Tensor`` objects (torch is only the device-memory and
stream plumbing); every call enqueues on the current torch stream of the
backend's device, like a WebGPU dispatch, and never allocates.
"""
from __future__ import annotations

import ctypes
import struct
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import (DT_BF16, DT_F32, KV_BF16, KV_F16, KV_F32, KV_Q8_0, KV_Q8_0_WGSL, HachiueError, check,
                   hcu_attention_params,
                   hcu_attn_prologue_params, hcu_conv1d_params, hcu_deltanet_params, hcu_gdn_prefill_params, hcu_gdn_step_params, hcu_kv_cache,
                   hcu_swa_params)

# The reference's op names on this path (src/kernels.ts SHADERS keys).
SHADERS = ("kv_append_q8", "attention_q8", "deltanet_gbeta", "deltanet_recur", "conv1d_causal", "deltanet_norm_gate",
           "rmsnorm", "rope", "split_q_gate", "sigmoid_gate")

_DTYPE_OF_FORMAT = {KV_F32: torch.float32, KV_F16: torch.float16, KV_BF16: torch.bfloat16, KV_Q8_0: torch.int8,
                    KV_Q8_0_WGSL: torch.int8}
_OPTIONS = {"attn_cuda_cores": _lib.OPT_ATTN_CUDA_CORES, "attn_chunk": _lib.OPT_ATTN_CHUNK,
            "gdn_scratch_mb": _lib.OPT_GDN_SCRATCH_MB, "swa_ctas": _lib.OPT_SWA_CTAS,
            "gdn_chain_cols": _lib.OPT_GDN_CHAIN_COLS}


def _current_raw_stream(index: int) -> int:
    f = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    return f(index) if f is not None else torch.cuda.current_stream(index).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise HachiueError(_lib.HCU_EINVAL, "hachiue: buffers must be CUDA tensors (no CPU fallback)")
    return t.data_ptr()


def f32_word(x: float) -> int:
    """A float uniform word, as mkUniform's setFloat32 (src/engine.ts:1043)."""
    return struct.unpack("<I", struct.pack("<f", x))[0]


@dataclass
class KVCache:
    """One layer's KV cache: K and V [rows, KV, Dh] (+ f32 scales [rows, KV,
    Dh/32] for Q8_0), the engine's kCacheQ/kCacheS/vCacheQ/vCacheS
    (src/engine.ts:339-343, :483-492)."""
    fmt: int
    k: torch.Tensor
    v: torch.Tensor
    k_scale: torch.Tensor | None = None
    v_scale: torch.Tensor | None = None

    @staticmethod
    def allocate(rows: int, kv_heads: int, head_dim: int, fmt: int = KV_Q8_0, device="cuda") -> "KVCache":
        dt = _DTYPE_OF_FORMAT[fmt]
        k = torch.zeros((rows, kv_heads, head_dim), dtype=dt, device=device)
        v = torch.zeros_like(k)
        ks = vs = None
        if fmt in (KV_Q8_0, KV_Q8_0_WGSL):
            ks = torch.zeros((rows, kv_heads, head_dim // 32), dtype=torch.float32, device=device)
            vs = torch.zeros_like(ks)
        return KVCache(fmt, k, v, ks, vs)

    @property
    def rows(self) -> int:
        return self.k.shape[0]

    def c_struct(self) -> hcu_kv_cache:
        """The C view of the cache, rebuilt only when a tensor changed (a
        decode step calls this once per layer)."""
        key = (self.fmt, self.k.data_ptr(), self.v.data_ptr(), self.k.shape[0],
               None if self.k_scale is None else self.k_scale.data_ptr(),
               None if self.v_scale is None else self.v_scale.data_ptr())
        cached = self.__dict__.get("_c_struct")
        if cached is None or cached[0] != key:
            cached = (key, hcu_kv_cache(self.fmt, self.rows, _ptr(self.k), _ptr(self.v), _ptr(self.k_scale),
                                        _ptr(self.v_scale)))
            self.__dict__["_c_struct"] = cached
        return cached[1]


class CudaBackend:
    """A libhachiue_cuda handle bound to one CUDA device."""

    def __init__(self, device: int | torch.device | None = None, workspace_bytes: int = 0):
        self.lib = _lib.load()
        if device is None:
            device = torch.cuda.current_device()
        self.device = torch.device("cuda", device if isinstance(device, int) else device.index or 0)
        h = ctypes.c_void_p()
        check(self.lib.hcu_create(self.device.index, workspace_bytes, ctypes.byref(h)))
        self._h = h
        self._stream = None  # the stream last bound to the handle
        self._attn_params = hcu_attention_params()

    # -- lifecycle -----------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_h", None):
            self.lib.hcu_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _bind_stream(self) -> None:
        """Binds the handle to the device's current torch stream (a ctypes
        call only when the stream changed since the last op)."""
        s = _current_raw_stream(self.device.index)
        if s != self._stream:
            check(self.lib.hcu_set_stream(self._h, ctypes.c_void_p(s)))
            self._stream = s

    def sync(self) -> None:
        self._bind_stream()
        check(self.lib.hcu_stream_sync(self._h))

    def device_status(self, clear: bool = True) -> int:
        self._bind_stream()
        st = ctypes.c_uint32()
        check(self.lib.hcu_device_status(self._h, ctypes.byref(st), int(clear)))
        return st.value

    def set_option(self, name: str, value: int) -> None:
        """hcu_set_option: ``attn_cuda_cores``, ``attn_chunk``,
        ``gdn_scratch_mb``, ``swa_ctas`` or ``gdn_chain_cols`` (0 restores the
        tuned default)."""
        check(self.lib.hcu_set_option(self._h, _OPTIONS[name], int(value)))

    def set_q8_convention(self, fmt: int) -> None:
        """Q8_0 scale convention of :meth:`dispatch`: ``KV_Q8_0`` (the JS
        backend's amax/127, default) or ``KV_Q8_0_WGSL`` (the WGSL ops' amax)."""
        check(self.lib.hcu_set_q8_convention(self._h, fmt))

    def selftest_dirty_tickets(self) -> None:
        """Leave every split ticket partly counted, as a decode call whose
        bounded wait gave up could; ``device_status(clear=True)`` re-arms them."""
        self._bind_stream()
        check(self.lib.hcu_selftest_dirty_tickets(self._h))

    def inject_failure(self, status: int, n: int = 1) -> None:
        """Make the next ``n`` op calls fail on the host with ``status``."""
        check(self.lib.hcu_inject_failure(self._h, status, n))

    def selftest_wait_timeout(self) -> None:
        """Launch a kernel whose bounded wait runs out (about 2 s): it records
        the timeout bit in the device status word and returns."""
        self._bind_stream()
        check(self.lib.hcu_selftest_wait_timeout(self._h))

    # -- the reference's seam --------------------------------------------------
    def dispatch(self, shader_name: str, words, buffers) -> None:
        """engine.dispatch(): ``words`` are up to eight u32 uniform words (use
        :func:`f32_word` for float words), ``buffers`` the storage buffers in
        binding order."""
        self._bind_stream()
        w = (ctypes.c_uint32 * 8)(*([int(x) & 0xFFFFFFFF for x in words] + [0] * (8 - len(words))))
        bufs = (ctypes.c_void_p * max(1, len(buffers)))(*[_ptr(b) for b in buffers])
        check(self.lib.hcu_dispatch(self._h, shader_name.encode(), w, bufs, len(buffers)))

    # -- typed ops -----------------------------------------------------------
    def kv_append(self, src: torch.Tensor, cache: KVCache, which: str, pos_base: int) -> None:
        """Append src f32 [S, KV, Dh] to K (``which='k'``) or V at row pos_base."""
        self._bind_stream()
        S, KV, Dh = src.shape
        data, scale = (cache.k, cache.k_scale) if which == "k" else (cache.v, cache.v_scale)
        if pos_base + S > cache.rows:
            raise HachiueError(_lib.HCU_EINVAL, f"hachiue: context length {pos_base + S} exceeds cache rows {cache.rows}")
        check(self.lib.hcu_kv_append(self._h, S, KV, Dh, pos_base, cache.fmt, _ptr(src.contiguous()), _ptr(data),
                                     _ptr(scale)))

    def kv_append_rows(self, src: torch.Tensor, cache: KVCache, which: str, dst_rows: torch.Tensor) -> None:
        """Append src f32 [n, KV, Dh]: row i goes to cache row dst_rows[i]
        (int64 CUDA tensor), e.g. one new token per sequence of a batch."""
        self._bind_stream()
        n, KV, Dh = src.shape
        data, scale = (cache.k, cache.k_scale) if which == "k" else (cache.v, cache.v_scale)
        check(self.lib.hcu_kv_append_rows(self._h, n, KV, Dh, cache.fmt, _ptr(src.contiguous()), _ptr(dst_rows),
                                          _ptr(data), _ptr(scale)))

    def kv_append_rows_kv(self, k_src: torch.Tensor, v_src: torch.Tensor, cache: KVCache,
                          dst_rows: torch.Tensor) -> None:
        """K and V rows of a decode step in one launch: row i of k_src / v_src
        (f32 [n, KV, Dh], contiguous) goes to cache row dst_rows[i]."""
        self._bind_stream()
        n, KV, Dh = k_src.shape
        kv = cache.c_struct()
        check(self.lib.hcu_kv_append_rows_kv(self._h, n, KV, Dh, _ptr(k_src), _ptr(v_src), _ptr(dst_rows),
                                             ctypes.byref(kv)))

    def attention(self, q: torch.Tensor, cache: KVCache, out: torch.Tensor, pos_base, window_size: int = 0,
                  kv_heads: int | None = None, kv_row_offset: torch.Tensor | None = None,
                  max_context: int = 0, seq_row_stride: int = 0, gate: torch.Tensor | None = None) -> None:
        """GQA attention of q [S, H, Dh] (or [B, S, H, Dh]) over ``cache``.

        ``pos_base`` is an int (single sequence) or an int32 CUDA tensor [B];
        batched sequences read cache rows ``kv_row_offset[b] + j``.  ``gate``
        (shaped like ``out``) applies the qwen35 output gate out *= sigmoid(gate)."""
        self._bind_stream()
        batched = q.dim() == 4
        B = q.shape[0] if batched else 1
        S, H, Dh = q.shape[-3:]
        KV = kv_heads or cache.k.shape[1]
        p = self._attn_params  # every field is set below
        p.S, p.H, p.KV, p.Dh = S, H, KV, Dh
        p.windowSize = window_size
        p.batch = B
        if isinstance(pos_base, torch.Tensor):
            p.posBase = 0
            p.pos_base = _ptr(pos_base)
            if not max_context:  # convenience only: costs a device sync; pass it on hot paths
                max_context = int(pos_base.max().item()) + S
        else:
            p.posBase = int(pos_base)
            p.pos_base = None
        p.max_context = max_context
        p.kv_row_offset = _ptr(kv_row_offset)
        p.seq_row_stride = seq_row_stride
        p.gate = _ptr(gate)
        kv = cache.c_struct()
        check(self.lib.hcu_attention(self._h, ctypes.byref(p), _ptr(q), ctypes.byref(kv), _ptr(out)))

    def attn_prologue(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_norm: torch.Tensor,
                      k_norm: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, q_out: torch.Tensor,
                      cache: KVCache, pos_base, eps: float, rotary_dim: int, gate_out: torch.Tensor | None = None,
                      kv_row_offset: torch.Tensor | None = None, seq_row_stride: int = 0) -> None:
        """Fused split / q-k RMSNorm / RoPE / K-V append: q f32 [(B,) S, H, Dh]
        (or [(B,) S, H, 2*Dh] with ``gate_out``, the qwen35 doubled
        projection); k, v f32 [(B,) S, KV, Dh]; q_out [(B,) S, H, Dh]."""
        self._bind_stream()
        batched = k.dim() == 4
        p = hcu_attn_prologue_params()
        p.batch = k.shape[0] if batched else 1
        p.S, p.KV, p.Dh = k.shape[-3], k.shape[-2], k.shape[-1]
        p.H = q.shape[-2]
        p.rotaryDim = rotary_dim
        p.split_gate = int(gate_out is not None)
        p.eps = float(eps)
        if isinstance(pos_base, torch.Tensor):
            p.posBase, p.pos_base = 0, _ptr(pos_base)
        else:
            p.posBase, p.pos_base = int(pos_base), None
        p.kv_row_offset = _ptr(kv_row_offset)
        p.seq_row_stride = seq_row_stride
        kv = cache.c_struct()
        check(self.lib.hcu_attn_prologue(self._h, ctypes.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(q_norm),
                                         _ptr(k_norm), _ptr(cos), _ptr(sin), _ptr(q_out), _ptr(gate_out),
                                         ctypes.byref(kv)))

    def rmsnorm(self, x: torch.Tensor, gamma: torch.Tensor, y: torch.Tensor, eps: float,
                add_unit_offset: bool = False) -> None:
        """rmsnorm over rows of gamma's length."""
        self._bind_stream()
        dim = gamma.shape[0]
        check(self.lib.hcu_rmsnorm(self._h, x.numel() // dim, dim, float(eps), int(add_unit_offset), _ptr(x),
                                   _ptr(gamma), _ptr(y)))

    def rope(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, rotary_dim: int, pos_base: int) -> None:
        """RoPE in place on x f32 [S, heads, head_dim]."""
        self._bind_stream()
        S, heads, hd = x.shape
        check(self.lib.hcu_rope(self._h, S, heads, hd, rotary_dim, pos_base, _ptr(cos), _ptr(sin), _ptr(x)))

    def deltanet_gbeta(self, a: torch.Tensor, b: torch.Tensor, a_neg: torch.Tensor, dt_bias: torch.Tensor,
                       out: torch.Tensor) -> None:
        """g / beta of a, b [S, NV] into out [2, S, NV]."""
        self._bind_stream()
        S, NV = a.shape
        check(self.lib.hcu_deltanet_gbeta(self._h, S, NV, _ptr(a), _ptr(b), _ptr(a_neg), _ptr(dt_bias), _ptr(out)))

    @staticmethod
    def _dn_params(qkv_conv: torch.Tensor, NK: int, NV: int, D: int, load_state: bool) -> hcu_deltanet_params:
        p = hcu_deltanet_params()
        batched = qkv_conv.dim() == 3
        p.batch = qkv_conv.shape[0] if batched else 1
        p.S = qkv_conv.shape[-2]
        p.H, p.DK, p.DV, p.HK = NV, D, D, NK
        p.loadState = int(bool(load_state))
        return p

    def deltanet_recur(self, qkv_conv: torch.Tensor, gbeta: torch.Tensor, state_in: torch.Tensor,
                       core: torch.Tensor, state_out: torch.Tensor, NK: int, NV: int, load_state: bool = True,
                       D: int = 128) -> None:
        """deltanet_recur: qkv_conv [(B,) S, convDim], gbeta [(B,) 2, S, NV],
        states [(B,) NV, D, D], core [(B,) S, NV, D]."""
        self._bind_stream()
        p = self._dn_params(qkv_conv, NK, NV, D, load_state)
        check(self.lib.hcu_deltanet_recur(self._h, ctypes.byref(p), _ptr(qkv_conv), _ptr(gbeta), _ptr(state_in),
                                          _ptr(core), _ptr(state_out)))

    def deltanet_decode(self, qkv_conv: torch.Tensor, a: torch.Tensor, b: torch.Tensor, a_neg: torch.Tensor,
                        dt_bias: torch.Tensor, state_in: torch.Tensor, core: torch.Tensor, state_out: torch.Tensor,
                        NK: int, NV: int, load_state: bool = True, D: int = 128) -> None:
        """deltanet_gbeta fused into deltanet_recur (a, b [(B,) S, NV])."""
        self._bind_stream()
        p = self._dn_params(qkv_conv, NK, NV, D, load_state)
        check(self.lib.hcu_deltanet_decode(self._h, ctypes.byref(p), _ptr(qkv_conv), _ptr(a), _ptr(b), _ptr(a_neg),
                                           _ptr(dt_bias), _ptr(state_in), _ptr(core), _ptr(state_out)))

    def conv1d_causal(self, x: torch.Tensor, w: torch.Tensor, state_in: torch.Tensor, y: torch.Tensor,
                      state_out: torch.Tensor, load_state: bool = True) -> None:
        """conv1d_causal + SiLU: x, y f32 [(B,) S, C]; w f32 [C, K]; conv states
        f32 [(B,) K-1, C] (state_in may be state_out)."""
        self._bind_stream()
        p = hcu_conv1d_params()
        p.batch = x.shape[0] if x.dim() == 3 else 1
        p.S, p.C = x.shape[-2], x.shape[-1]
        p.K = w.shape[1]
        p.loadState = int(bool(load_state))
        check(self.lib.hcu_conv1d_causal(self._h, ctypes.byref(p), _ptr(x), _ptr(w), _ptr(state_in), _ptr(y),
                                         _ptr(state_out)))

    def deltanet_norm_gate(self, core: torch.Tensor, z: torch.Tensor, gamma: torch.Tensor, y: torch.Tensor,
                           eps: float) -> None:
        """Gated RMSNorm over rows of DV: core, z, y f32 [..., DV]; gamma f32 [DV]."""
        self._bind_stream()
        DV = gamma.shape[0]
        check(self.lib.hcu_deltanet_norm_gate(self._h, core.numel() // DV, DV, float(eps), _ptr(core), _ptr(z),
                                              _ptr(gamma), _ptr(y)))

    def gdn_layer_step(self, qkv_mixed: torch.Tensor, conv_w: torch.Tensor, conv_in: torch.Tensor,
                       conv_out: torch.Tensor, a: torch.Tensor, b: torch.Tensor, a_neg: torch.Tensor,
                       dt_bias: torch.Tensor, z: torch.Tensor, gamma: torch.Tensor, state_in: torch.Tensor,
                       state_out: torch.Tensor, out: torch.Tensor, NK: int, NV: int, eps: float,
                       load_state: bool = True, D: int = 128) -> None:
        """One GDN layer step for one token per sequence, fused (conv1d_causal,
        g / beta, recurrence, gated RMSNorm): qkv_mixed f32 [B, C]; conv_w f32
        [C, 4]; conv states f32 [B, 3, C] (in and out different); a, b f32
        [B, NV]; z f32 [B, NV*D]; gamma f32 [D]; states f32 [B, NV, D, D];
        out f32 [B, NV*D]."""
        self._bind_stream()
        p = hcu_gdn_step_params()
        p.batch = qkv_mixed.shape[0] if qkv_mixed.dim() == 2 else 1
        p.H, p.HK, p.DK, p.DV, p.K = NV, NK, D, D, conv_w.shape[1]
        p.loadState = int(bool(load_state))
        p.eps = float(eps)
        check(self.lib.hcu_gdn_layer_step(self._h, ctypes.byref(p), _ptr(qkv_mixed), _ptr(conv_w), _ptr(conv_in),
                                          _ptr(conv_out), _ptr(a), _ptr(b), _ptr(a_neg), _ptr(dt_bias), _ptr(z),
                                          _ptr(gamma), _ptr(state_in), _ptr(state_out), _ptr(out)))

    def swa_prefill(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor,
                    window: int = 0) -> None:
        """Causal sliding-window attention over whole prompts: q bf16 [B, T, H, D],
        k / v bf16 [B, T, KV, D], out bf16 or f32 [B, T, H, D]; window 0 = causal."""
        self._bind_stream()
        for t in (q, k, v):
            if t.dtype != torch.bfloat16 or not t.is_contiguous():
                raise HachiueError(_lib.HCU_EINVAL, "hachiue: swa_prefill takes contiguous bf16 q / k / v")
        B, T, H, D = q.shape
        p = hcu_swa_params(B, T, H, k.shape[2], D, window,
                           DT_BF16 if out.dtype == torch.bfloat16 else DT_F32)
        check(self.lib.hcu_swa_prefill(self._h, ctypes.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(out)))

    def deltanet_chunked_prefill(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor,
                                 beta: torch.Tensor, core: torch.Tensor, state_out: torch.Tensor,
                                 state_in: torch.Tensor | None = None, snapshots: torch.Tensor | None = None,
                                 snap_every: int = 0) -> None:
        """Gated DeltaNet over whole prompts, 64-token chunks on the tensor cores.

        q, k bf16 [B, T, NK, D]; v bf16 [B, T, NV, D] (token-major views with
        unit stride inside a head are accepted); g, beta f32 [B, T, NV];
        core f32 [B, T, NV, D]; states f32 [B, NV, D, D] ([dk][dv]).
        ``state_in`` None starts from a zero state.  With ``snapshots`` f32
        [B, T // (64 * snap_every), NV, D, D], snapshot j receives the state
        after token 64 * snap_every * (j + 1) (for prefix reuse)."""
        self._bind_stream()
        B, T, NK, D = q.shape
        NV = v.shape[2]
        for t in (q, k, v):
            if t.dtype != torch.bfloat16 or t.stride(3) != 1 or t.stride(2) != D:
                raise HachiueError(_lib.HCU_EINVAL, "hachiue: q / k / v must be bf16 with contiguous heads")
        for t in (g, beta):
            if t.dtype != torch.float32 or t.stride(2) != 1:
                raise HachiueError(_lib.HCU_EINVAL, "hachiue: g / beta must be f32 [B, T, NV]")
        p = hcu_gdn_prefill_params()
        p.B, p.T, p.NK, p.NV, p.D = B, T, NK, NV, D
        p.load_state = int(state_in is not None)
        p.q_row_stride, p.k_row_stride, p.v_row_stride = q.stride(1), k.stride(1), v.stride(1)
        p.q_seq_stride, p.k_seq_stride, p.v_seq_stride = q.stride(0), k.stride(0), v.stride(0)
        p.gb_row_stride, p.gb_seq_stride = g.stride(1), g.stride(0)
        if beta.stride() != g.stride():
            raise HachiueError(_lib.HCU_EINVAL, "hachiue: g and beta must share strides")
        if snapshots is not None:
            n_snap = T // (64 * snap_every) if snap_every > 0 else 0
            if (snapshots.dtype != torch.float32 or not snapshots.is_contiguous()
                    or tuple(snapshots.shape) != (B, n_snap, NV, D, D)):
                raise HachiueError(_lib.HCU_EINVAL,
                                   f"hachiue: snapshots must be contiguous f32 [{B}, {n_snap}, {NV}, {D}, {D}]")
            check(self.lib.hcu_deltanet_chunked_prefill_snap(
                self._h, ctypes.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(state_in),
                _ptr(core), _ptr(state_out), snap_every, _ptr(snapshots)))
            return
        check(self.lib.hcu_deltanet_chunked_prefill(self._h, ctypes.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(g),
                                                    _ptr(beta), _ptr(state_in), _ptr(core), _ptr(state_out)))

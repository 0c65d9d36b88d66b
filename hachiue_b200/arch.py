"""Shape parameters of the hot path, the layer rules that pick each layer's
kernel, and the per-layer device state a decode loop owns.

Mirrors the reference's ``ModelArch`` / ``HybridLayerConfig`` /
``SlidingWindowConfig`` (src/types.ts:66-103) as ``parseModelArch`` fills
them (src/gguf.ts:497-525), and the engine's per-layer buffers and counters
(src/engine.ts:339-347, :476-501, :900-902, :1352-1353, :1481-1483).  Only the
fields this path reads are kept; the loader, tokenizer and GEMV weights stay
in the reference.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from ._lib import KV_Q8_0
from .backend import KVCache


def swa_layer_types(layers: int, pattern: int) -> list[str]:
    """plamo3: every ``pattern``-th layer is full attention, the rest use the
    sliding window (src/gguf.ts:502: ``(li + 1) % pattern === 0 ? 'full'``)."""
    if pattern < 1:
        raise ValueError("hachiue: sliding_window_pattern must be >= 1")
    return ["full" if (li + 1) % pattern == 0 else "swa" for li in range(layers)]


def hybrid_layer_types(layers: int, interval: int) -> list[str]:
    """qwen35: the last layer of every ``interval`` is full attention, the rest
    Gated DeltaNet (src/gguf.ts:516: ``li % interval === interval - 1``)."""
    if interval < 1:
        raise ValueError("hachiue: full_attention_interval must be >= 1")
    return ["full" if li % interval == interval - 1 else "linear" for li in range(layers)]


@dataclass
class SlidingWindowConfig:
    window_size: int
    pattern: int
    layer_types: list[str]


@dataclass
class HybridLayerConfig:
    layer_types: list[str]
    linear_key_heads: int    # NK (ssm.group_count)
    linear_value_heads: int  # NV (ssm.time_step_rank)
    linear_head_dim: int     # DK = DV (ssm.state_size)
    conv_kernel: int         # ssm.conv_kernel

    @property
    def conv_dim(self) -> int:
        """Channels of the causal conv: q, k (NK heads each) and v (NV heads)."""
        return (2 * self.linear_key_heads + self.linear_value_heads) * self.linear_head_dim


@dataclass
class ModelArch:
    arch_name: str  # 'qwen3' | 'qwen35' | 'plamo3'
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    rms_eps: float
    rotary_dim: int
    max_positions: int
    hybrid: HybridLayerConfig | None = None
    swa: SlidingWindowConfig | None = None

    def layer_kind(self, li: int) -> str:
        """'linear' (Gated DeltaNet), 'swa' or 'full' attention."""
        if not 0 <= li < self.layers:
            raise IndexError(f"hachiue: layer {li} of {self.layers}")
        if self.hybrid is not None and self.hybrid.layer_types[li] == "linear":
            return "linear"
        if self.swa is not None and self.swa.layer_types[li] == "swa":
            return "swa"
        return "full"

    def attention_window(self, li: int) -> int:
        """The attention's windowSize uniform word for layer li: the window on
        SWA layers, 0 (whole context) otherwise (src/engine.ts:1284-1286)."""
        return self.swa.window_size if self.layer_kind(li) == "swa" else 0


@dataclass
class LayerStates:
    """The device state of one sequence's decode loop: a KV cache of
    ``max_seq_len`` rows per attention layer (the engine's Q8_0 kCache / vCache
    maps by default) and, per Gated DeltaNet layer, two recurrent states
    [NV, DK, DV] and two conv states [K-1, convDim], ping-ponged by
    ``ssm_parity``.  ``cache_pos`` counts the tokens already in the cache."""
    arch: ModelArch
    max_seq_len: int
    kv_format: int = KV_Q8_0
    device: str | torch.device = "cuda"
    caches: dict[int, KVCache] = field(default_factory=dict)
    rec_states: dict[int, tuple[torch.Tensor, torch.Tensor]] = field(default_factory=dict)
    conv_states: dict[int, tuple[torch.Tensor, torch.Tensor]] = field(default_factory=dict)
    cache_pos: int = 0
    ssm_parity: int = 0

    def __post_init__(self):
        a = self.arch
        for li in range(a.layers):
            if a.layer_kind(li) == "linear":
                hy = a.hybrid
                d = hy.linear_head_dim
                rec = [torch.zeros((hy.linear_value_heads, d, d), device=self.device) for _ in range(2)]
                conv = [torch.zeros((hy.conv_kernel - 1, hy.conv_dim), device=self.device) for _ in range(2)]
                self.rec_states[li] = (rec[0], rec[1])
                self.conv_states[li] = (conv[0], conv[1])
            else:
                self.caches[li] = KVCache.allocate(self.max_seq_len, a.kv_heads, a.head_dim, self.kv_format,
                                                   device=self.device)

    @property
    def load_state(self) -> bool:
        """The recurrences start from the stored state once a token is cached
        (src/engine.ts:1352: ``loadState = cachePos > 0``)."""
        return self.cache_pos > 0

    def gdn_states(self, li: int) -> tuple[torch.Tensor, torch.Tensor]:
        """(state in, state out) of Gated DeltaNet layer li for this segment."""
        s = self.rec_states[li]
        return s[self.ssm_parity], s[self.ssm_parity ^ 1]

    def conv_state_pair(self, li: int) -> tuple[torch.Tensor, torch.Tensor]:
        """(conv state in, conv state out) of layer li for this segment."""
        s = self.conv_states[li]
        return s[self.ssm_parity], s[self.ssm_parity ^ 1]

    def advance(self, tokens: int) -> None:
        """After a segment of ``tokens`` tokens: the states written become the
        next segment's input (src/engine.ts:1481-1483)."""
        if self.cache_pos + tokens > self.max_seq_len:
            raise ValueError(f"hachiue: context length {self.cache_pos + tokens} exceeds {self.max_seq_len}")
        if self.arch.hybrid is not None:
            self.ssm_parity ^= 1
        self.cache_pos += tokens

    def reset(self) -> None:
        """resetCache (src/engine.ts:900-902): stale contents are masked by
        cache_pos and replaced because load_state is false."""
        self.cache_pos = 0
        self.ssm_parity = 0

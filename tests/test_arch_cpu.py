"""Layer rules and per-layer decode state (hachiue_b200/arch.py) against the
reference's parseModelArch loops (src/gguf.ts:497-525) and the engine's buffer
sizes and counters (src/engine.ts:476-501, :900-902, :1352, :1481-1483)."""
import pytest
import torch

from hachiue_b200 import KV_F16, KV_Q8_0
from hachiue_b200.arch import (HybridLayerConfig, LayerStates, ModelArch, SlidingWindowConfig, hybrid_layer_types,
                               swa_layer_types)


def test_layer_rules():
    assert swa_layer_types(8, 4) == ["swa", "swa", "swa", "full"] * 2
    assert swa_layer_types(5, 8) == ["swa"] * 5
    assert swa_layer_types(3, 1) == ["full"] * 3
    assert hybrid_layer_types(8, 4) == ["linear", "linear", "linear", "full"] * 2
    assert hybrid_layer_types(6, 1) == ["full"] * 6
    with pytest.raises(ValueError):
        hybrid_layer_types(4, 0)


def plamo3(layers=8):
    return ModelArch("plamo3", layers, 16, 4, 128, 1e-6, 128, 4096,
                     swa=SlidingWindowConfig(1024, 4, swa_layer_types(layers, 4)))


def qwen35(layers=8):
    return ModelArch("qwen35", layers, 16, 2, 256, 1e-6, 64, 4096,
                     hybrid=HybridLayerConfig(hybrid_layer_types(layers, 4), 16, 32, 128, 4))


def test_layer_kind_and_window():
    a = plamo3()
    assert [a.layer_kind(li) for li in range(8)] == ["swa"] * 3 + ["full"] + ["swa"] * 3 + ["full"]
    assert [a.attention_window(li) for li in range(4)] == [1024, 1024, 1024, 0]
    b = qwen35()
    assert [b.layer_kind(li) for li in range(4)] == ["linear"] * 3 + ["full"]
    assert b.attention_window(3) == 0
    with pytest.raises(IndexError):
        b.layer_kind(8)


def test_state_sizes_match_the_engine():
    a = qwen35(4)
    st = LayerStates(a, max_seq_len=64, kv_format=KV_Q8_0, device="cpu")
    kv_dim = a.kv_heads * a.head_dim
    c = st.caches[3]
    assert c.k.numel() == 64 * kv_dim and c.k.dtype == torch.int8           # qBytes = maxSeqLen * kvDim
    assert c.k_scale.numel() * 4 == 64 * (kv_dim // 32) * 4                 # sBytes
    hy = a.hybrid
    conv_dim = (hy.linear_key_heads * 2 + hy.linear_value_heads) * hy.linear_head_dim
    for li in range(3):
        assert li not in st.caches
        for t in st.conv_states[li]:
            assert t.numel() * 4 == (hy.conv_kernel - 1) * conv_dim * 4     # convStateBytes
        for t in st.rec_states[li]:
            assert t.numel() * 4 == hy.linear_value_heads * 128 * 128 * 4   # recStateBytes
    p = LayerStates(plamo3(8), max_seq_len=32, kv_format=KV_F16, device="cpu")
    assert sorted(p.caches) == list(range(8)) and not p.rec_states


def test_counters_and_ping_pong():
    st = LayerStates(qwen35(4), max_seq_len=16, device="cpu")
    assert not st.load_state
    s_in, s_out = st.gdn_states(0)
    assert s_in is st.rec_states[0][0] and s_out is st.rec_states[0][1]
    st.advance(5)
    assert st.load_state and st.cache_pos == 5 and st.ssm_parity == 1
    s_in, s_out = st.gdn_states(0)
    assert s_in is st.rec_states[0][1] and s_out is st.rec_states[0][0]
    c_in, c_out = st.conv_state_pair(1)
    assert c_in is st.conv_states[1][1]
    st.advance(1)
    assert st.ssm_parity == 0 and st.cache_pos == 6
    with pytest.raises(ValueError):
        st.advance(11)
    st.reset()
    assert st.cache_pos == 0 and st.ssm_parity == 0 and not st.load_state
    # without GDN layers the parity never flips (src/engine.ts:1481)
    p = LayerStates(plamo3(4), max_seq_len=16, device="cpu")
    p.advance(3)
    assert p.ssm_parity == 0

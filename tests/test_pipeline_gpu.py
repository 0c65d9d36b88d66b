"""HostPipeline (hachiue_b200/pipeline.py): decode steps fed from pinned host
memory over two buffer slots and three streams.  Six steps with distinct
host inputs and outputs go through both slots three times; every step's
output must equal, bit for bit, the same attention call made directly on the
device, and match the oracle (relative L2 <= 1e-4)."""
import numpy as np
import pytest
import torch

import oracle
from hachiue_b200 import KV_F16
from hachiue_b200.backend import KVCache
from hachiue_b200.pipeline import HostPipeline
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu
dev = "cuda"


def test_pipelined_steps_match_direct_calls(backend):
    rng = np.random.default_rng(17)
    B, H, KV, Dh, steps = 4, 8, 2, 128, 6
    lens = np.array([200, 513, 64, 1000])
    off = np.concatenate([[0], np.cumsum(lens)[:-1]])
    k = rng.standard_normal((lens.sum(), KV, Dh), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((lens.sum(), KV, Dh), dtype=np.float32).astype(np.float16)
    cache = KVCache(KV_F16, torch.from_numpy(k.view(np.int16)).to(dev).view(torch.float16),
                    torch.from_numpy(v.view(np.int16)).to(dev).view(torch.float16))
    pos = torch.tensor(lens - 1, dtype=torch.int32, device=dev)
    offs = torch.tensor(off, dtype=torch.int64, device=dev)
    qs = [rng.standard_normal((B, 1, H, Dh), dtype=np.float32) for _ in range(steps)]
    q_host = [torch.from_numpy(q).pin_memory() for q in qs]
    out_host = [torch.full((B, 1, H, Dh), float("nan")).pin_memory() for _ in range(steps)]

    def compute(ins, outs):
        backend.attention(ins[0], cache, outs[0], pos, 0, kv_row_offset=offs, max_context=int(lens.max()))

    pipe = HostPipeline(dev, [((B, 1, H, Dh), torch.float32)], [((B, 1, H, Dh), torch.float32)])
    pipe.begin()
    for i in range(steps):
        pipe.submit([q_host[i]], [out_host[i]], compute)
    pipe.drain()
    torch.cuda.synchronize()
    for i in range(steps):
        direct = torch.zeros((B, 1, H, Dh), device=dev)
        backend.attention(torch.from_numpy(qs[i]).to(dev), cache, direct, pos, 0, kv_row_offset=offs,
                          max_context=int(lens.max()))
        torch.cuda.synchronize()
        got = out_host[i].numpy()
        assert np.array_equal(got, direct.cpu().numpy()), i
        ref = oracle.attention_batch(qs[i], k.view(np.uint16), v.view(np.uint16), lens - 1, off, 0, oracle.KV_F16)
        assert rel_l2(got, ref) < 1e-4, i
    assert backend.device_status() == 0

"""Single-process multi-GPU through the C ABI (hcu_comm_create / hcu_allgather,
one NCCL communicator per device by ncclCommInitAll), as a Node host driving
several GPUs would use it: decode attention sharded by KV head over two GPUs,
joined by the all-gather, against the unsharded result.  Skipped with fewer
than two GPUs."""
import numpy as np
import pytest
import torch

from hachiue_b200 import KV_F16, CudaBackend
from hachiue_b200.backend import KVCache
from hachiue_b200.dist import DeviceComm, kv_head_range
from tests.conftest import rel_l2

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs in this process")]


def test_head_sharded_decode_over_two_gpus():
    rng = np.random.default_rng(17)
    S, H, KV, D, pos = 1, 32, 8, 128, 700
    G = H // KV
    q = rng.standard_normal((S, H, D), dtype=np.float32)
    k = rng.standard_normal((pos + 1, KV, D)).astype(np.float16)
    v = rng.standard_normal((pos + 1, KV, D)).astype(np.float16)
    # unsharded on GPU 0
    be0 = CudaBackend(0)
    full = torch.zeros((S, H, D), device="cuda:0")
    be0.attention(torch.from_numpy(q).to("cuda:0"), KVCache(KV_F16, torch.from_numpy(k).to("cuda:0"),
                                                             torch.from_numpy(v).to("cuda:0")), full, pos)
    # rank r on GPU r owns KV heads [lo, hi) and their query heads
    devs, bes, sends, recvs = [0, 1], [be0, CudaBackend(1)], [], []
    for r, d in enumerate(devs):
        lo, hi = kv_head_range(KV, 2, r)
        dev = f"cuda:{d}"
        cache = KVCache(KV_F16, torch.from_numpy(np.ascontiguousarray(k[:, lo:hi])).to(dev),
                        torch.from_numpy(np.ascontiguousarray(v[:, lo:hi])).to(dev))
        out = torch.zeros((S, (hi - lo) * G, D), device=dev)
        with torch.cuda.device(d):
            bes[r].attention(torch.from_numpy(np.ascontiguousarray(q[:, lo * G:hi * G])).to(dev), cache, out, pos)
        sends.append(out)
        recvs.append(torch.zeros((2,) + tuple(out.shape), device=dev))
    comm = DeviceComm(devs)
    try:
        comm.all_gather(sends, recvs)
        for d in devs:
            torch.cuda.synchronize(d)
    finally:
        comm.close()
    joined = recvs[0].permute(1, 0, 2, 3).reshape(S, H, D)  # [rank][S][H_local][D] -> [S][H][D]
    assert rel_l2(joined.cpu().numpy(), full.cpu().numpy()) < 1e-5
    assert torch.equal(recvs[0].cpu(), recvs[1].cpu())
    for be in bes:
        assert be.device_status() == 0

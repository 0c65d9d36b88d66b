"""hcu_attention_noalloc: decode attention for callers that cannot allocate.

Some callers cannot let this library call cudaMalloc: a serving process that
reserves its whole HBM budget in its own pool, or a plugin behind a stateless
FFI call that cannot keep a handle (creating one allocates a workspace).  The
entry point takes no handle and uses a fixed-size static device array as its
split-K scratch.  This test calls it through the C ABI and checks it against
the allocating entry point (hcu_attention) and against the oracle
(runAttentionQ8's restatement) on two calls in a row, for the tensor-core path
(f16 cache) and the CUDA-core path (f32 cache); checks that its status word,
the only failure report such a caller has, reads 0 and clears; then checks
that an oversized call is refused with a clear error.  It is collected last so
a failure here never hides the other tests' results.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from hachiue_b200 import KV_F16, KV_F32, CudaBackend, HachiueError, _lib
from hachiue_b200.backend import KVCache
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _params(q, pos_base, row_offset, max_context, KV):
    B, S, H, Dh = q.shape
    p = _lib.hcu_attention_params()
    p.S, p.H, p.KV, p.Dh = S, H, KV, Dh
    p.batch = B
    p.max_context = max_context
    p.pos_base = pos_base.data_ptr()
    p.kv_row_offset = row_offset.data_ptr()
    return p


def _noalloc(q, cache, out, p):
    lib = _lib.load()
    kv = cache.c_struct()
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.hcu_attention_noalloc(ctypes.byref(p), q.data_ptr(), ctypes.byref(kv), out.data_ptr(),
                                         ctypes.c_void_p(stream)))


@pytest.mark.parametrize("fmt", [KV_F16, KV_F32])
def test_noalloc_matches_hcu_attention_twice(fmt):
    dev = "cuda"
    rng = np.random.default_rng(31 + fmt)
    lens = np.array([300, 5000, 1, 2049, 777, 4096, 128, 3001])
    off = np.concatenate([[0], np.cumsum(lens)[:-1]])
    B, H, KV, Dh = len(lens), 32, 8, 128
    kf = rng.standard_normal((lens.sum(), KV, Dh), dtype=np.float32)
    vf = rng.standard_normal((lens.sum(), KV, Dh), dtype=np.float32)
    dt = torch.float16 if fmt == KV_F16 else torch.float32
    cache = KVCache(fmt, torch.from_numpy(kf).to(dev).to(dt), torch.from_numpy(vf).to(dev).to(dt))
    q = torch.from_numpy(rng.standard_normal((B, 1, H, Dh), dtype=np.float32)).to(dev)
    pos = torch.tensor(lens - 1, dtype=torch.int32, device=dev)
    roff = torch.tensor(off, dtype=torch.int64, device=dev)
    maxc = int(lens.max())

    be = CudaBackend(0)
    ref = torch.zeros_like(q)
    be.attention(q, cache, ref, pos, 0, kv_row_offset=roff, max_context=maxc)
    torch.cuda.synchronize()
    ref_np = ref.cpu().numpy()
    be.close()

    if fmt == KV_F16:
        kc, vc, ofmt = kf.astype(np.float16).view(np.uint16), vf.astype(np.float16).view(np.uint16), oracle.KV_F16
    else:
        kc, vc, ofmt = kf, vf, oracle.KV_F32
    want = oracle.attention_batch(q.cpu().numpy(), kc, vc, lens - 1, off, 0, ofmt)
    assert rel_l2(ref_np, want) < TOL

    p = _params(q, pos, roff, maxc, KV)
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        _noalloc(q, cache, out, p)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        assert rel_l2(got, ref_np) < TOL
        assert rel_l2(got, want) < TOL
        assert _status(clear=False) == 0


def _status(clear: bool) -> int:
    lib = _lib.load()
    st = ctypes.c_uint32(0xFFFFFFFF)
    _lib.check(lib.hcu_attention_noalloc_status(ctypes.byref(st), int(clear),
                                                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    return st.value


def test_noalloc_status_word_reads_and_clears():
    """The handle-free status word: 0 after good calls, and a clear leaves it 0."""
    torch.zeros(1, device="cuda")  # a context on the current device
    assert _status(clear=True) == 0
    assert _status(clear=False) == 0


def test_noalloc_refuses_oversized_calls():
    dev = "cuda"
    B, H, KV, Dh = 4000, 32, 8, 128  # 32000 units: their partials exceed the static scratch
    q = torch.zeros((B, 1, H, Dh), device=dev)
    cache = KVCache.allocate(16, KV, Dh, KV_F16)
    pos = torch.zeros(B, dtype=torch.int32, device=dev)
    roff = torch.zeros(B, dtype=torch.int64, device=dev)
    p = _params(q, pos, roff, 16, KV)
    with pytest.raises(HachiueError, match="HCU_NOALLOC_SCRATCH_BYTES"):
        _noalloc(q, cache, torch.zeros_like(q), p)

"""Multi-GPU partitioning of the attention hot path (one process per GPU).

The path shards by (sequence, KV / QK head): every unit is independent, so a
rank computes its units alone and the per-head outputs are joined with one
all-gather (NCCL over NVLink on GPUs, gloo on CPU).  The reference has no
multi-device path (one GPUDevice per engine, src/engine.ts:320).

Partitions:
  * by sequence (``seq_range``): rank r owns a contiguous range of sequences
    with all their heads (the benchmark's weak-scaling layout);
  * by KV head (``kv_head_range``): rank r owns a contiguous range of KV heads
    of every sequence and the G = H / KV query heads that read them, so each
    rank stores only its heads' cache.  GDN layers shard by QK head the same
    way: V heads h and h + NK read QK head h (tiled map), so a rank owning QK
    heads [a, b) owns V heads {h : h % NK in [a, b)}.

Executors: ``HeadShardedDecode`` (decode attention), ``HeadShardedSWA`` (SWA
prefill) and ``QKHeadShardedGDN`` (GDN decode and chunked prefill); the
all-gathers are torch.distributed's (``gather_*``) or this library's own
NCCL communicator (``RankComm``, ``DeviceComm``).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def _split(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous near-equal split of range(n): rank's [lo, hi)."""
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def seq_range(batch: int, world: int, rank: int) -> tuple[int, int]:
    return _split(batch, world, rank)


def kv_head_range(kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    if kv_heads % world:
        raise ValueError(f"hachiue: {kv_heads} KV heads do not split over {world} ranks")
    return _split(kv_heads, world, rank)


def v_heads_of_qk_range(nk: int, nv: int, lo: int, hi: int) -> list[int]:
    """V heads served by QK heads [lo, hi) under the tiled map h % NK."""
    return [h for h in range(nv) if lo <= h % nk < hi]


def gather_seq_shards(local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather equal sequence shards [b_local, ...] into [world*b_local, ...]."""
    world = dist.get_world_size(group)
    out = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    return out


def gather_head_shards(local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather per-head outputs: local [B, S, H_local, D] (this rank's
    contiguous head range) -> [B, S, world*H_local, D] on every rank.  The
    collective moves [world][B, S, H_local, D] (each rank's block contiguous);
    one local permute restores head order."""
    world = dist.get_world_size(group)
    B, S, hl, D = local.shape
    buf = torch.empty((world, B, S, hl, D), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(buf.view(world * B, S, hl, D), local.contiguous(), group=group)
    return buf.permute(1, 2, 0, 3, 4).reshape(B, S, world * hl, D)


def qk_shard(nk: int, nv: int, world: int, rank: int) -> tuple[int, int, list[int]]:
    """The QK heads [lo, hi) of ``rank`` and the V heads that read them under
    the tiled map h % NK (src/kernels.ts:1511), in local order: local V head j
    is global V head (j // NKl) * NK + lo + j % NKl, so local V head j reads
    local QK head j % NKl, the same tiled map over the local heads."""
    if nv % nk:
        raise ValueError(f"hachiue: {nv} V heads are not a multiple of {nk} QK heads")
    lo, hi = kv_head_range(nk, world, rank)
    return lo, hi, v_heads_of_qk_range(nk, nv, lo, hi)


def gather_v_head_shards(local: torch.Tensor, nk: int, group=None) -> torch.Tensor:
    """All-gather per-V-head outputs of a QK-head partition: local [..., NVl,
    D] (local V heads in :func:`qk_shard` order) -> [..., NV, D] in global V
    head order on every rank.  One collective moves [world][..., NVl, D];
    a local permute places head (c, rank, i) at c * NK + rank * NKl + i."""
    world = dist.get_world_size(group)
    *lead, nvl, D = local.shape
    nkl = nk // world
    m = nvl // nkl
    buf = torch.empty((world,) + tuple(local.shape), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(buf.view(world * local.shape[0], *local.shape[1:]), local.contiguous(),
                                group=group)
    buf = buf.view(world, *lead, m, nkl, D)
    nl = len(lead)
    perm = tuple(range(1, nl + 1)) + (nl + 1, 0, nl + 2, nl + 3)
    return buf.permute(perm).reshape(*lead, m * world * nkl, D)


def local_qkv_conv(qkv_conv: torch.Tensor, nk: int, nv: int, lo: int, hi: int, v_heads: list[int],
                   D: int = 128) -> torch.Tensor:
    """The rank's slice of a qkvConv row [..., 2*NK*D + NV*D] (q heads, k
    heads, v heads: src/wasm-backend.ts:1060-1062): its QK heads' q and k and
    its V heads' v, laid out as the same [q | k | v] row over the local heads."""
    q = qkv_conv[..., lo * D:hi * D]
    k = qkv_conv[..., (nk + lo) * D:(nk + hi) * D]
    vv = qkv_conv[..., 2 * nk * D:].unflatten(-1, (nv, D))[..., v_heads, :].flatten(-2)
    return torch.cat([q, k, vv], dim=-1).contiguous()


class HeadShardedSWA:
    """Sliding-window prefill (plamo3, configuration 3) sharded by KV head: the
    rank owns KV heads [lo, hi) of every sequence and the G = H / KV query
    heads that read them, runs hcu_swa_prefill on those, and the per-head
    outputs of all ranks are gathered by head.  No exchange inside the math."""

    def __init__(self, backend, H: int, KV: int, group=None):
        self.be, self.group = backend, group
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        self.kv_lo, self.kv_hi = kv_head_range(KV, world, rank)
        G = H // KV
        self.h_lo, self.h_hi = self.kv_lo * G, self.kv_hi * G

    def shard(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
        """This rank's contiguous q [B, T, H_local, D] and k, v [B, T, KV_local, D]."""
        return (q[:, :, self.h_lo:self.h_hi].contiguous(), k[:, :, self.kv_lo:self.kv_hi].contiguous(),
                v[:, :, self.kv_lo:self.kv_hi].contiguous())

    def __call__(self, q_local, k_local, v_local, out_local: torch.Tensor, window: int) -> torch.Tensor:
        self.be.swa_prefill(q_local, k_local, v_local, out_local, window)
        return gather_head_shards(out_local, self.group)


class QKHeadShardedGDN:
    """Gated DeltaNet (qwen35, configurations 4-5) sharded by QK head: the
    rank owns QK heads [lo, hi) and the V heads {h : h % NK in [lo, hi)}
    (:func:`qk_shard`), so each V head's state stays on one rank and no state
    crosses ranks; the per-V-head outputs are all-gathered."""

    def __init__(self, backend, NK: int, NV: int, group=None):
        self.be, self.group, self.NK, self.NV = backend, group, NK, NV
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        self.lo, self.hi, self.v_heads = qk_shard(NK, NV, world, rank)
        self.nkl, self.nvl = self.hi - self.lo, len(self.v_heads)

    def shard_prefill(self, q, k, v, g, beta):
        """Local q, k [B, T, NKl, D], v [B, T, NVl, D], g, beta [B, T, NVl]."""
        vh = torch.tensor(self.v_heads, device=v.device)
        return (q[:, :, self.lo:self.hi].contiguous(), k[:, :, self.lo:self.hi].contiguous(),
                v.index_select(2, vh).contiguous(), g.index_select(2, vh).contiguous(),
                beta.index_select(2, vh).contiguous())

    def shard_v_heads(self, x: torch.Tensor, dim: int) -> torch.Tensor:
        """Rows of x along ``dim`` for the local V heads (states, a, b, aNeg, dtBias)."""
        return x.index_select(dim, torch.tensor(self.v_heads, device=x.device)).contiguous()

    def prefill(self, q, k, v, g, beta, core_local, state_local, state_in_local=None) -> torch.Tensor:
        self.be.deltanet_chunked_prefill(q, k, v, g, beta, core_local, state_local, state_in=state_in_local)
        return gather_v_head_shards(core_local, self.NK, self.group)

    def decode(self, qkv_conv, a, b, a_neg, dt_bias, state_local, core_local) -> torch.Tensor:
        """One deltanet_decode step on the local heads (qkv_conv [B, S, convDim]
        global, sliced here; a, b [B, S, NV] global; a_neg, dt_bias [NV]
        global; state_local [B, NVl, D, D] updated in place)."""
        ql = local_qkv_conv(qkv_conv, self.NK, self.NV, self.lo, self.hi, self.v_heads)
        self.be.deltanet_decode(ql, self.shard_v_heads(a, 2), self.shard_v_heads(b, 2), self.shard_v_heads(a_neg, 0),
                                self.shard_v_heads(dt_bias, 0), state_local, core_local, state_local, self.nkl,
                                self.nvl)
        return gather_v_head_shards(core_local, self.NK, self.group)


class HeadShardedDecode:
    """Decode attention with this rank's KV heads: q [B, S, H, Dh] is sliced to
    the rank's query heads, attention runs on the rank's cache (which holds
    only its KV heads) and the outputs of all ranks are gathered by head."""

    def __init__(self, backend, H: int, KV: int, group=None):
        self.be = backend
        self.group = group
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        self.kv_lo, self.kv_hi = kv_head_range(KV, world, rank)
        G = H // KV
        self.h_lo, self.h_hi = self.kv_lo * G, self.kv_hi * G

    def __call__(self, q: torch.Tensor, cache, out_local: torch.Tensor, pos_base, **kw) -> torch.Tensor:
        ql = q[:, :, self.h_lo:self.h_hi].contiguous()
        self.be.attention(ql, cache, out_local, pos_base, **kw)
        return gather_head_shards(out_local, self.group)


class PeerLost(RuntimeError):
    """A rank stopped taking steps: raised on the host before the next
    collective, instead of blocking in it."""


class StepWatch:
    """Host-side failure detection between steps.  Every rank posts ``step`` to
    the process group's store after finishing a step's launches; before the
    next collective, ``check(step)`` waits (up to ``timeout_s``) for every
    peer's post of that step and raises :class:`PeerLost` naming the ranks
    that never posted.  A rank therefore leaves only between steps, with none
    of its kernels or collectives in flight, and its peers learn of it on the
    host rather than inside a collective."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 5.0, prefix: str = "hachiue/step"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix = timeout_s, prefix

    def _key(self, rank: int, step: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def post(self, step: int) -> None:
        self.store.set(self._key(self.rank, step), "1")

    def check(self, step: int) -> None:
        import time
        keys = [self._key(r, step) for r in range(self.world) if r != self.rank]
        deadline = time.monotonic() + self.timeout_s
        missing = keys
        while True:
            missing = [k for k in missing if not self.store.check([k])]
            if not missing or time.monotonic() > deadline:
                break
            time.sleep(0.01)
        if missing:
            lost = sorted(int(k.rsplit("/", 1)[1]) for k in missing)
            raise PeerLost(f"hachiue: rank(s) {lost} did not finish step {step} within {self.timeout_s} s")


class RankComm:
    """The path's all-gather through this library's C ABI under one process
    per GPU (torchrun): rank 0 makes an NCCL id (hcu_comm_unique_id), the
    process group broadcasts it, and every rank joins with its own device
    (hcu_comm_init_rank).  ``all_gather`` enqueues hcu_allgather on the
    device's current torch stream."""

    def __init__(self, device: int, group=None, max_ctas: int = 0):
        """``max_ctas`` > 0 caps the SMs the gathers occupy (small per-step
        gathers overlapping the next step's kernels); 0 is NCCL's choice."""
        import ctypes
        from . import _lib
        self._ct, self._lib, self.lib = ctypes, _lib, _lib.load()
        self.device = int(device)
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        uid = (ctypes.c_uint8 * _lib.COMM_ID_BYTES)()
        if self.rank == 0:
            _lib.check(self.lib.hcu_comm_unique_id(uid))
        t = torch.tensor(list(bytes(uid)), dtype=torch.uint8, device=f"cuda:{self.device}")
        dist.broadcast(t, src=0, group=group)
        uid = (ctypes.c_uint8 * _lib.COMM_ID_BYTES)(*t.cpu().tolist())
        h = ctypes.c_void_p()
        _lib.check(self.lib.hcu_comm_init_rank(self.world, self.rank, uid, self.device, int(max_ctas),
                                               ctypes.byref(h)))
        self._c = h

    def all_gather(self, send: torch.Tensor, recv: torch.Tensor) -> None:
        """recv[r] = rank r's send (recv: (world,) + send.shape, contiguous)."""
        ct, L = self._ct, self._lib
        nbytes = send.numel() * send.element_size()
        if (not send.is_contiguous() or not recv.is_contiguous() or recv.dtype != send.dtype
                or recv.numel() != self.world * send.numel()):
            raise L.HachiueError(L.HCU_EINVAL, "hachiue: all_gather buffers")
        vp = ct.c_void_p
        stream = torch.cuda.current_stream(self.device).cuda_stream
        L.check(self.lib.hcu_allgather(self._c, (vp * 1)(send.data_ptr()), (vp * 1)(recv.data_ptr()), nbytes,
                                       (vp * 1)(stream)))

    def close(self) -> None:
        if getattr(self, "_c", None):
            self.lib.hcu_comm_destroy(self._c)
            self._c = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DeviceComm:
    """One process driving several GPUs (as a Node host of the reference
    would): a communicator over ``devices`` (hcu_comm_create, ncclCommInitAll)
    and the path's all-gather (hcu_allgather) on each device's current torch
    stream.  Rank i is ``devices[i]``."""

    def __init__(self, devices):
        import ctypes
        from . import _lib
        self._ct, self.lib = ctypes, _lib.load()
        self.devices = [int(d) for d in devices]
        n = len(self.devices)
        h = ctypes.c_void_p()
        _lib.check(self.lib.hcu_comm_create(n, (ctypes.c_int * n)(*self.devices), ctypes.byref(h)))
        self._c = h

    def all_gather(self, sends: list[torch.Tensor], recvs: list[torch.Tensor]) -> None:
        """recvs[i][r] = sends[r] for every rank: sends[i] on devices[i],
        recvs[i] of shape (n,) + sends[i].shape, same dtype."""
        from . import _lib
        ct, n = self._ct, len(self.devices)
        if len(sends) != n or len(recvs) != n:
            raise _lib.HachiueError(_lib.HCU_EINVAL, f"hachiue: all_gather takes {n} send and receive buffers")
        nbytes = sends[0].numel() * sends[0].element_size()
        for i, (s, r) in enumerate(zip(sends, recvs)):
            if (s.device.index != self.devices[i] or r.device.index != self.devices[i] or not s.is_contiguous()
                    or not r.is_contiguous() or s.numel() * s.element_size() != nbytes
                    or r.numel() * r.element_size() != n * nbytes):
                raise _lib.HachiueError(_lib.HCU_EINVAL, f"hachiue: all_gather buffers of rank {i}")
        streams = [torch.cuda.current_stream(d).cuda_stream for d in self.devices]
        vp = ct.c_void_p
        _lib.check(self.lib.hcu_allgather(self._c, (vp * n)(*[s.data_ptr() for s in sends]),
                                          (vp * n)(*[r.data_ptr() for r in recvs]), nbytes, (vp * n)(*streams)))

    def close(self) -> None:
        if getattr(self, "_c", None):
            self.lib.hcu_comm_destroy(self._c)
            self._c = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

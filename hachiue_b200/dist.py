"""Multi-GPU partitioning of the attention hot path (one process per GPU).

The path shards by (sequence, KV / QK head): every unit is independent, so a
rank computes its units alone and the per-head outputs are joined with one
all-gather (NCCL over NVLink on GPUs, gloo on CPU).  The reference has no
multi-device path (one GPUDevice per engine, src/engine.ts:320).

Two partitions are provided:
  * by sequence (``seq_range``): rank r owns a contiguous range of sequences
    with all their heads (the benchmark's weak-scaling layout);
  * by KV head (``kv_head_range``): rank r owns a contiguous range of KV heads
    of every sequence and the G = H / KV query heads that read them, so each
    rank stores only its heads' cache.  GDN layers shard by QK head the same
    way: V heads h and h + NK read QK head h (tiled map), so a rank owning QK
    heads [a, b) owns V heads {h : h % NK in [a, b)}.
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

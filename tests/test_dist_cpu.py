"""Multi-rank partitioning on CPU: world_size-2 gloo process groups.

Each rank computes its shard with the oracle (the GPU kernels are covered by
the single-GPU parity tests) and the gathered result must equal the unsharded
computation exactly: the collective and the re-ordering move bits only."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hachiue_b200 import dist as hdist


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _attention_inputs(seed=0, B=4, S=2, H=8, KV=4, D=128, T=40):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, S, H, D), dtype=np.float32)
    k = rng.standard_normal((B * T, KV, D), dtype=np.float32)
    v = rng.standard_normal((B * T, KV, D), dtype=np.float32)
    pos = np.full(B, T - S, np.int32)
    off = (np.arange(B) * T).astype(np.int64)
    return q, k, v, pos, off


def _worker(rank, world, port, mode, result_q):
    import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v, pos, off = _attention_inputs()
        B, S, H, D = q.shape
        KV = k.shape[1]
        if mode == "heads":
            lo, hi = hdist.kv_head_range(KV, world, rank)
            G = H // KV
            ql = np.ascontiguousarray(q[:, :, lo * G:hi * G])
            kl = np.ascontiguousarray(k[:, lo:hi])
            vl = np.ascontiguousarray(v[:, lo:hi])
            local = oracle.attention_batch(ql, kl, vl, pos, off, 0, oracle.KV_F32, threads=1)
            full = hdist.gather_head_shards(torch.from_numpy(local))
        else:
            lo, hi = hdist.seq_range(B, world, rank)
            local = oracle.attention_batch(np.ascontiguousarray(q[lo:hi]), k, v, pos[lo:hi], off[lo:hi], 0,
                                           oracle.KV_F32, threads=1)
            full = hdist.gather_seq_shards(torch.from_numpy(local))
        if rank == 0:
            result_q.put(full.numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["heads", "sequences"])
def test_two_rank_shard_and_gather_matches_unsharded(mode):
    import oracle
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, result_q)) for r in range(2)]
    for p in procs:
        p.start()
    got = result_q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    q, k, v, pos, off = _attention_inputs()
    ref = oracle.attention_batch(q, k, v, pos, off, 0, oracle.KV_F32, threads=1)
    np.testing.assert_array_equal(got, ref)


def test_partitions_cover_everything():
    for world in (1, 2, 4, 8):
        seqs = [hdist.seq_range(64, world, r) for r in range(world)]
        assert seqs[0][0] == 0 and seqs[-1][1] == 64
        assert all(a[1] == b[0] for a, b in zip(seqs, seqs[1:]))
        heads = [hdist.kv_head_range(8, world, r) for r in range(world)]
        assert sum(hi - lo for lo, hi in heads) == 8
    # GDN: V heads h and h + NK follow their QK head h % NK to the same rank
    owned = [hdist.v_heads_of_qk_range(16, 32, lo, hi) for lo, hi in (hdist.kv_head_range(16, 4, r) for r in range(4))]
    assert sorted(sum(owned, [])) == list(range(32))
    assert all(((h + 16) in o) for o in owned for h in o if h < 16)
    with pytest.raises(ValueError):
        hdist.kv_head_range(8, 3, 0)


def _watch_worker(rank, world, port, fail_rank, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=30))
    dist.init_process_group("gloo", rank=rank, world_size=world, store=dist.PrefixStore("pg", store))
    watch = hdist.StepWatch(store, rank, world, timeout_s=2.0)
    out = torch.zeros(world)
    try:
        for step in range(4):
            if rank == fail_rank and step == 2:
                raise RuntimeError("rank failed between steps")  # leaves with nothing in flight
            watch.post(step)
            watch.check(step)  # every peer finished this step's work: the collective may start
            dist.all_gather_into_tensor(out, torch.full((1,), float(rank + step)))
        result_q.put((rank, "done", out.tolist()))
    except hdist.PeerLost as e:
        result_q.put((rank, "peer_lost", str(e)))
    except RuntimeError as e:
        result_q.put((rank, "raised", str(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_a_rank_that_leaves_is_reported_not_waited_for():
    """Host-side failure detection with 2 gloo ranks: rank 1 raises between
    steps; rank 0 learns of it from the store before its next all-gather and
    raises PeerLost naming rank 1 instead of blocking."""
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_watch_worker, args=(r, 2, port, 1, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict((r, (kind, msg)) for r, kind, msg in (q.get(timeout=120) for _ in range(2)))
    for p in ps:
        p.join(timeout=60)
    assert got[1][0] == "raised"
    assert got[0][0] == "peer_lost" and "[1]" in got[0][1] and "step 2" in got[0][1]


def test_step_watch_without_failures():
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_watch_worker, args=(r, 2, port, -1, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict((r, (kind, msg)) for r, kind, msg in (q.get(timeout=120) for _ in range(2)))
    for p in ps:
        p.join(timeout=60)
    assert got[0] == ("done", [3.0, 4.0]) and got[1] == ("done", [3.0, 4.0])


def _swa_inputs(seed=3, B=2, T=48, H=4, KV=2, D=128):
    rng = np.random.default_rng(seed)
    bf = lambda x: (torch.from_numpy(x).to(torch.bfloat16).float().numpy())  # noqa: E731
    return (bf(rng.standard_normal((B, T, H, D), dtype=np.float32)),
            bf(rng.standard_normal((B, T, KV, D), dtype=np.float32)),
            bf(rng.standard_normal((B, T, KV, D), dtype=np.float32)))


def _swa_ref(q, k, v, W):
    import oracle
    return np.stack([oracle.attention(np.ascontiguousarray(q[b]), np.ascontiguousarray(k[b]),
                                      np.ascontiguousarray(v[b]), 0, W) for b in range(q.shape[0])])


def _gdn_inputs(seed=4, B=2, T=12, NK=2, NV=4, D=128):
    rng = np.random.default_rng(seed)
    l2 = lambda x: (x / np.linalg.norm(x, axis=-1, keepdims=True)).astype(np.float32)  # noqa: E731
    q = l2(rng.standard_normal((B, T, NK, D), dtype=np.float32))
    k = l2(rng.standard_normal((B, T, NK, D), dtype=np.float32))
    v = rng.standard_normal((B, T, NV, D), dtype=np.float32)
    g = -np.abs(rng.standard_normal((B, T, NV), dtype=np.float32)) * 0.3
    beta = (1 / (1 + np.exp(-rng.standard_normal((B, T, NV))))).astype(np.float32)
    st = (0.02 * rng.standard_normal((B, NV, D, D))).astype(np.float32)
    return q, k, v, g, beta, st


def _gdn_ref(q, k, v, g, beta, st, NK, NV):
    """Token-serial recurrence per sequence (oracle) on [q | k | v] rows."""
    import oracle
    B, T = q.shape[:2]
    cores, states = [], []
    for b in range(B):
        qkv = np.concatenate([q[b].reshape(T, -1), k[b].reshape(T, -1), v[b].reshape(T, -1)], 1)
        gb = np.ascontiguousarray(np.stack([g[b], beta[b]]))
        c, s = oracle.deltanet_recur(np.ascontiguousarray(qkv), gb, st[b], NK, NV, True)
        cores.append(c)
        states.append(s)
    return np.stack(cores), np.stack(states)


def _exec_worker(rank, world, port, mode, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        if mode == "swa":
            q, k, v = _swa_inputs()
            ex = hdist.HeadShardedSWA(None, q.shape[2], k.shape[2])
            ql, kl, vl = (x.numpy() for x in ex.shard(*(torch.from_numpy(x) for x in (q, k, v))))
            full = hdist.gather_head_shards(torch.from_numpy(_swa_ref(ql, kl, vl, 16)))
            result = full.numpy()
        else:
            q, k, v, g, beta, st = _gdn_inputs()
            NK, NV = q.shape[2], v.shape[2]
            ex = hdist.QKHeadShardedGDN(None, NK, NV)
            tq = [torch.from_numpy(x) for x in (q, k, v, g, beta)]
            st_l = ex.shard_v_heads(torch.from_numpy(st), 1).numpy()
            if mode == "gdn_prefill":
                ql, kl, vl, gl, bl = (x.numpy() for x in ex.shard_prefill(*tq))
            else:  # decode: the qkvConv row of each token sliced by local_qkv_conv
                B, T, D = q.shape[0], q.shape[1], q.shape[3]
                qkv = torch.cat([tq[0].flatten(2), tq[1].flatten(2), tq[2].flatten(2)], -1)
                ql_row = hdist.local_qkv_conv(qkv, NK, NV, ex.lo, ex.hi, ex.v_heads, D).numpy()
                ql = ql_row[..., :ex.nkl * D].reshape(B, T, ex.nkl, D)
                kl = ql_row[..., ex.nkl * D:2 * ex.nkl * D].reshape(B, T, ex.nkl, D)
                vl = ql_row[..., 2 * ex.nkl * D:].reshape(B, T, ex.nvl, D)
                gl, bl = ex.shard_v_heads(tq[3], 2).numpy(), ex.shard_v_heads(tq[4], 2).numpy()
            core_l, st_out_l = _gdn_ref(ql, kl, vl, gl, bl, st_l, ex.nkl, ex.nvl)
            full = hdist.gather_v_head_shards(torch.from_numpy(core_l), NK)
            states = [torch.empty_like(torch.from_numpy(st_out_l)) for _ in range(world)]
            dist.all_gather(states, torch.from_numpy(st_out_l))
            owned = [hdist.qk_shard(NK, NV, world, r)[2] for r in range(world)]
            st_full = np.zeros_like(st)
            for r in range(world):
                st_full[:, owned[r]] = states[r].numpy()
            result = (full.numpy(), st_full)
        if rank == 0:
            result_q.put(result)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["swa", "gdn_prefill", "gdn_decode"])
def test_two_rank_swa_and_gdn_executors_match_unsharded(mode):
    """HeadShardedSWA (by KV head) and QKHeadShardedGDN (by QK head, V heads
    h and h + NK together): each rank slices with the executor, computes its
    heads with the oracle, and the gathered outputs (and, for GDN, the states
    that stay on their rank) equal the unsharded computation bit for bit."""
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exec_worker, args=(r, 2, port, mode, result_q)) for r in range(2)]
    for p in procs:
        p.start()
    got = result_q.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    if mode == "swa":
        q, k, v = _swa_inputs()
        np.testing.assert_array_equal(got, _swa_ref(q, k, v, 16))
    else:
        q, k, v, g, beta, st = _gdn_inputs()
        core, states = _gdn_ref(q, k, v, g, beta, st, q.shape[2], v.shape[2])
        np.testing.assert_array_equal(got[0], core)
        np.testing.assert_array_equal(got[1], states)

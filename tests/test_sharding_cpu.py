"""Session sharding across ranks, session transfer and failure detection on
CPU ranks (gloo, world size 2).  Failures are made on the host: a rank that
never sends, a rank that stops its heartbeat."""
import os
import queue
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from infercache_b200.sharding import (PeerMonitor, SessionTransferError, ShardMap, max_over_ranks, recv_session,
                                      send_session, session_state_like, shard_sessions)


def _cfg():
    from infercache_b200 import CacheConfig
    return CacheConfig(num_layers=3, num_kv_heads=2, head_dim=128, sink_size=4, recent_size=8, important_size=20,
                       dtype=torch.float16)


@pytest.mark.parametrize("mode", ["contiguous", "round_robin"])
@pytest.mark.parametrize("n,world", [(16, 1), (16, 2), (17, 4), (3, 8), (64, 8)])
def test_shards_partition_sessions(n, world, mode):
    seen = []
    for r in range(world):
        ids = shard_sessions(n, world, r, mode)
        seen += ids
        assert len(ids) in (n // world, n // world + 1)
    assert sorted(seen) == list(range(n))
    m = ShardMap(n, world, mode)
    for g in range(n):
        r, i = m.owner(g)
        assert m.local_sessions(r)[i] == g


def test_shard_map_move():
    m = ShardMap(8, 2)
    m.move(1, 1, 4)
    assert m.owner(1) == (1, 4)
    assert 1 not in m.local_sessions(0) and m.local_sessions(1)[4] == 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, scenario, q):
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    try:
        from datetime import timedelta
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=20))
        if scenario == "transfer":
            cfg = _cfg()
            like = session_state_like(cfg, "cpu")
            assert max_over_ranks(float(rank + 1)) == float(world)
            if rank == 0:
                g = torch.Generator().manual_seed(7)
                st = {k: (torch.randn(v.shape, generator=g).to(v.dtype) if v.is_floating_point()
                          else torch.randint(0, 100, v.shape, generator=g).to(v.dtype)) for k, v in like.items()}
                send_session(st, 1, timeout_s=10)
                q.put(("sent", {k: v.numpy().tobytes() for k, v in st.items()}))
            else:
                got = recv_session(like, 0, timeout_s=10)
                q.put(("got", {k: v.numpy().tobytes() for k, v in got.items()}))
            dist.barrier()
        elif scenario == "silent_peer":
            cfg = _cfg()
            like = session_state_like(cfg, "cpu")
            if rank == 0:
                t0 = time.monotonic()
                try:
                    recv_session(like, 1, timeout_s=2.0)
                    q.put(("no-error", 0.0))
                except SessionTransferError:
                    q.put(("error", time.monotonic() - t0))
            else:
                time.sleep(4.0)  # never sends
                q.put(("idle", 0.0))
        elif scenario == "heartbeat":
            store = dist.distributed_c10d._get_default_store()
            mon = PeerMonitor(store, rank, world)
            mon.beat(0)
            dist.barrier()
            if rank == 1:
                q.put(("stopped", 0))  # rank 1 beats once and stops
                time.sleep(3.0)
            else:
                fresh = mon.stale_peers(max_age_s=5.0)
                time.sleep(1.5)
                mon.beat(1)
                stale = mon.stale_peers(max_age_s=1.0)
                q.put(("seen", (fresh, stale, mon.last(1)[1])))
        dist.destroy_process_group()
    except Exception as e:  # report to the parent instead of hanging it
        q.put(("exception", repr(e)))


def _run(scenario, world=2, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = []
    deadline = time.monotonic() + timeout
    while len(out) < world and time.monotonic() < deadline:
        try:
            out.append(q.get(timeout=1.0))
        except queue.Empty:
            pass
    for p in procs:
        p.join(timeout=max(1.0, deadline - time.monotonic()))
        if p.is_alive():
            p.kill()
    assert len(out) == world, f"workers reported {out}"
    assert not [o for o in out if o[0] == "exception"], out
    return dict((o[0], o[1]) for o in out)


def test_session_transfer_gloo():
    res = _run("transfer")
    assert set(res["sent"]) == set(res["got"])
    for k in res["sent"]:
        assert res["sent"][k] == res["got"][k], k


def test_silent_peer_times_out_instead_of_hanging():
    res = _run("silent_peer")
    assert "error" in res, res
    assert 1.5 <= res["error"] < 10.0


def test_heartbeat_detects_stopped_rank():
    res = _run("heartbeat")
    fresh, stale, last_step = res["seen"]
    assert fresh == [] and stale == [1] and last_step == 0

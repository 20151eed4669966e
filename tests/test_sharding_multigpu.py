"""Moving a session between GPUs over NCCL (needs two GPUs; skipped with one).

Rank 0 and rank 1 build the same two-session batch and decode the same steps;
rank 0 then sends its session 1 to rank 1 (``rebalance_session``), which
imports it into its session 0 row (``receive_rebalanced``).  Rank 1 then
decodes both rows with identical inputs: the imported row must reproduce its
native copy bit for bit, outputs and metadata alike."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs")]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _batch(dev):
    from infercache_b200 import CacheConfig, SessionBatch
    cfg = CacheConfig(num_layers=3, num_kv_heads=2, head_dim=128, sink_size=4, recent_size=16, important_size=40,
                      dtype=torch.float16, decay=0.99)
    b = SessionBatch(cfg, 2, dev)
    g = torch.Generator().manual_seed(21)
    for s in range(2):
        T = 150 + 20 * s
        pkv = tuple((torch.randn(1, 2, T, 128, generator=g).half().to(dev),
                     torch.randn(1, 2, T, 128, generator=g).half().to(dev)) for _ in range(3))
        b.load_prompt(s, pkv, torch.rand(T, generator=g).to(dev))
    return b, g


def _worker(rank, port, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        from datetime import timedelta
        import torch.distributed as dist
        from infercache_b200.sharding import rebalance_session, receive_rebalanced
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                                timeout=timedelta(seconds=60), device_id=dev)
        b, g = _batch(dev)
        qs = torch.randn(8, 3, 2, 16, 128, generator=g).half()
        ks = torch.randn(8, 3, 2, 2, 128, generator=g).half()
        vs = torch.randn(8, 3, 2, 2, 128, generator=g).half()
        for t in range(3):
            b.step(qs[t].to(dev), ks[t].to(dev), vs[t].to(dev), [400 + t, 500 + t])
        torch.cuda.synchronize()
        if rank == 0:
            rebalance_session(b, 1, 1, timeout_s=30)
            torch.cuda.synchronize()
            ok = bool((b.positions[1] == -1).all()) and not bool(b.occupied[1].any())
            q.put(("sender", ok, ""))
        else:
            receive_rebalanced(b, 0, 0, timeout_s=30)
            torch.cuda.synchronize()
            same = True
            why = ""
            for t in range(3, 8):
                qq, kk, vv = qs[t].clone(), ks[t].clone(), vs[t].clone()
                qq[:, 0], kk[:, 0], vv[:, 0] = qq[:, 1], kk[:, 1], vv[:, 1]  # row 0 now mirrors row 1
                o = b.step(qq.to(dev), kk.to(dev), vv.to(dev), [500 + t, 500 + t])
                if not torch.equal(o[:, 0], o[:, 1]):
                    same, why = False, f"output differs at step {t}"
                    break
            for key in ("positions", "importance", "occupied", "ctrl", "counters"):
                tns = getattr(b, key)
                if same and not torch.equal(tns[0], tns[1]):
                    same, why = False, f"{key} differs"
            b.check_device_status()
            q.put(("receiver", same, why))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which fails the test
        q.put(("error", False, f"rank {rank}: {type(e).__name__}: {e}"))


def test_session_moves_between_gpus_bit_exact():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = []
    try:
        for _ in range(2):
            results.append(q.get(timeout=240))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for who, ok, why in results:
        assert ok, (who, why)
    assert sorted(r[0] for r in results) == ["receiver", "sender"], results

"""The reference's decode path on the host cores: one process per core, each
owning a share of the sessions and running the oracle decode protocol.

TEST INFRASTRUCTURE / CPU BASELINE ONLY (see ``oracle/__init__.py``).  Used
by ``bench.py`` for its ``cpu_baseline`` leg and its ``--impl reference`` arm.
Processes are started with ``spawn`` so they never inherit a CUDA context.
"""
from __future__ import annotations

import multiprocessing as mp
import os
import time
from typing import List


def _worker(conn, sessions: List[int], spec: dict, seed: int, threads: int):
    os.environ["OMP_NUM_THREADS"] = str(threads)
    os.environ["OPENBLAS_NUM_THREADS"] = str(threads)
    os.environ["MKL_NUM_THREADS"] = str(threads)
    import numpy as np
    from oracle.hier_cache import OracleCache, TierGeometry, decode_step

    L, Hq, Hkv, D, T = spec["layers"], spec["hq"], spec["hkv"], spec["d"], spec["prompt"]
    kv = np.float16 if spec["dtype"] == "float16" else np.float32
    geo = TierGeometry(L, Hkv, D, spec["sink"], spec["recent"], spec["important"])
    caches = []
    ring = 4
    inputs = []
    for s in sessions:
        rng = np.random.default_rng(seed * 100003 + s)
        pk = rng.standard_normal((L, Hkv, T, D), dtype=np.float32).astype(kv)
        pv = rng.standard_normal((L, Hkv, T, D), dtype=np.float32).astype(kv)
        u = rng.random(T, dtype=np.float32)
        c = OracleCache(geo, kv)
        c.load_from_hf_output(pk, pv, (u / u.sum()).astype(np.float32))
        caches.append(c)
        inputs.append([(rng.standard_normal((L, Hq, D), dtype=np.float32).astype(kv).astype(np.float32),
                        rng.standard_normal((L, Hkv, D), dtype=np.float32).astype(kv),
                        rng.standard_normal((L, Hkv, D), dtype=np.float32).astype(kv)) for _ in range(ring)])
    conn.send("ready")
    pos = T
    while True:
        n = conn.recv()
        if n is None:
            break
        t0 = time.perf_counter()
        for i in range(n):
            for c, inp in zip(caches, inputs):
                q, k, v = inp[(pos + i) % ring]
                decode_step(c, q, k, v, pos + i, spec["decay"])
        pos += n
        conn.send(time.perf_counter() - t0)
    conn.close()


class CpuDecodeFleet:
    """Sessions split over `workers` single-threaded processes."""

    def __init__(self, spec: dict, workers: int = 0, seed: int = 0):
        n = spec["sessions"]
        workers = workers or min(os.cpu_count() or 1, n)
        self.workers = workers
        self.spec = spec
        ctx = mp.get_context("spawn")
        self.conns, self.procs = [], []
        # Children re-import the parent's main module before running _worker,
        # so the one-thread-per-process limits must already be in the
        # environment they inherit.
        keys = ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")
        saved = {k: os.environ.get(k) for k in keys}
        for k in keys:
            os.environ[k] = "1"
        try:
            for w in range(workers):
                mine = list(range(w, n, workers))
                a, b = ctx.Pipe()
                p = ctx.Process(target=_worker, args=(b, mine, spec, seed, 1), daemon=True)
                p.start()
                self.conns.append(a)
                self.procs.append(p)
        finally:
            for k, v in saved.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = v
        for c in self.conns:
            assert c.recv() == "ready"

    def run(self, steps: int) -> float:
        """Decode `steps` tokens in every session; returns the slowest worker's seconds."""
        for c in self.conns:
            c.send(int(steps))
        return max(c.recv() for c in self.conns)

    def close(self):
        for c in self.conns:
            try:
                c.send(None)
            except Exception:
                pass
        for p in self.procs:
            p.join(timeout=10)
            if p.is_alive():
                p.terminate()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

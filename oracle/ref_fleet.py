"""The reference's own decode path on the host cores, as the CPU baseline.

CPU BASELINE INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): used by
``bench.py``'s ``cpu_baseline`` leg and its ``--impl reference`` arm, never by
the package.

Each worker process imports the unmodified reference package ``inference``
(``baseline/_ref``, installed by ``oracle/ref_install.py``, or the tree named
by ``$INFERCACHE_REF``), owns a share of the sessions -- one
``inference.hierarchical_cache.HierarchicalKVCache`` each, primed through its
``load_from_hf_output`` -- and runs the decode protocol the parity harness
uses, through the reference's public API: per step ``to_hf_past_key_values``
(the slots in position order, hierarchical_cache.py:297-351), GQA attention
in torch float32 with scale head_dim ** -0.5 over those slots plus the new
token, the received mass summed over the query heads of each KV head, the
importance decayed, then ``push(k, v, position, attn_weights=mass)``
(:241-294).  Processes are started with ``spawn`` so they never inherit a
CUDA context.
"""
from __future__ import annotations

import multiprocessing as mp
import os
import sys
import tempfile
import time
from pathlib import Path
from typing import List, Optional

ROOT = Path(__file__).resolve().parents[1]


def reference_dir() -> Optional[str]:
    """A directory from which ``import inference`` loads the reference, or None."""
    installed = ROOT / "baseline" / "_ref"
    if (installed / "inference" / "hierarchical_cache.py").exists():
        return str(installed)
    src = os.environ.get("INFERCACHE_REF")
    if src and (Path(src) / "hierarchical_cache.py").exists():
        d = tempfile.mkdtemp(prefix="icref_")
        os.symlink(src, os.path.join(d, "inference"))
        return d
    return None


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _worker(conn, sessions: List[int], spec: dict, seed: int, threads: int, ref_dir: str):
    for k in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[k] = str(threads)
    import torch
    torch.set_num_threads(threads)
    sys.path.insert(0, ref_dir)
    from inference.cache_safety import normalise_kv
    from inference.hierarchical_cache import CacheConfig, HierarchicalKVCache

    L, Hq, Hkv, D = spec["layers"], spec["hq"], spec["hkv"], spec["d"]
    dt = torch.float16 if spec["dtype"] == "float16" else torch.float32
    G = Hq // Hkv
    scale = D ** -0.5
    cfg = CacheConfig(num_layers=L, num_kv_heads=Hkv, head_dim=D, sink_size=spec["sink"],
                      recent_size=spec["recent"], important_size=spec["important"], decay=spec["decay"], dtype=dt)
    caches, positions, inputs = [], [], []
    ring = 4
    t0 = time.perf_counter()
    with torch.no_grad():
        for s in sessions:
            g = torch.Generator().manual_seed(seed * 100003 + s)
            T = spec["prompt_lens"][s] if "prompt_lens" in spec else spec["prompt"]
            pkv = tuple((torch.randn(1, Hkv, T, D, generator=g).to(dt), torch.randn(1, Hkv, T, D, generator=g).to(dt))
                        for _ in range(L))
            u = torch.rand(T, generator=g)
            c = HierarchicalKVCache(cfg)
            c.load_from_hf_output(pkv, u / u.sum())
            caches.append(c)
            positions.append(T)
            inputs.append([(torch.randn(L, Hq, D, generator=g).to(dt), torch.randn(L, Hkv, D, generator=g).to(dt),
                            torch.randn(L, Hkv, D, generator=g).to(dt)) for _ in range(ring)])
    conn.send(("ready", time.perf_counter() - t0))

    def step(cache, q, k, v, position):
        past = normalise_kv(cache.to_hf_past_key_values())
        masses = []
        for l in range(L):
            K = torch.cat([past[l][0][0].float(), k[l][:, None, :].float()], 1)
            V = torch.cat([past[l][1][0].float(), v[l][:, None, :].float()], 1)
            p = (torch.einsum("hgd,hfd->hgf", q[l].float().view(Hkv, G, D), K) * scale).softmax(-1)
            torch.einsum("hgf,hfd->hgd", p, V)  # the step's attention output
            masses.append(p.sum(1))
        w = torch.stack(masses)[:, :, None, :]
        cache.importance[cache.occupied] *= spec["decay"]
        cache.push(k[:, :, None, :], v[:, :, None, :], position=position, attn_weights=w)

    n_done = 0
    while True:
        n = conn.recv()
        if n is None:
            break
        t0 = time.perf_counter()
        with torch.no_grad():
            for i in range(n):
                for j, c in enumerate(caches):
                    q, k, v = inputs[j][(n_done + i) % ring]
                    step(c, q, k, v, positions[j])
                    positions[j] += 1
        n_done += n
        conn.send(time.perf_counter() - t0)
    conn.close()


class RefDecodeFleet:
    """The sessions of `spec` spread over worker processes running the
    reference's cache; `threads` torch threads per process."""

    def __init__(self, spec: dict, ref_dir: str, workers: int = 0, seed: int = 0):
        n = spec["sessions"]
        cores = os.cpu_count() or 1
        workers = workers or max(1, min(cores, n))
        self.workers = workers
        self.threads = max(1, cores // workers)
        self.cores = min(cores, workers * self.threads)
        ctx = mp.get_context("spawn")
        self.conns, self.procs = [], []
        keys = ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")
        saved = {k: os.environ.get(k) for k in keys}
        for k in keys:
            os.environ[k] = str(self.threads)
        try:
            for w in range(workers):
                a, b = ctx.Pipe()
                p = ctx.Process(target=_worker, args=(b, list(range(w, n, workers)), spec, seed, self.threads, ref_dir),
                                daemon=True)
                p.start()
                self.conns.append(a)
                self.procs.append(p)
        finally:
            for k, v in saved.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = v
        self.prime_s = 0.0
        for c in self.conns:
            tag, secs = c.recv()
            assert tag == "ready"
            self.prime_s = max(self.prime_s, secs)

    def run(self, steps: int) -> float:
        """Decode `steps` tokens in every session; the slowest worker's seconds."""
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


def measure(spec: dict, budget_s: float, max_steps: int, ref_dir: str, seed: int = 0) -> dict:
    """session-tokens/s of the reference's decode path on this host: one
    warm-up step, then as many steps as fit `budget_s` (at most max_steps)."""
    with RefDecodeFleet(spec, ref_dir, seed=seed) as fleet:
        t1 = fleet.run(1)
        steps = max(1, min(max_steps, int(budget_s / max(t1, 1e-3))))
        t = fleet.run(steps)
        return {"value": spec["sessions"] * steps / t, "steps": steps, "seconds": t, "workers": fleet.workers,
                "threads_per_worker": fleet.threads, "cores": fleet.cores, "host_cores": os.cpu_count(),
                "cpu_model": cpu_model(), "prime_s": fleet.prime_s}

"""The GPU graph cache against fixtures made by the reference GraphKVCache:
after pushing every token (one launch per push) or a bulk load_from_summary
(one routing launch + one copy pass), every region's positions, the cluster
fills, scores, centroid counts and centroids (bit-identical), the K/V rows
of every layer and head, and retrieve()'s selection, order and rows."""
import numpy as np
import pytest
import torch

import specs

pytestmark = pytest.mark.gpu


def make_cache(name):
    from infercache_b200 import ClusterConfig, GraphKVCache
    sp = specs.GRAPH[name]
    cfg = ClusterConfig(num_layers=sp["L"], num_kv_heads=sp["H"], head_dim=sp["D"], n_clusters=sp["n_clusters"],
                        cluster_capacity=sp["cap"], sim_threshold=sp["threshold"], sink_size=sp["sink"],
                        recent_size=sp["recent"], dtype=torch.float16)
    return GraphKVCache(cfg, "cuda:0")


def fill_cache(name):
    sp = specs.GRAPH[name]
    k, v, scores, qs = specs.graph_inputs(name)
    c = make_cache(name)
    if name == "push":
        for t in range(sp["T"]):
            c.push(k[:, :, t:t + 1].cuda(), v[:, :, t:t + 1].cuda(), t, float(scores[t]))
    else:
        c.load_from_summary(tuple((k[li][None].cuda(), v[li][None].cuda()) for li in range(sp["L"])), scores.cuda())
    torch.cuda.synchronize()
    return c, k, v, qs


@pytest.mark.parametrize("name", list(specs.GRAPH))
def test_graph_cache_matches_reference(golden, name):
    ref = golden(f"graph_{name}")
    sp = specs.GRAPH[name]
    c, k, v, qs = fill_cache(name)
    SK, R, C, cap = sp["sink"], sp["recent"], sp["n_clusters"], sp["cap"]
    pos = c.positions.cpu().numpy()
    assert np.array_equal(pos[:SK], ref["sink_pos"])
    assert np.array_equal(pos[SK:SK + R], ref["rec_pos"])
    assert np.array_equal(pos[SK + R:].reshape(C, cap), ref["cl_pos"])
    ctrl = c.ctrl.cpu().numpy()
    assert (ctrl[0], ctrl[1], ctrl[2]) == (int(ref["sink_fill"]), int(ref["rec_ptr"]), int(ref["rec_fill"]))
    assert np.array_equal(c.cl_fill.cpu().numpy(), ref["cl_fill"])
    assert np.array_equal(c.c_count.cpu().numpy(), ref["c_count"])
    assert np.array_equal(c.scores.cpu().numpy().reshape(C, cap), ref["cl_score"])
    assert np.array_equal(c.centroid.cpu().numpy(), ref["centroid"])
    # every occupied slot holds its token's rows in every layer and head
    K, V = c.K.cpu(), c.V.cpu()
    occ = np.nonzero(pos >= 0)[0]
    assert torch.equal(K[:, :, occ], k[:, :, pos[occ]]) and torch.equal(V[:, :, occ], v[:, :, pos[occ]])
    empty = np.nonzero(pos < 0)[0]
    assert not K[:, :, empty].any() and not V[:, :, empty].any()
    for qi, (thr, top) in enumerate(specs.GRAPH_QUERIES):
        pkv, sel = c.retrieve(qs[qi].cuda(), threshold=thr, top_n_clusters=top)
        assert np.array_equal(sel.numpy(), ref["q_selected"][qi]), qi
        a, b = ref["q_offsets"][qi], ref["q_offsets"][qi + 1]
        rpos = ref["q_positions"][a:b]
        for li in range(sp["L"]):
            assert torch.equal(pkv[li][0][0].cpu(), k[li][:, rpos]), (qi, li)
            assert torch.equal(pkv[li][1][0].cpu(), v[li][:, rpos]), (qi, li)


def test_graph_cache_push_after_load_and_reset():
    """Single pushes on top of a bulk load agree with pushing every token
    one by one; reset empties every region."""
    name = "load"
    sp = specs.GRAPH[name]
    k, v, scores, _ = specs.graph_inputs(name)
    a = make_cache(name)
    b = make_cache(name)
    T0 = 150
    a.load_from_summary(tuple((k[li][None, :, :T0].cuda(), v[li][None, :, :T0].cuda()) for li in range(sp["L"])),
                        scores[:T0].cuda())
    for t in range(T0):
        b.push(k[:, :, t:t + 1].cuda(), v[:, :, t:t + 1].cuda(), t, float(scores[t]))
    for t in range(T0, sp["T"]):
        a.push(k[:, :, t:t + 1].cuda(), v[:, :, t:t + 1].cuda(), t, float(scores[t]))
        b.push(k[:, :, t:t + 1].cuda(), v[:, :, t:t + 1].cuda(), t, float(scores[t]))
    for key in ("positions", "scores", "centroid", "cl_fill", "c_count", "ctrl", "K", "V"):
        assert torch.equal(getattr(a, key), getattr(b, key)), key
    assert a.active_cluster_count == sp["n_clusters"]
    s = a.cluster_summary()
    assert [x["fill"] for x in s] == a.cl_fill.tolist()
    a.reset()
    assert a.active_cluster_count == 0 and bool((a.positions == -1).all()) and not a.K.any()
    pkv, sel = a.retrieve(torch.randn(sp["H"], sp["D"]))
    assert pkv is None and sel.sum() == 1


GEOMETRIES = [
    # (L, H, n_clusters, cap, sink, recent, threshold, T)
    (1, 1, 1, 1, 0, 1, 0.3, 40),      # one cluster of one slot, ring of one, no sinks
    (2, 2, 3, 2, 4, 2, 0.0, 60),      # threshold 0: any positive similarity routes
    (2, 1, 5, 4, 2, 3, 0.99, 80),     # threshold near 1: mostly first-empty / least-filled
    (1, 2, 8, 3, 4, 5, 0.3, 3),       # fewer tokens than sinks
    (3, 2, 2, 16, 1, 7, 0.5, 150),
]


@pytest.mark.parametrize("geo", GEOMETRIES)
def test_graph_random_geometries_vs_oracle(geo):
    """Edge geometries against the oracle, pushed one token at a time and
    loaded in bulk.  Inputs whose routing would come within 5e-5 of a tie or
    the threshold are redrawn (the decision would then depend on how a cosine
    is summed)."""
    from infercache_b200 import ClusterConfig, GraphKVCache
    from oracle.graph_cache import ClusterGeometry, GraphOracle
    L, H, C, cap, sink, recent, thr, T = geo
    D = 128
    for seed in range(50):
        g = torch.Generator().manual_seed(1000 + seed)
        dirs = torch.randn(4, D, generator=g)
        dirs = dirs / dirs.norm(dim=1, keepdim=True)
        k = torch.randn(L, H, T, D, generator=g)
        k[0, 0] = dirs[torch.randint(0, 4, (T,), generator=g)] * 3.0 + torch.randn(T, D, generator=g)
        k, v = k.half(), torch.randn(L, H, T, D, generator=g).half()
        scores = torch.rand(T, generator=g)
        o = GraphOracle(ClusterGeometry(L, H, D, C, cap, thr, sink, recent))
        kn, vn = k.float().numpy(), v.float().numpy()
        margins = []
        for t in range(T):
            if not (t < sink and o.sink_fill < sink) and o.rec_pos[o.rec_ptr] >= 0:
                margins.append(o.route_margin(o.rec_k[0, 0, o.rec_ptr].astype(np.float32)))
            o.push(kn[:, :, t], vn[:, :, t], t, float(scores[t]))
        if not margins or min(margins) > 5e-5:
            break
    cfg = ClusterConfig(num_layers=L, num_kv_heads=H, head_dim=D, n_clusters=C, cluster_capacity=cap,
                        sim_threshold=thr, sink_size=sink, recent_size=recent)
    one = GraphKVCache(cfg, "cuda:0")
    bulk = GraphKVCache(cfg, "cuda:0")
    for t in range(T):
        one.push(k[:, :, t:t + 1].cuda(), v[:, :, t:t + 1].cuda(), t, float(scores[t]))
    bulk.load_from_summary(tuple((k[li][None].cuda(), v[li][None].cuda()) for li in range(L)), scores.cuda())
    want = np.concatenate([o.sink_pos, o.rec_pos, o.cl_pos.reshape(-1)])
    for c in (one, bulk):
        assert np.array_equal(c.positions.cpu().numpy(), want)
        assert np.array_equal(c.centroid.cpu().numpy(), o.centroid)
        assert np.array_equal(c.scores.cpu().numpy(), o.cl_score.reshape(-1))
        assert np.array_equal(c.cl_fill.cpu().numpy(), o.cl_fill)
        pos = c.positions.cpu().numpy()
        occ = np.nonzero(pos >= 0)[0]
        assert torch.equal(c.K.cpu()[:, :, occ], k[:, :, pos[occ]])
    for key in ("positions", "scores", "centroid", "cl_fill", "c_count", "ctrl", "K", "V"):
        assert torch.equal(getattr(one, key), getattr(bulk, key)), key


def test_graph_push_of_nothing_and_bad_shapes():
    from infercache_b200 import ClusterConfig, GraphKVCache
    cfg = ClusterConfig(num_layers=2, num_kv_heads=2, head_dim=128, n_clusters=2, cluster_capacity=2, recent_size=2)
    c = GraphKVCache(cfg, "cuda:0")
    c._push_many(torch.zeros(2, 2, 0, 128), torch.zeros(2, 2, 0, 128), torch.zeros(0, dtype=torch.int64), None,
                 reset=False)
    assert bool((c.positions == -1).all())
    with pytest.raises(ValueError):
        c.push(torch.zeros(3, 2, 1, 128), torch.zeros(3, 2, 1, 128), 0)

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

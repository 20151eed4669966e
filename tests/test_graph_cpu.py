"""The graph-cache oracle against fixtures made by the reference GraphKVCache
(graph_cache.py:218-495): cluster routing, in-cluster eviction, centroids,
the ring and sinks, and retrieve()'s cluster selection and token order."""
import numpy as np
import pytest

import specs
from oracle.graph_cache import ClusterGeometry, GraphOracle


def geometry(name):
    sp = specs.GRAPH[name]
    return ClusterGeometry(num_layers=sp["L"], num_kv_heads=sp["H"], head_dim=sp["D"], n_clusters=sp["n_clusters"],
                           cluster_capacity=sp["cap"], sim_threshold=sp["threshold"], sink_size=sp["sink"],
                           recent_size=sp["recent"])


def run_oracle(name):
    sp = specs.GRAPH[name]
    k, v, scores, _ = specs.graph_inputs(name)
    k, v, scores = k.float().numpy(), v.float().numpy(), scores.numpy()
    o = GraphOracle(geometry(name), np.float16)
    if name == "push":
        for t in range(sp["T"]):
            o.push(k[:, :, t], v[:, :, t], t, float(scores[t]))
    else:
        o.load_from_summary(k, v, scores)
    return o


def check_state(o, ref):
    assert np.array_equal(o.sink_pos, ref["sink_pos"]) and o.sink_fill == int(ref["sink_fill"])
    assert np.array_equal(o.rec_pos, ref["rec_pos"])
    assert o.rec_ptr == int(ref["rec_ptr"]) and o.rec_fill == int(ref["rec_fill"])
    assert np.array_equal(o.cl_fill, ref["cl_fill"])
    assert np.array_equal(o.cl_pos, ref["cl_pos"])
    assert np.array_equal(o.cl_score, ref["cl_score"])
    assert np.array_equal(o.c_count, ref["c_count"])
    # centroid updates are elementwise float32 operations: bit-identical
    assert np.array_equal(o.centroid, ref["centroid"])


@pytest.mark.parametrize("name", list(specs.GRAPH))
def test_graph_oracle_matches_reference(golden, name):
    ref = golden(f"graph_{name}")
    o = run_oracle(name)
    check_state(o, ref)
    assert np.array_equal(np.array(o.decisions, np.int64).reshape(-1, 3), ref["decisions"])
    _, _, _, qs = specs.graph_inputs(name)
    for qi, (thr, top) in enumerate(specs.GRAPH_QUERIES):
        sel = o.select(qs[qi].numpy(), thr, top)
        assert np.array_equal(sel, ref["q_selected"][qi]), qi
        pos = o.retrieve_positions(sel)
        a, b = ref["q_offsets"][qi], ref["q_offsets"][qi + 1]
        assert np.array_equal(pos, ref["q_positions"][a:b]), qi


def test_graph_oracle_retrieve_returns_the_tokens_in_order():
    """retrieve()'s K rows are the input rows of the positions it lists."""
    name = "push"
    o = run_oracle(name)
    k, v, _, qs = specs.graph_inputs(name)
    ks, vs, sel = o.retrieve(qs[0].numpy())
    pos = o.retrieve_positions(sel)
    kin = k.numpy()
    for li in range(len(ks)):
        assert np.array_equal(ks[li], kin[li][:, pos]), li

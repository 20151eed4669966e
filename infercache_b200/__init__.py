"""infercache_b200: the fixed-budget KV-cache decode hot path of infercache,
built for the B200 (sm_100a).

Public API (the reference's names):
    CacheConfig, CacheStats, HierarchicalKVCache      hierarchical_cache
    SessionBatch                                       batched sessions + hot-path verbs
    PAGE_SIZE, PagedCacheConfig, PagePool, KVAllocator,
    PagedSessionView, MultiSessionCache                paged_cache
    summary_score, attention_mass, SummaryScores       summary (kernel C)
    TwoPassConfig, SummaryResult, TwoPassEngine        two_pass
    gather_cache_kv, scatter_importance, topk_min_slot,
    compact_sdp_attention, GPUImportanceTracker        cache_ops (the triton_ops names)
    ClusterConfig, GraphKVCache, MultiClusterCache     graph_cache (cluster-routed L2)

Importing the package needs no GPU; constructing a cache does.
"""
from .hierarchical_cache import CacheConfig, CacheStats, HierarchicalKVCache, HostStepper, SessionBatch  # noqa: F401
from .paged_cache import (PAGE_SIZE, KVAllocator, MultiSessionCache, PagedCacheConfig,  # noqa: F401
                          PagedSessionView, PagePool)
from .summary import SummaryScores, attention_mass, summary_score  # noqa: F401
from .two_pass import SummaryResult, TwoPassConfig, TwoPassEngine  # noqa: F401
from .cache_ops import (GPUImportanceTracker, compact_sdp_attention, gather_cache_kv,  # noqa: F401
                        scatter_importance, topk_min_slot)
from .graph_cache import ClusterConfig, GraphKVCache, MultiClusterCache  # noqa: F401

__version__ = "0.1.0"

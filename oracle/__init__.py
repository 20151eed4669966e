"""CPU oracle for the infercache decode hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in ``infercache_b200`` imports this
package: only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
legs of ``bench.py`` use it, and only to check results or as the timed CPU
baseline, never as a product code path.  ``ref_fleet`` and ``ref_install``
run and install the reference itself for that baseline.

The oracle is a numpy restatement of the reference implementation
(the ``inference`` package of ravirajb/infercache):

* ``hier_cache``  -- ``HierarchicalKVCache`` (hierarchical_cache.py:109-477)
  and the per-step decode protocol that drives it (attention, received mass
  summed over the query heads of each KV group, decay, push).
* ``summary``     -- ``_attention_mass`` (two_pass.py:104-137), computed in
  query chunks so that long prompts never materialise T x T at once, plus
  the tier fill done by ``load_from_hf_output``.
* ``paged``       -- ``PagePool`` / ``KVAllocator`` / ``PagedSessionView``
  (paged_cache.py:99-454) with a logical clock in place of
  ``time.monotonic`` so that LRU order is reproducible.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference itself
on seeded inputs and commits small fixtures; ``tests/test_oracle_golden.py``
checks this oracle against them.
"""

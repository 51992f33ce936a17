"""CPU oracle for the sparse-attention hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy (fp64 where the contract needs it), the
algorithms of xiaolong-li1/SparseAttnFunctions that the CUDA library
replaces.  It is the checker, never the thing measured or shipped: only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it.  The product path
(``sparseattnfunctions_b200``) never imports it and has no CPU fallback.

Modules
  selection  -- block mean-pool, pooled scores, top-k + forced text blocks
                (mask_related.py:40-81, block_sparse_attn_kernel.py:31-39,
                SparseGen_Plus.py:12-84).
  attention  -- block-sparse attention as the reference's kron-mask path
                (block_sparse_attn_kernel.py:326-334) and the query-chunked
                torch CPU masked SDPA used as the timed CPU baseline.
  tome       -- ToMe bipartite soft matching, merge and unmerge
                (utils/merge_unmerge.py:34-154).
  ulysses    -- the pack / unpack layout of the sequence <-> head
                all-to-all (no reference counterpart: single-GPU reference).

Pinning: ``tests/golden/make_golden.py`` imports the reference from its
source tree (only where that tree exists, i.e. not on the GPU box) and
records its outputs; ``tests/test_oracle_golden.py`` checks this package
against those fixtures.
"""

"""CPU oracle for the tree-verification hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
directory.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline /
reference leg of ``bench.py`` may import it, and there only as the checker (or
as the timed CPU restatement of the reference's own CPU path), never as the
thing measured for the GPU path.

Every function restates the reference algorithm (DiffSpec, package
``diffspec``) in plain numpy / torch-on-CPU code and cites the reference
``file:line`` it follows.  The restatements are pinned against golden vectors
produced by running the reference itself (``tests/golden/make_golden.py``),
checked by ``tests/test_oracle_golden.py``.

Modules
-------
attention   prefix / tree-masked attention + LSE merge (fp32 torch on CPU)
acceptance  greedy and sample-and-match acceptance, path trace, contiguous
            KV compaction (numpy, integer work bit-exact)
paged       page-table copy-on-write bookkeeping and paged compaction
arena       chunk-arena differential update
bundles     branching-ancestor bundle grouping
rope        rotary embedding of q / k and the KV-cache append (numpy, bit-exact
            emulation of the reference's bf16 / fp16 / fp32 element-wise ops)
tree        final draft-tree build: node order, parent positions, ancestor
            mask and the root-prepended verify bitmask
retrieval   draft-side chunk scores, top-k, interval union and row gather
"""

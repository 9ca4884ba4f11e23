"""CPU oracle for Anvil's int8 graph semantics: TEST INFRASTRUCTURE, never the product.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this package, and only as the checker
(or, for bench.py --impl reference, as the timed CPU stand-in for the reference interpreter). The anvil package and
libanvil_cuda.so never import, link or call it.

    oracle.semantics   checked-int32 numpy restatement of anvil/semantics.py and of the missing xf.golden base ops
    oracle.interp      whole-tensor graph interpreter (anvil/interp/graph.py:43-92)
    oracle.loops       scalar loop-nest restatements (graph_to_tensor / vortexv codegen) for cross-checks

Parity pins: known-answer vectors from the reference's own tests, agreement of the independent in-repo
restatements, and the reference's own semantics.py / quantize.py executed over this base (tests/golden). The
xf.golden outputs themselves are not available here, so value-level parity of the base ops is pinned only through
those restatements.
"""

"""CPU oracle for pageserve's decode-step hot path — TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's own algorithm (Rakshit-gen/pageserve,
engine/paged_attention.py, engine/quantization.py, engine/model.py,
engine/tensor_parallel.py); every function cites the reference file:line it
follows. Parity is pinned: ``tests/test_oracle_golden.py`` checks this
restatement against golden vectors produced by running the unmodified
reference (``tests/golden/make_golden.py``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
legs may import this package, and only as the checker / the timed CPU
baseline. The product package ``pageserve_b200`` never imports it and has no
CPU fallback.
"""

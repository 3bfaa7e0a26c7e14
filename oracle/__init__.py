"""CPU oracle for the compressed Butterfly attention path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy and plain Python integers, the algorithm of the
reference project's compressed attention path so that the CUDA implementation in
``butterfly_b200`` can be checked against it.  It is imported only by ``tests/``,
``__graft_entry__.smoke()`` (as the checker) and ``bench.py``'s CPU-baseline leg.
The product path (``butterfly_b200``) never imports it and has no CPU fallback.

Parity pinning: ``tests/golden/`` holds vectors produced by running the reference's
own PyTorch functions (``bna/torch/attention_wayfinder_permute.py``) in a container
where the reference source was importable (generator: ``tests/golden/make_golden.py``).
``tests/test_oracle_golden.py`` checks this oracle against them, so the oracle is
"parity pinned" for selection tables, block means, prefill and active (decode) outputs.
The two-pool cache restatement (``oracle.cache``) follows the reference's MLX cache,
which cannot run here; it is pinned indirectly: decoding from the restated cache must
equal the reference's torch ``butterfly_compressed_attention_active`` outputs.

Modules:
  topology   — butterfly width / stage / partner rules and block-neighbour rows
  compressed — selection tables, block means, prefill and active attention (+ LSE)
  cache      — two-pool (tail + summary) cache and decode-from-cache streams
"""

"""CPU oracle for nanoengine's speculative step -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import this package, and only as the checker or the timed CPU
baseline. The product path (the package ``inference-engine-from-scratch_b200``) never imports it
and has no CPU fallback.

What it restates, each function citing the reference (``ak7270090/inference-engine-from-scratch``,
paths relative to ``nanoengine/src/nanoengine``):

* ``qwen3``      -- the Qwen3 forward over a paged KV pool (``models/qwen3.py``,
                    ``models/attention_context.py``, ``models/int8_quantization.py``,
                    ``engine/memory/kv_cache_pool.py``).
* ``ngram``      -- ``NgramProposer.propose`` (``engine/speculative/proposers.py:44-57``).
* ``verify``     -- ``verify_proposal`` / ``compute_token_probabilities`` / ``apply_top_p``
                    (``engine/speculative/verifier.py:21-60``, ``engine/sampling.py:21-51``) with the
                    random draws taken from an injected uniform stream.
* ``philox``     -- Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11, "Parallel random numbers:
                    as easy as 1, 2, 3"), the per-request uniform stream of sampled acceptance.
* ``speculative``-- the serial speculative generator with the paged FIFO block allocator
                    (``engine/speculative/speculative_generator.py:42-90``,
                    ``engine/memory/paged_allocator.py``, ``engine/memory/block_allocator.py``).

Parity pinning: ``tests/golden/make_golden.py`` imports the real reference (Python, CPU) in the
build container and records its outputs as fixtures under ``tests/golden/``; the not-gpu tests
check this oracle against those fixtures, so the oracle is pinned to the reference itself.
"""

"""CPU oracle for the paged-KV attention path.  TEST INFRASTRUCTURE ONLY.

This package is a numpy restatement of InferKernelLab's reference algorithms for
the paged KV cache and paged attention (``src/inferkernellab/cache.py``,
``src/inferkernellab/attention.py`` and the rotary helpers of
``src/inferkernellab/hf_benchmark.py`` in the reference project).  It is the checker
that the CUDA path is compared against, never a code path of the product:

* only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
  ``--impl reference`` legs of ``bench.py`` may import it;
* the product package ``inferkernellab_b200`` must never import it (a test
  scans the package sources to enforce this).

Parity is pinned: ``tests/golden/make_golden.py`` imports the reference project
itself and records its outputs on seeded inputs into ``tests/golden/*.npz``;
``tests/test_oracle_golden.py`` checks this restatement against those fixtures.
"""

from .paged_ref import (  # noqa: F401
    bf16_bits_to_f32,
    f32_to_bf16_bits,
    to_f32,
    slot_mapping,
    write_slots,
    rotary_embed,
    read_tokens,
    dense_decode_attention,
    paged_decode_attention,
    paged_prefill_attention,
    paged_prefill_attention_packed,
)

"""CPU oracle for the Ulysses context-parallel attention path (TEST INFRASTRUCTURE ONLY).

This package restates, in plain torch-on-CPU arithmetic, what cozy-runtime computes on the path
the product library accelerates. It is the checker, never the thing measured or shipped: only
`tests/`, `__graft_entry__.smoke()` and the `cpu_baseline` / `--impl reference` legs of
`bench.py` may import it. The product path (`cozy_runtime_b200`) never imports it and fails loudly
when its CUDA library is missing.

Pinning: every function here is checked against golden vectors produced by running the
reference's own code (`tests/golden/make_golden.py`, fixtures `tests/golden/*.npz`) in
`tests/test_oracle_golden.py`.
"""

from oracle.ulysses_oracle import (  # noqa: F401
    attention_fp32,
    exchange,
    exchange_group,
    exchange_narrow,
    fp8_attention_law,
    hadamard_matrix,
    head_norm_rope,
    heads_padded,
    narrow_law,
    narrow_law_back,
    owned_heads,
    quantise_e4m3_per_head,
    quantise_fp8_blocks,
    rotate_bf16,
    sequence_rows,
    turned,
)

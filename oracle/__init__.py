"""CPU oracle for the pre-norm causal Transformer forward.

TEST INFRASTRUCTURE ONLY. Nothing in the shipped package imports this
directory: only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` may use it, and only as the checker (or as the timed CPU
baseline), never as the thing measured on the GPU.

Parity is pinned: ``tests/golden/make_golden.py`` ran the reference's own
``BaselineTransformer`` (torch_transformer_benchmark.py:204-317) and
``compare_outputs`` (torch_transformer_benchmark.py:1237-1304) in the build
container and committed the outputs; ``tests/test_oracle.py`` checks this
restatement against them.
"""

from .baseline import (  # noqa: F401
    AccuracyResult,
    BaselineSelfAttention,
    BaselineTransformer,
    BaselineTransformerBlock,
    TransformerConfig,
    compare_outputs,
    generate_random_case,
    make_baseline,
    state_dict_checksum,
)

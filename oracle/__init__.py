"""CPU oracle for the single transformer-layer forward (test infrastructure only).

This package restates, on the CPU, the arithmetic of the reference's PyTorch
layer (dalberrt/COBRA-GPU-Kernel, ``torch_transformer_benchmark.py``) so that
the CUDA path can be checked against it. It is the checker, never the product:
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import it. The product path (``cobra-gpu-kernel_b200``)
never imports this package and has no CPU fallback.

Parity is pinned: ``tests/golden/make_golden.py`` ran the reference's own
``BaselineSelfAttention`` and ``nn.LayerNorm`` classes (imported from the
reference source tree) and stored inputs/outputs as fixtures; the oracle
reproduces those outputs bit for bit (see ``tests/test_oracle.py``).
"""

from .ref_layer import (  # noqa: F401
    TransformerConfig,
    ReferenceSelfAttention,
    ReferenceLayer,
    ReferenceBlock,
    ReferenceTransformer,
    build_reference_layer,
    build_reference_transformer,
    generate_random_case,
    streamed_layer_rows_fp64,
    streamed_attention_rows_fp64,
    streamed_keys,
    streamed_ctx_rows,
    streamed_output_rows,
)
from .compare import AccuracyResult, compare_outputs  # noqa: F401

"""Drop-in for the reference's compiled op module ``server.paged_attention_cpp``.

``paged_attention(query, keys, values, block_table, length, block_size, groups,
scaling)`` keeps the positional signature of csrc/paged_attention.cpp:76-79 and
its error behaviour (RuntimeError on malformed input), so it can be injected
where the reference injects its op: ``PagedKVPool(..., attention=paged_attention)``
(src/server/torch_model.py:116-119) or ``PagedBackend(..., attention=...)``
(src/server/backend/paged.py:29-32).  It takes CUDA tensors, or the host
tensors of the reference's own pool, which it stages on the current CUDA device
(the arithmetic always runs in this package's kernels).
"""

from .ops import paged_attention

__all__ = ["paged_attention"]

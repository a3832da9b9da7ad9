"""B200-native paged-attention path of the BatchStream inference engine.

The package holds the sm_100a kernels and their C ABI (``csrc/``, built into
``libbatchstream_b200.so`` by ``build.py``) and the host side that mirrors the
reference interface: the drop-in op (``paged_attention_cuda``), batched ops
(``ops``), the block allocator with device-resident tables
(``block_allocator``), the paged model and backend that call them
(``torch_model``, ``backend``) and the one-replica-per-GPU runner
(``replicas``).
"""

__version__ = "0.1.0"

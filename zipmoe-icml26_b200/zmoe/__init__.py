"""Host-side Python of the B200 ZipMoE expert hot path.

``zmoe.ops`` wraps the C ABI of libzmoe.so for torch tensors; ``zmoe.synthetic``
builds seeded workloads.  Importing ``zmoe.ops`` requires the built library.
"""

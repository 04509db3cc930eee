"""B200-native (sm_100a) kernels behind the torch.ops.vlak operators.

Drop-in for the reference package of the same name: ``kernels.softmax`` and
``kernels.attention`` keep the reference's Python API, operator schemas and
fake (meta) implementations, and call hand-written sm_100a CUDA kernels
through the C ABI declared in ``include/vlak_b200.h``.
"""

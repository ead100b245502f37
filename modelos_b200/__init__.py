"""B200 (sm_100a) product-key-memory hot path.

Drop-in replacements for the reference's ``pkm`` and ``fwpkm`` packages
(``modelos_b200.pkm.memory.HashingMemory``,
``modelos_b200.fwpkm.fwpkm.FastWeightProductKeyMemory``) on hand-written CUDA
kernels exposed through the C ABI in ``include/pkm_b200.h``.
"""

__version__ = "0.1.0"

"""B200-native model forward of sys1rust: the ModernBERT encoder plus the typed-decision head.

The compute path is the C-ABI library ``libs1c.so`` (hand-written sm_100a CUDA, built from
``sys1rust_b200/csrc``). This package holds the host side around it: the reference's batch
formats and packing (``batch``), checkpoint config (``config``) and seeded weights
(``weights``), and ``backend.CudaBackend``, the mirror of ``laya_core::Backend``.
"""
__all__ = ["batch", "config", "weights"]

"""mentat_b200: B200-native entropy-gated prefix-tree decode path.

Drop-in replacements for the reference's ``core/paged_kv_cache.py``
(:class:`PagedKVCacheManager`) and ``adapters/attention_backend.py``
(:mod:`mentat_b200.attention_backend`), plus the fused entropy gate
(:mod:`mentat_b200.gate`).  Kernels live in libmentat_b200.so (C ABI:
``include/mentat_b200.h``), built by ``python -m mentat_b200.build``.
"""

from .paged_kv_cache import PagedKV, PagedKVCacheManager, SequenceState  # noqa: F401

__all__ = ["PagedKVCacheManager", "PagedKV", "SequenceState"]

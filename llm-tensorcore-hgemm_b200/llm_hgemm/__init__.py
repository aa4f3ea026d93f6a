"""B200 (sm_100a) FP16 HGEMM for LLM linear layers.

Drop-in for the reference package of the same name
(reference llm_hgemm/__init__.py:3-5): ``hgemm`` and ``available_providers``.
Importing it loads the native extension and fails loudly when it is missing.
"""

from .ops import available_providers, hgemm

__all__ = ["available_providers", "hgemm"]

"""evspark_b200 — B200-native (sm_100a) block-verification hot path for EvSpark.

Same public surface as the reference ``evspark`` package for that path:
``EvSpark.load/generate/generate_native/close``, ``GenerateResult``, ``clean_prompt``,
``ids_to_text``; the block driver / state slicing / loop under ``evspark_b200.specdec.block``;
the verifier and sampling transform under ``evspark_b200.specdec``.  All compute goes through
``libevspark_sm100.so`` (C ABI in include/evspark_sm100.h).
"""

from evspark_b200.api import DEFAULT_CKPT, EvSpark, GenerateResult, clean_prompt, ids_to_text

__version__ = "0.1.0"

__all__ = ["DEFAULT_CKPT", "EvSpark", "GenerateResult", "clean_prompt", "ids_to_text", "__version__"]

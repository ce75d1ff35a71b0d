"""Speculative decoding on the device: verifier, sampling transform, block path."""

from evspark_b200.specdec.transforms import apply_transform
from evspark_b200.specdec.verifier import VerifyResult, sample_categorical, verify_round, verify_round_greedy

__all__ = ["VerifyResult", "apply_transform", "sample_categorical", "verify_round", "verify_round_greedy"]

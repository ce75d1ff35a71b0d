"""Minimal stand-in for the absent ``vortex`` runtime (TEST INFRASTRUCTURE ONLY).

Exposes the oracle StripedHyena2 (``oracle.model``) under the names EvSpark's
block path imports (evspark/specdec/block/chunk.py:43-44, driver.py:90), so the
reference's own code can run unmodified on CPU to produce golden fixtures.
"""

"""Checkpoint publication contract, legacy import and upcycling loaders."""
from mimir_b200.ckpt.contract import MANIFEST, publish, resolve, restore_rng, rng_state, validate

__all__ = ["MANIFEST", "publish", "resolve", "restore_rng", "rng_state", "validate"]

"""Speculative verification on the native folded pass (drop-in for ``actfold.speculative``'s engine)."""

from actfold_b200.speculative.block_decoding import (BlockDecoder, BlockDecodingConfig, BlockDecodingResult,
                                                     SyntheticDraft)
from actfold_b200.speculative.verification_engine import ActFoldVerificationEngine, Branch, VerificationResult

__all__ = ["ActFoldVerificationEngine", "Branch", "VerificationResult", "BlockDecoder", "BlockDecodingConfig",
           "BlockDecodingResult", "SyntheticDraft"]

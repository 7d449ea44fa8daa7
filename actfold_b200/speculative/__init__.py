"""Speculative verification on the native folded pass (drop-in for ``actfold.speculative``'s engine)."""

from actfold_b200.speculative.block_decoding import (BlockDecoder, BlockDecodingConfig, BlockDecodingResult,
                                                     SyntheticDraft)
from actfold_b200.speculative.acceptance_policy import (AcceptancePolicy, GreedyAcceptancePolicy,
                                                         ThresholdAcceptancePolicy)
from actfold_b200.speculative.branch_tree import BranchNode, BranchTree
from actfold_b200.speculative.folded_generation import FoldedGenerationResult, folded_generate
from actfold_b200.speculative.verification_engine import ActFoldVerificationEngine, Branch, VerificationResult

__all__ = ["ActFoldVerificationEngine", "Branch", "VerificationResult", "BlockDecoder", "BlockDecodingConfig",
           "BlockDecodingResult", "SyntheticDraft", "AcceptancePolicy", "GreedyAcceptancePolicy",
           "ThresholdAcceptancePolicy", "BranchNode", "BranchTree", "FoldedGenerationResult", "folded_generate"]

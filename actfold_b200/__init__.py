"""ActFold-B200: Branch Folding verification on B200 (sm_100a) CUDA kernels.

The Python API mirrors ActFold's (``actfold.core``, ``actfold.profiler``,
``actfold.speculative``) under ``actfold_b200.*``; every tensor operation on
the folding path runs in ``libactfold_b200.so`` (see ``actfold_b200._lib``).
"""

__version__ = "0.1.0"

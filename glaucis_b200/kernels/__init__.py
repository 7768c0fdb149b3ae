"""Kernel templates with the entry points of the Glaucis evaluator's templates
(KE/examples/kernels/gmm_fp8_blockwise.py, KE/examples/kernels/chunk_gla.py),
backed by the sm_100a kernels.  The evaluator exec()s a template's text, so
each file is self-contained."""

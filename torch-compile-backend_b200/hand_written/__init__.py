"""Standalone kernels with the reference's hand_written/ API, backed by the
sm_100a library instead of Triton."""

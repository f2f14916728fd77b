"""Module-name shim for callers of the reference's src/triton_kernel.py.  The name is the
reference's; the implementation is CUDA (gpusparse), not Triton."""
from gpusparse.scoring import triton_fused_score, triton_wand_score  # noqa: F401

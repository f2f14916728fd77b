"""Module-name shim for callers of the reference's src/triton_kernel_chunked.py (CUDA
implementation)."""
from gpusparse.scoring import build_chunk_boundaries, triton_chunked_score  # noqa: F401

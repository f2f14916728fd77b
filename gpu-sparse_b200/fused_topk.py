"""Module-name shim for callers of the reference's src/fused_topk.py (CUDA implementation)."""
from gpusparse.scoring import compacted_topk, triton_chunked_score_fused  # noqa: F401

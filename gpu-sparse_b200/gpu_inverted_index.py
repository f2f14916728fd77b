"""Module-name shim for callers of the reference's src/gpu_inverted_index.py."""
from gpusparse.index import (BLOCK_SIZE, GPUInvertedIndex, build_gpu_inverted_index,  # noqa: F401
                             build_gpu_inverted_index_from_sparse, generate_synthetic_splade_data,
                             index_memory_stats)

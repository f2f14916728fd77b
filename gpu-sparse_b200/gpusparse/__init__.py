"""gpusparse: exact learned-sparse (SPLADE) retrieval on B200 (sm_100a).

Drop-in for GPUSparse's scoring path: the reference's names (GPUInvertedIndex, the index
builders, triton_fused_score, triton_chunked_score, build_chunk_boundaries,
compacted_topk, triton_chunked_score_fused) backed by hand-written CUDA kernels in
libgpusparse.so, reached through the C ABI of include/gpusparse.h.  No Triton, no CPU
fallback: every entry point raises if the library or a CUDA device is missing.

Beyond the reference: streamed index builds (build_streamed, build_from_host_csr),
index persistence (save_index, load_index), a captured fixed-shape scorer
(CapturedScorer), and, in gpusparse.distributed, doc-range sharding over the GPUs of a
node.
"""
from .index import (BLOCK_DOCS, BLOCK_SIZE, VOCAB_SIZE, GPUInvertedIndex,  # noqa: F401
                    build_from_csr_tensors, build_from_host_csr, build_gpu_index_from_csr,
                    build_gpu_inverted_index, build_streamed,
                    build_gpu_inverted_index_from_sparse, build_index_from_scipy,
                    dequantized_weights, generate_synthetic_splade_data, index_memory_stats,
                    load_index, quantize_, save_index)
from .scoring import (CapturedScorer, build_chunk_boundaries, compacted_topk, merge_topk,  # noqa: F401
                      score_topk, triton_chunked_score, triton_chunked_score_fused,
                      triton_fused_score, triton_wand_score)

__version__ = "0.1.0"

"""rsllm_b200 -- B200-native (sm_100a) KV-cache hot path for rsLLM.

FP8 E4M3FN quantize-on-append into a paged pool, paged gather + dequant to
bf16, indexer top-k selection, sparse gather + dequant, and page moves for
copy-on-write and compaction, compressor emission (aggregate, RMSNorm, RoPE,
quantize-on-append) and MLA decode attention, as hand-written CUDA behind the C
ABI in ``include/rsllm_kv_cuda.h``.  ``rsllm_b200.kvcache`` and
``rsllm_b200.compressor`` are the host API.
"""
from .kvcache import *  # noqa: F401,F403
from .kvcache import __all__  # noqa: F401
from .compressor import (CompressorBank, IndexerCompressorBank, compress_expf, compress_expf_table_size,  # noqa: F401
                         compress_rope_table)

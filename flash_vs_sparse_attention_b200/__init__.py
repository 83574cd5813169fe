"""B200-native (sm_100a) two-stage content-adaptive block-sparse attention.

Drop-in variant for the reference's block indexer
(``attention/block_indexer_triton.py``, ``attention/block_indexer.py``):

    from flash_vs_sparse_attention_b200 import block_indexer_b200
    O = block_indexer_b200.attention(Q, K, V, causal=True, block_size=64, top_k=16)

The arithmetic lives in ``libbsattn.so`` (C ABI: ``include/bsattn.h``); see
``sharding`` for the (batch x head) multi-GPU split.
"""

from . import block_indexer_b200, flops  # noqa: F401
from .block_indexer_b200 import attention, select_blocks, pool_k, fine  # noqa: F401
from .block_indexer_b200 import attention_trainable, backward  # noqa: F401

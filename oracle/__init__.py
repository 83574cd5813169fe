"""CPU oracle for the two-stage block-sparse attention path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
directory; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline /
reference arm of ``bench.py`` use it, and only as the checker or as the timed
CPU baseline.

Parity is pinned: ``tests/golden/`` holds vectors produced by running the
reference's own ``attention/block_indexer.py`` (script
``tests/golden/make_golden.py``), and ``tests/test_oracle.py`` checks this
restatement against every one of them.
"""

from .block_indexer_np import (  # noqa: F401
    attention,
    attention_unit,
    coarse_scores,
    select_blocks,
    fine_stage,
    pool_k,
    canonical_rows,
    index_parity,
)
from .decode_np import decode_rows, pool_k_prefix  # noqa: F401
from .qblock_np import qblock_attention_unit, qblock_scores  # noqa: F401
from .inputs import CONFIGS, unit_inputs, make_inputs, round_to_bf16  # noqa: F401

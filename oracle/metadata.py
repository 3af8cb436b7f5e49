"""numpy/Python restatement of the engine's per-step slot mapping — TEST
INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

``slot_mapping`` restates the host loop of ModelRunner.prepare_model_input
(nanovllm/engine/model_runner.py:414-425): for every sequence with a block
table, the new tokens occupy positions [num_cached_tokens, num_context_tokens)
and are written block by block; cacheless sequences contribute -1 per query
token (model_runner.py:409-413).
"""

from __future__ import annotations


def slot_mapping(block_tables, num_cached_tokens, num_context_tokens, block_size):
    """block_tables: per-sequence lists of physical block ids (may be empty)."""
    slots = []
    for table, cached, context in zip(block_tables, num_cached_tokens, num_context_tokens):
        if not table:
            slots.extend([-1] * (context - cached))
            continue
        first_block = cached // block_size
        for i in range(first_block, len(table)):
            if i == first_block:
                start = table[i] * block_size + cached % block_size
            else:
                start = table[i] * block_size
            if i == len(table) - 1:
                end = (table[i] * block_size + context % block_size
                       if context % block_size else (table[i] + 1) * block_size)
            else:
                end = (table[i] + 1) * block_size
            slots.extend(range(start, end))
    return slots


def block_tables(block_lists):
    """ModelRunner.prepare_block_tables (nanovllm/engine/model_runner.py:354-358):
    every sequence's block list padded with -1 to the longest one."""
    width = max(len(b) for b in block_lists)
    return [list(b) + [-1] * (width - len(b)) for b in block_lists]

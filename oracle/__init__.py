"""CPU oracle of the paged-KV attention path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this package, and only as the checker / the timed CPU
baseline. The product path (``my_vllm_b200``) never calls it.
"""

from .paged_attention import (  # noqa: F401
    bf16_bits_to_f32,
    block_tables_to_csr,
    f32_to_bf16_bits,
    kv_append,
    paged_attention,
    paged_attention_from_tables,
    to_f32,
)
from .metadata import block_tables, slot_mapping  # noqa: F401,E402
from .rope import cos_sin_cache, rms_norm, rope_neox  # noqa: F401,E402
from . import fp8  # noqa: F401,E402

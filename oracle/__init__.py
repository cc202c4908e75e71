"""CPU oracle of mini-vLLM's paged KV write, gather, decode and RoPE — test infrastructure.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may use this package, and only as the checker or the timed CPU
baseline.  The product (``mini_vllm_b200`` and ``libmvb200.so``) never imports
it.  See ``oracle.py`` for the functions and the reference lines they restate.
"""

from .oracle import (  # noqa: F401
    ORACLE_BLOCK_ID,
    ORACLE_KV_LEN,
    ORACLE_OK,
    ORACLE_TABLE_SHORT,
    build_oracle,
    cache_write,
    cache_write_numpy,
    decode,
    decode_numpy,
    gather,
    from_float32,
    max_threads,
    rope_numpy,
    round_to_dtype,
    step_metadata_numpy,
    to_float32,
)

"""inferd_b200 -- sm_100a-native decode hot path with the reference's Python interface.

Modules mirror the reference's (likhith-v1/inferd) call surface:

    inferd_b200.paged_attn            <- core/paged_attn.py
    inferd_b200.paged_cache           <- core/paged_cache.py
    inferd_b200.paged_attn_interface  <- core/paged_attn_interface.py
    inferd_b200.fp8_linear            <- bench/model_loader.py FP8 weight-only linear
    inferd_b200.sampling              <- core/spec_decode.py nucleus_probs / sample_from
    inferd_b200.sharded               sequence shards per GPU, outputs gathered over NCCL

All kernels live in libinferd_sm100a.so (C ABI: include/inferd_b200.h), built with
`python -m inferd_b200.build`.  There is no CPU fallback.
"""

from .paged_attn import (  # noqa: F401
    dense_attention,
    gather_paged_kv,
    paged_attention,
    paged_attention_batched,
    paged_attention_reference,
    paged_decode,
    paged_verify,
    reserve_sms,
    sdpa_reference,
)
from .paged_cache import (  # noqa: F401
    BlockAllocator,
    PagedHybridCache,
    PagedKVCache,
    SequencePageTable,
)

__version__ = "0.1.0"

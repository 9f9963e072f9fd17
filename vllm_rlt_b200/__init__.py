"""B200-native (sm_100a) attention hot path for looped (recurrent-depth)
transformers, drop-in for vllm-rlt's attention backend operator API.

Public surface (mirrors vllm_rlt/kernels):
  * ``B200PagedAttention`` -- backend object (``__call__`` decode,
    ``.prefill`` packed chunked prefill, ``.info``, ``.generation``);
  * ``b200_paged_attention`` / ``paged_attention`` -- decode call;
  * ``paged_prefill`` -- packed prefill call;
  * ``plan_shared_prefix`` / ``paged_attention_shared`` -- decode that reads
    pages shared by several rows (prefix caching) once per group;
  * ``write_kv`` / ``finalize`` -- KV page write and LAST-EXITED exit copy;
  * ``metadata``, ``gather``, ``scatter``, ``stage_prefill``,
    ``expand_prefill`` -- routing and prefill-metadata kernels;
  * ``install`` -- put the backend into a reference KV cache manager.

Importing the package does not initialise CUDA; the shared library is loaded
on first use and its absence raises (there is no fallback path).
"""

from .backend import install  # noqa: F401
from .kernels.cache_ops import finalize, write_kv  # noqa: F401
from .kernels.paged_attention import (  # noqa: F401
    B200PagedAttention,
    b200_paged_attention,
    decode_bytes,
    paged_attention,
    paged_attention_lse,
)
from .kernels.paged_prefill import paged_prefill  # noqa: F401
from .kernels.shared_prefix import (  # noqa: F401
    find_shared_prefixes,
    paged_attention_shared,
    plan_shared_prefix,
)
from .kernels.prefill_metadata import expand_prefill, stage_prefill  # noqa: F401
from .kernels.routing import gather, metadata, scatter  # noqa: F401

"""Install the B200 backend into a reference KV cache manager.

The reference selects its attention backend from a fixed set of strings
(vllm_rlt/core/kv_cache_manager.py:109-131) and calls whatever object sits in
``cache.attention`` -- from ``_attend_prepared`` (:559-586) and from the
CUDA-graph proxy (vllm_rlt/worker/cuda_graph.py:21-29), which reads the
attribute at call time. Its own tests swap that attribute the same way
(tests/test_flash_attention.py:128). The KV page write has no hook: it is an
index-put inside ``_write_prepared`` (:519-534) and inside the graph proxy's
``_write_prepared`` (cuda_graph.py:16-19); ``install`` rebinds both to the
sm_100a write kernel while keeping the reference's validation and written-
prefix bookkeeping unchanged.
"""

from __future__ import annotations

from .kernels.cache_ops import write_kv
from .kernels.paged_attention import B200PagedAttention


def install(cache, *, graph_proxy_class=None, replace_write=True):
    """Make ``cache`` (a reference ``KVCacheManager``) run on the B200 kernels.

    ``graph_proxy_class`` is the reference's ``_DeviceCache`` (from
    ``vllm_rlt.worker.cuda_graph``); when given, its page write is rebound too
    so captured graphs contain the sm_100a write kernel. Returns the backend.
    """
    backend = B200PagedAttention(cache.device, cache.dtype, cache.head_dim, cache.block_size)
    cache.attention = backend
    cache.attention_info = backend.info
    if replace_write:

        def _write_prepared(layer, batch, k, v):
            # Same checks, in the same order, as the reference method.
            cache._validate_layer(layer)
            cache._require_live_batch(batch)
            if not batch.writable:
                raise ValueError("a read-only prepared KV batch cannot be written")
            cache._validate_tensor(k, len(batch.position_ids), "k")
            cache._validate_tensor(v, len(batch.position_ids), "v")
            if not batch.rows:
                return
            write_kv(cache.key_cache, cache.value_cache, layer, batch.write_blocks,
                     batch.write_offsets, k, v)
            for allocation, depth, position in batch.rows:
                allocation.written[cache._plane(depth)][layer].add(position)

        cache._write_prepared = _write_prepared
    if graph_proxy_class is not None:

        def _proxy_write(self, layer, batch, k, v):
            write_kv(self.cache.key_cache, self.cache.value_cache, layer, batch.write_blocks,
                     batch.write_offsets, k, v)

        graph_proxy_class._write_prepared = _proxy_write
    return backend

"""Install the B200 backend into a reference KV cache manager and runner.

The reference selects its attention backend from a fixed set of strings
(vllm_rlt/core/kv_cache_manager.py:109-131) and calls whatever object sits in
``cache.attention`` -- from ``_attend_prepared`` (:559-586) and from the
CUDA-graph proxy (vllm_rlt/worker/cuda_graph.py:21-29), which reads the
attribute at call time. Its own tests swap that attribute the same way
(tests/test_flash_attention.py:128).

The KV page write has no hook: it is a pair of index-puts,
``key_cache[write_blocks, layer, write_offsets] = k`` then the same for V,
inside ``KVCacheManager._write_prepared`` (:519-534) and inside the graph
proxy's ``_write_prepared`` (cuda_graph.py:16-19). ``install`` keeps running
the reference's own method bodies -- their validation, their order of checks
and their written-prefix bookkeeping, whatever version is installed -- and
hands them a stand-in for the cache whose ``key_cache`` / ``value_cache``
turn that pair of assignments into one sm_100a page write (``rlt_kv_write``).

The runner's other Triton launches (routing metadata, hidden-state gather /
scatter, the LAST-EXITED exit copy, packed-prefill metadata staging and
expansion) are looked up as module attributes at every call
(vllm_rlt/worker/async_state.py:47-111, vllm_rlt/worker/model_runner.py:511-557,
vllm_rlt/worker/prefill_metadata.py:20-86). ``install_routing`` replaces those
attributes with launch adapters that accept the Triton ``kernel[grid](...)``
form and argument order and run the sm_100a kernels instead.
"""

from __future__ import annotations

from .kernels import cache_ops, prefill_metadata, routing
from .kernels.cache_ops import write_kv
from .kernels.paged_attention import B200PagedAttention


class _PoolSide:
    """``key_cache`` or ``value_cache`` of a ``_PageWriteRoute``: an
    assignment ``side[blocks, layer, offsets] = rows`` is handed to the route;
    reads go to the real pool tensor."""

    def __init__(self, route, side, pool):
        self._route, self._side, self._pool = route, side, pool

    def __setitem__(self, index, rows):
        self._route._assign(self._side, index, rows)

    def __getitem__(self, index):
        return self._pool[index]

    def __getattr__(self, name):
        return getattr(self._pool, name)


class _PageWriteRoute:
    """Stands in for a reference cache while one of its page-write methods
    runs. Every attribute is the real cache's except ``key_cache`` and
    ``value_cache``: the method's two index-puts (same addresses, K then V)
    are collected and issued as one ``rlt_kv_write`` of both pools."""

    def __init__(self, cache):
        self._cache = cache
        self._held = {}
        self.key_cache = _PoolSide(self, "k", cache.key_cache)
        self.value_cache = _PoolSide(self, "v", cache.value_cache)

    def __getattr__(self, name):
        return getattr(self._cache, name)

    def _assign(self, side, index, rows):
        if not isinstance(index, tuple) or len(index) != 3:
            raise RuntimeError("the B200 page write expects pool[blocks, layer, offsets] = rows")
        if side in self._held:
            raise RuntimeError(f"two {side.upper()} page writes without the matching "
                               f"{'V' if side == 'k' else 'K'} write")
        self._held[side] = (index, rows)
        if len(self._held) < 2:
            return
        (kb, kl, ko), k = self._held.pop("k")
        (vb, vl, vo), v = self._held.pop("v")
        same = (kl == vl and kb.shape == vb.shape and ko.shape == vo.shape
                and kb.data_ptr() == vb.data_ptr() and ko.data_ptr() == vo.data_ptr())
        if not same:
            raise RuntimeError("K and V page writes must address the same slots")
        write_kv(self._cache.key_cache, self._cache.value_cache, int(kl), kb, ko, k, v)

    def finish(self):
        if self._held:
            raise RuntimeError("a K or V page write was left without its pair")


class _ProxySelf:
    """``self`` for the graph proxy's page write: its ``cache`` is routed."""

    def __init__(self, proxy):
        self._proxy = proxy
        self.cache = _PageWriteRoute(proxy.cache)

    def __getattr__(self, name):
        return getattr(self._proxy, name)


def _routed_method(method):
    """Run the reference's unbound page-write ``method`` with its pool
    assignments routed to the sm_100a write kernel."""

    def routed(cache, layer, batch, k, v):
        route = _PageWriteRoute(cache)
        method(route, layer, batch, k, v)
        route.finish()

    return routed


def install(cache, *, graph_proxy_class=None, replace_write=True):
    """Make ``cache`` (a reference ``KVCacheManager``) run on the B200 kernels.

    ``graph_proxy_class`` is the reference's ``_DeviceCache`` (from
    ``vllm_rlt.worker.cuda_graph``); when given, its page write is routed too
    so captured graphs contain the sm_100a write kernel (the class attribute
    is replaced once; later installs reuse it). Returns the backend.
    """
    backend = B200PagedAttention(cache.device, cache.dtype, cache.head_dim, cache.block_size)
    cache.attention = backend
    cache.attention_info = backend.info
    if replace_write:
        method = type(cache)._write_prepared
        routed = _routed_method(method)
        cache._write_prepared = lambda layer, batch, k, v: routed(cache, layer, batch, k, v)
    if graph_proxy_class is not None and not getattr(graph_proxy_class, "_rlt_routed", False):
        proxy_method = graph_proxy_class._write_prepared

        def _proxy_write(self, layer, batch, k, v):
            shim = _ProxySelf(self)
            proxy_method(shim, layer, batch, k, v)
            shim.cache.finish()

        graph_proxy_class._rlt_original_write = proxy_method
        graph_proxy_class._write_prepared = _proxy_write
        graph_proxy_class._rlt_routed = True
    return backend


def uninstall_graph_proxy(graph_proxy_class):
    """Undo ``install``'s change to the graph proxy class."""
    if getattr(graph_proxy_class, "_rlt_routed", False):
        graph_proxy_class._write_prepared = graph_proxy_class._rlt_original_write
        del graph_proxy_class._rlt_original_write
        graph_proxy_class._rlt_routed = False


class _GridLaunch:
    """``kernel[grid](*args)`` with a Triton kernel's argument order, run by
    ``launch(grid, *args)`` on the sm_100a kernels."""

    def __init__(self, name, launch):
        self.name, self._launch = name, launch
        self.calls = 0  # launches made through this adapter (process lifetime)

    def __getitem__(self, grid):
        grid = tuple(grid) if isinstance(grid, (tuple, list)) else (grid,)

        def launch(*args):
            self.calls += 1
            return self._launch(grid, *args)

        return launch

    def __repr__(self):
        return f"<sm_100a launch adapter for {self.name}>"


def _metadata(grid, d, tables, slots, positions, lengths, blocks, offsets, out_tables, n, size,
              width, page, planes, out_width, tile=None):
    # vllm_rlt/kernels/routing.py:7-41: one program per row of the bank (grid[0] == size)
    if tables.shape[2] != int(width):
        raise ValueError("metadata: WIDTH must equal the resident tables' width")
    routing.metadata(d, tables, slots, positions, lengths, blocks, offsets, out_tables, int(n),
                     int(grid[0]), int(page), int(planes), int(out_width))


def _gather(grid, pool, slots, out, n, h, in_stride, out_stride, tile=None):
    # vllm_rlt/kernels/routing.py:44-60: grid[0] rows, zeros past n
    if pool.stride(0) != int(in_stride) or out.stride(0) != int(out_stride):
        raise ValueError("gather: strides must be the tensors' row strides")
    pool2 = pool if pool.ndim > 1 else pool.view(-1, 1)
    routing.gather(pool2, slots, out, int(n), int(grid[0]))


def _scatter(grid, values, slots, pool, h, in_stride, out_stride, tile=None):
    # vllm_rlt/kernels/routing.py:63-76: grid[0] rows
    if values.stride(0) != int(in_stride) or pool.stride(0) != int(out_stride):
        raise ValueError("scatter: strides must be the tensors' row strides")
    routing.scatter(values, slots, pool, int(grid[0]))


def _finalize(grid, d, tables, k, v, width, planes, page, layers, channels, block_stride,
              layer_stride, token_stride, tile=None):
    # vllm_rlt/kernels/routing.py:79-109: grid[0] descriptor rows
    if tuple(k.stride()[:3]) != (int(block_stride), int(layer_stride), int(token_stride)):
        raise ValueError("finalize: strides must be the pool's")
    if tables.shape[1:] != (int(planes), int(width)) or k.shape[1] != int(layers):
        raise ValueError("finalize: WIDTH / PLANES / LAYERS disagree with the tensors")
    if k.shape[3] * k.shape[4] != int(channels) or k.shape[2] != int(page):
        raise ValueError("finalize: CHANNELS / PAGE disagree with the pool")
    cache_ops.finalize(d, tables, k, v, rows=int(grid[0]))


def _stage_prefill(grid, source, target, target32, n, tile=None):
    # vllm_rlt/kernels/prefill_metadata.py:7-12
    prefill_metadata.stage_prefill(source, target, target32, int(n))


def _expand_prefill(grid, positions, sequences, tables, blocks, offsets, n, width, page,
                    tile=None):
    # vllm_rlt/kernels/prefill_metadata.py:15-32
    prefill_metadata.expand_prefill(positions, sequences, tables, blocks, offsets, int(n),
                                    int(width), int(page))


ROUTING_LAUNCHES = {
    "metadata_kernel": _GridLaunch("metadata_kernel", _metadata),
    "gather_kernel": _GridLaunch("gather_kernel", _gather),
    "scatter_kernel": _GridLaunch("scatter_kernel", _scatter),
    "finalize_kernel": _GridLaunch("finalize_kernel", _finalize),
}
PREFILL_LAUNCHES = {
    "stage_prefill": _GridLaunch("stage_prefill", _stage_prefill),
    "expand_prefill": _GridLaunch("expand_prefill", _expand_prefill),
}


def install_routing(routing_module, prefill_metadata_module=None):
    """Replace the Triton kernels of the reference's ``vllm_rlt.kernels.routing``
    (and ``vllm_rlt.kernels.prefill_metadata``) module with sm_100a launch
    adapters. The runner imports them by name at every call, so the change
    takes effect at the next launch. Returns a function that restores the
    originals."""
    saved = []
    for module, launches in ((routing_module, ROUTING_LAUNCHES),
                             (prefill_metadata_module, PREFILL_LAUNCHES)):
        if module is None:
            continue
        for name, adapter in launches.items():
            saved.append((module, name, getattr(module, name)))
            setattr(module, name, adapter)

    def restore():
        for module, name, original in reversed(saved):
            setattr(module, name, original)

    return restore

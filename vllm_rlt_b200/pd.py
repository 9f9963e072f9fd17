"""KV page transport for prefill/decode disaggregation, over NVLink.

The reference's PD engine moves a request's KV pages from a prefill worker to
a decode worker with NIXL one-sided WRITEs between registered GPU pools
(vllm_rlt/pd/transport.py:18-176). On a B200 node every GPU reaches every
other at full NVLink bandwidth through NVSwitch, so the transport here is one
kernel launch per batch of segments that stores straight into the peer pool
(``rlt_copy_segments``), mapped into this process either by peer access (both
pools in one process) or by CUDA IPC (a pool tensor received from the other
process through ``torch.multiprocessing``).

* ``kv_segments`` / ``partition_segments`` -- the reference's segment lists
  (vllm_rlt/pd/transport.py:18-72): the wire contract between a prefill and
  a decode worker, so they are kept identical (pinned by the reference's own
  outputs in tests/golden/pd_segments.json);
* ``pool_info`` -- the geometry record the reference advertises
  (``NixlConnector.info``, :80-100);
* ``PageTransport`` -- ``connect`` / ``submit`` / ``poll`` / ``busy`` /
  ``close`` with the reference connector's meaning (:102-176): bounded
  in-flight bytes, a transfer is finished when its copy has completed on the
  device (a CUDA event instead of a NIXL status).
"""

from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass
from itertools import zip_longest

import torch

from . import _lib


def kv_segments(info, tables, start, end):
    """(address, bytes, device) segments holding tokens [start, end) of a
    request whose per-plane block tables are ``tables``, K then V, every
    layer. A block whose tokens are all inside the range is one segment (all
    layers are contiguous in a block); a partly covered block gives one
    segment per layer, covering only the valid tokens."""
    page = info["block_size"]
    if not 0 <= start < end:
        raise ValueError("invalid KV range")
    block_bytes, layer_bytes = info["block_bytes"], info["layer_bytes"]
    token_bytes, device = info["token_bytes"], info["device"]
    for table in tables:
        if end > len(table) * page:
            raise ValueError("KV range exceeds allocation")
        for logical in range(start // page, (end - 1) // page + 1):
            block = table[logical]
            if not 0 <= block < info["num_blocks"]:
                raise ValueError("physical block outside registered pool")
            first = max(start - logical * page, 0)
            stop = min(end - logical * page, page)
            whole = first == 0 and stop == page
            for base in (info["key_ptr"], info["value_ptr"]):
                origin = base + block * block_bytes
                if whole:
                    yield (origin, block_bytes, device)
                    continue
                for layer in range(info["num_layers"]):
                    yield (origin + layer * layer_bytes + first * token_bytes,
                           (stop - first) * token_bytes, device)


def partition_segments(source, target, byte_limit, descriptor_limit):
    """Pair source and target segments and cut them into transfers of at most
    ``byte_limit`` bytes and ``descriptor_limit`` segments (a segment that
    crosses the byte limit is split); yields (local, remote, bytes)."""
    local, remote, size = [], [], 0
    for src, dst in zip_longest(source, target):
        if src is None or dst is None or src[1] != dst[1]:
            raise ValueError("incompatible source/target KV geometry")
        done = 0
        while done < src[1]:
            take = min(src[1] - done, byte_limit - size)
            local.append((src[0] + done, take, src[2]))
            remote.append((dst[0] + done, take, dst[2]))
            size += take
            done += take
            if size == byte_limit or len(local) == descriptor_limit:
                yield local, remote, size
                local, remote, size = [], [], 0
    if local:
        yield local, remote, size


def pool_info(key_cache: torch.Tensor, value_cache: torch.Tensor, block_size: int, depths=None):
    """Geometry of a [blocks, layers, page, Hkv, D] KV pool pair."""
    if key_cache.shape != value_cache.shape or key_cache.dtype != value_cache.dtype:
        raise ValueError("key and value pools must match")
    element = key_cache.element_size()
    return dict(
        key_ptr=key_cache.data_ptr(), value_ptr=value_cache.data_ptr(),
        device=key_cache.device.index if key_cache.device.type == "cuda" else -1,
        num_blocks=key_cache.shape[0], block_size=block_size, num_layers=key_cache.shape[1],
        depths=depths, block_bytes=key_cache.stride(0) * element,
        layer_bytes=key_cache.stride(1) * element, token_bytes=key_cache.stride(2) * element,
    )


_GEOMETRY = ("block_size", "num_layers", "depths", "block_bytes", "layer_bytes", "token_bytes")


@dataclass
class Transfer:
    event: torch.cuda.Event
    transfer_id: str
    sequence: int
    size: int
    submitted: float


class PageTransport:
    """One-sided KV page writes from this process's GPU pool into peer pools.

    ``connect(name, key_cache, value_cache)`` takes the peer's pool tensors as
    this process sees them (another device here, or CUDA-IPC-shared tensors
    from the peer process). ``submit`` launches the copies on the transport's
    own stream and returns False, launching nothing, when the transfer would
    exceed the in-flight byte budget (the reference's back-pressure)."""

    def __init__(self, key_cache, value_cache, block_size, *, depths=None,
                 transfer_chunk_bytes=64 << 20, descriptor_limit=4096,
                 max_inflight_bytes=1 << 30, request_timeout=60.0):
        if key_cache.device.type != "cuda":
            raise ValueError("the KV page transport requires CUDA pools")
        if transfer_chunk_bytes <= 0 or max_inflight_bytes < transfer_chunk_bytes:
            raise ValueError("transfer chunk must be positive and fit the in-flight budget")
        self.device = key_cache.device
        self.info = pool_info(key_cache, value_cache, block_size, depths)
        self.storage = (key_cache, value_cache)
        self.chunk_bytes = transfer_chunk_bytes
        self.descriptor_limit = descriptor_limit
        self.max_inflight_bytes = max_inflight_bytes
        self.request_timeout = request_timeout
        self.stream = torch.cuda.Stream(device=self.device)
        self.peers = {}
        self.pending = deque()
        self.inflight_bytes = 0
        self.bytes_sent = 0
        self.transfers = 0
        self.transfer_seconds = 0.0

    def connect(self, name, key_cache, value_cache, depths=None):
        info = pool_info(key_cache, value_cache, self.info["block_size"], depths)
        for key in _GEOMETRY:
            if info[key] != self.info[key]:
                raise ValueError(f"PD KV geometry mismatch: {key}")
        if key_cache.device != self.device:
            with torch.cuda.device(self.device):
                _lib.check(_lib.load().rlt_enable_peer_access(key_cache.device.index),
                           "enable peer access")
        self.peers[name] = (info, key_cache, value_cache)

    def submit(self, transfer_id, sequence, peer, local_tables, remote_tables, start, end):
        """Copy tokens [start, end) of every plane to the peer's pages; the
        tables are the request's per-plane block tables on each side."""
        info = self.peers[peer][0]
        source = list(kv_segments(self.info, local_tables, start, end))
        target = list(kv_segments(info, remote_tables, start, end))
        batches = list(partition_segments(source, target, self.chunk_bytes, self.descriptor_limit))
        size = sum(n for _, _, n in batches)
        if self.inflight_bytes + size > self.max_inflight_bytes:
            return False
        lib = _lib.load()
        status = _lib.status_word(self.device).data_ptr()
        with torch.cuda.stream(self.stream):
            for local, remote, n in batches:
                rows = [(a[0], b[0], a[1]) for a, b in zip(local, remote)]
                host = torch.tensor(rows, dtype=torch.int64).pin_memory()
                desc = host.to(self.device, non_blocking=True)
                code = lib.rlt_copy_segments(desc.data_ptr(), len(rows), max(r[2] for r in rows),
                                             status, self.stream.cuda_stream)
                _lib.check(code, "KV page transport")
                desc.record_stream(self.stream)
            event = torch.cuda.Event()
            event.record(self.stream)
        self.pending.append(Transfer(event, transfer_id, sequence, size, time.monotonic()))
        self.inflight_bytes += size
        return True

    def poll(self):
        """Transfers whose copies completed since the last poll."""
        remaining, finished = deque(), []
        for ticket in self.pending:
            if not ticket.event.query():
                if time.monotonic() - ticket.submitted > self.request_timeout:
                    raise TimeoutError("KV page transfer timed out")
                remaining.append(ticket)
                continue
            self.inflight_bytes -= ticket.size
            self.bytes_sent += ticket.size
            self.transfers += 1
            self.transfer_seconds += time.monotonic() - ticket.submitted
            finished.append(ticket)
        self.pending = remaining
        return finished

    def busy(self, transfer_id):
        return any(t.transfer_id == transfer_id for t in self.pending)

    def close(self):
        if self.pending:
            raise RuntimeError("cannot release the pools with in-flight transfers")
        self.peers.clear()
        self.storage = None

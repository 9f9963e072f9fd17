"""KV page transport for prefill/decode disaggregation, over NVLink.

The reference's PD engine moves a request's KV pages from a prefill worker to
a decode worker with one-sided writes between registered GPU pools
(vllm_rlt/pd/transport.py:18-176). On a B200 node every GPU reaches every
other at full NVLink bandwidth through NVSwitch, so a transfer here is one
kernel launch per batch of segments that stores straight into the peer pool
(``rlt_copy_segments``), mapped into this process either by peer access (both
pools in one process) or by CUDA IPC (a pool tensor received from the other
process through ``torch.multiprocessing``).

The segment list is the contract between the two workers: both sides must
describe the same bytes in the same order, so a prefill worker built on this
package can feed a decode worker built on the reference. Its format:

* for each plane table in order, for each logical page touched by tokens
  [start, end) in order, the K segments then the V segments of that page;
* a page whose ``block_size`` tokens all lie in the range is one segment of
  ``block_bytes`` at the block's start (all layers of a block are
  contiguous);
* a partly covered page gives one segment per layer, at
  ``block * block_bytes + layer * layer_bytes + first * token_bytes``, of
  ``(stop - first) * token_bytes`` bytes, where [first, stop) are the
  covered in-page token offsets;
* each segment is (address, bytes, device).

A list of paired segments is cut into transfers of at most ``byte_limit``
bytes and ``descriptor_limit`` segments, in order; a segment that would
overflow the byte limit is split there and its remainder opens the next
transfer. ``tests/golden/pd_segments.json`` holds the reference's own lists
for seeded cases and pins both functions.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib


def kv_segments(info, tables, start, end) -> np.ndarray:
    """Segments of tokens [start, end) of a request whose per-plane block
    tables are ``tables``: an int64 array [n, 3] of (address, bytes, device)
    rows in the order the module docstring states."""
    page = int(info["block_size"])
    if not (0 <= start < end):
        raise ValueError(f"empty or negative token range [{start}, {end})")
    tables = [np.asarray(t, dtype=np.int64) for t in tables]
    if not tables:
        return np.zeros((0, 3), dtype=np.int64)
    first_page, last_page = start // page, (end - 1) // page
    logical = np.arange(first_page, last_page + 1, dtype=np.int64)
    for t in tables:
        if len(t) * page < end:
            raise ValueError(f"token range ends at {end}, past the {len(t) * page} tokens the "
                             f"block table holds")
    blocks = np.stack([t[logical] for t in tables])  # [planes, pages]
    if ((blocks < 0) | (blocks >= int(info["num_blocks"]))).any():
        raise ValueError("a block table names a block outside the pool")
    first = np.maximum(start - logical * page, 0)  # covered in-page offsets [first, stop)
    stop = np.minimum(end - logical * page, page)
    whole = (first == 0) & (stop == page)
    layers = int(info["num_layers"])
    block_bytes, layer_bytes = int(info["block_bytes"]), int(info["layer_bytes"])
    token_bytes = int(info["token_bytes"])
    planes, pages = blocks.shape
    # One group per (plane, page, K/V) in output order; a group holds one
    # segment (whole page) or one per layer (partial page).
    g_block = np.repeat(blocks.reshape(-1), 2)
    g_base = np.tile(np.array([info["key_ptr"], info["value_ptr"]], dtype=np.int64),
                     planes * pages)
    g_page = np.tile(np.repeat(np.arange(pages), 2), planes)
    g_whole = whole[g_page]
    count = np.where(g_whole, 1, layers)
    group = np.repeat(np.arange(len(count)), count)
    # index of each segment within its group (the layer, for partial pages)
    starts = np.cumsum(count) - count
    layer = np.arange(len(group)) - starts[group]
    p = g_page[group]
    is_whole = g_whole[group]
    address = g_base[group] + g_block[group] * block_bytes
    address = address + np.where(is_whole, 0, layer * layer_bytes + first[p] * token_bytes)
    size = np.where(is_whole, block_bytes, (stop[p] - first[p]) * token_bytes)
    device = np.full(len(group), int(info["device"]), dtype=np.int64)
    return np.stack([address, size, device], axis=1).astype(np.int64)


def partition_segments(source, target, byte_limit, descriptor_limit):
    """Cut paired source/target segment lists into transfers; returns a list
    of (local [m, 3], remote [m, 3], bytes) with at most ``byte_limit`` bytes
    and ``descriptor_limit`` segments each.

    Works transfer by transfer on the running byte total: a transfer that
    begins ``consumed`` bytes into the stream ends at the first segment
    boundary reaching ``consumed + byte_limit`` (found by binary search on
    the cumulative sizes) or after ``descriptor_limit`` segments, whichever
    comes first; only the byte bound can fall inside a segment."""
    src = np.asarray(source, dtype=np.int64).reshape(-1, 3)
    dst = np.asarray(target, dtype=np.int64).reshape(-1, 3)
    if src.shape != dst.shape or not np.array_equal(src[:, 1], dst[:, 1]):
        raise ValueError("source and target segment lists describe different byte layouts")
    if byte_limit <= 0 or descriptor_limit <= 0:
        raise ValueError("transfer limits must be positive")
    ends = np.cumsum(src[:, 1])  # stream offset where each segment ends
    total = int(ends[-1]) if len(ends) else 0
    out = []
    consumed, index = 0, 0  # stream bytes already sent; the segment they stop in
    while consumed < total:
        limit = consumed + byte_limit
        # the last segment this transfer may touch by bytes, then by count
        last = min(int(np.searchsorted(ends, limit, side="left")), len(ends) - 1,
                   index + descriptor_limit - 1)
        stop = min(int(ends[last]), limit)
        seg_start = ends[index : last + 1] - src[index : last + 1, 1]
        lo = np.maximum(seg_start, consumed)  # covered part of each segment
        hi = np.minimum(ends[index : last + 1], stop)
        offset = lo - seg_start
        local = np.stack([src[index : last + 1, 0] + offset, hi - lo,
                          src[index : last + 1, 2]], axis=1)
        remote = np.stack([dst[index : last + 1, 0] + offset, hi - lo,
                           dst[index : last + 1, 2]], axis=1)
        out.append((local, remote, int(stop - consumed)))
        consumed = stop
        index = last if stop < ends[last] else last + 1
    return out


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


# pool geometry two workers must share before pages can move between them
_MATCHING = ("block_size", "num_layers", "depths", "block_bytes", "layer_bytes", "token_bytes")


@dataclass
class Ticket:
    """One submitted transfer: done when ``event`` has completed."""

    transfer_id: str
    sequence: int
    size: int
    event: torch.cuda.Event
    submitted: float = field(default_factory=time.monotonic)


class _DescriptorRing:
    """Pinned host staging for segment descriptors, reused across submits.

    Each slot is a pinned host buffer and a device buffer of (src, dst,
    bytes) rows; a slot is refilled only after the event recorded behind its
    last launch has completed, so the host never overwrites rows a pending
    copy still reads."""

    def __init__(self, device, slots=4, rows=256):
        self.device = device
        self.slots = [self._make(rows) for _ in range(slots)]
        self.next = 0

    def _make(self, rows):
        return dict(host=torch.empty((rows, 3), dtype=torch.int64).pin_memory(),
                    dev=torch.empty((rows, 3), dtype=torch.int64, device=self.device),
                    event=None)

    def stage(self, rows: np.ndarray, stream) -> torch.Tensor:
        slot = self.slots[self.next]
        self.next = (self.next + 1) % len(self.slots)
        if slot["event"] is not None:
            slot["event"].synchronize()
        if len(rows) > slot["host"].shape[0]:
            grown = self._make(1 << (len(rows) - 1).bit_length())
            slot.update(host=grown["host"], dev=grown["dev"])
        slot["host"].numpy()[: len(rows)] = rows
        dev = slot["dev"][: len(rows)]
        dev.copy_(slot["host"][: len(rows)], non_blocking=True)
        slot["event"] = torch.cuda.Event()
        return dev, slot

    @staticmethod
    def fence(slot, stream):
        slot["event"].record(stream)


class PageTransport:
    """One-sided KV page writes from this process's GPU pool into peer pools.

    ``connect(name, key_cache, value_cache)`` takes the peer's pool tensors as
    this process sees them (another device here, or CUDA-IPC-shared tensors
    from the peer process). ``submit`` launches the copies on the transport's
    own stream and returns False, launching nothing, when the transfer would
    take the bytes in flight past ``max_inflight_bytes`` (back-pressure, as
    the reference's connector applies). ``poll`` returns the transfers whose
    copies have completed on the device."""

    def __init__(self, key_cache, value_cache, block_size, *, depths=None,
                 transfer_chunk_bytes=64 << 20, descriptor_limit=4096,
                 max_inflight_bytes=1 << 30, request_timeout=60.0):
        if key_cache.device.type != "cuda":
            raise ValueError("the KV page transport moves pages between CUDA pools only")
        if transfer_chunk_bytes <= 0 or max_inflight_bytes < transfer_chunk_bytes:
            raise ValueError("transfer_chunk_bytes must be positive and at most "
                             "max_inflight_bytes")
        self.device = key_cache.device
        self.info = pool_info(key_cache, value_cache, block_size, depths)
        self.storage = (key_cache, value_cache)
        self.limits = (int(transfer_chunk_bytes), int(descriptor_limit))
        self.max_inflight_bytes = int(max_inflight_bytes)
        self.request_timeout = request_timeout
        self.stream = torch.cuda.Stream(device=self.device)
        self.ring = _DescriptorRing(self.device)
        self.peers = {}
        self.pending: list[Ticket] = []
        self.stats = dict(bytes=0, transfers=0, seconds=0.0)

    @property
    def inflight_bytes(self) -> int:
        return sum(t.size for t in self.pending)

    def connect(self, name, key_cache, value_cache, depths=None):
        info = pool_info(key_cache, value_cache, self.info["block_size"], depths)
        differing = [k for k in _MATCHING if info[k] != self.info[k]]
        if differing:
            raise ValueError(f"peer pool {name!r} has a different KV geometry "
                             f"({', '.join(differing)})")
        if key_cache.device != self.device:
            with torch.cuda.device(self.device):
                _lib.check(_lib.load().rlt_enable_peer_access(key_cache.device.index),
                           "enable peer access")
        self.peers[name] = (info, key_cache, value_cache)

    def submit(self, transfer_id, sequence, peer, local_tables, remote_tables, start, end):
        """Copy tokens [start, end) of every plane to the peer's pages; the
        tables are the request's per-plane block tables on each side."""
        info = self.peers[peer][0]
        source = kv_segments(self.info, local_tables, start, end)
        target = kv_segments(info, remote_tables, start, end)
        transfers = partition_segments(source, target, *self.limits)
        size = sum(n for _, _, n in transfers)
        if self.inflight_bytes + size > self.max_inflight_bytes:
            return False
        lib = _lib.load()
        status = _lib.status_word(self.device).data_ptr()
        with torch.cuda.stream(self.stream):
            for local, remote, _ in transfers:
                rows = np.stack([local[:, 0], remote[:, 0], local[:, 1]], axis=1)
                desc, slot = self.ring.stage(rows, self.stream)
                code = lib.rlt_copy_segments(desc.data_ptr(), len(rows), int(rows[:, 2].max()),
                                             status, self.stream.cuda_stream)
                _lib.check(code, "KV page transport")
                self.ring.fence(slot, self.stream)
            event = torch.cuda.Event()
            event.record(self.stream)
        self.pending.append(Ticket(transfer_id, sequence, size, event))
        return True

    def poll(self):
        """Transfers whose copies completed since the last poll; raises
        ``TimeoutError`` for one pending longer than ``request_timeout``."""
        now = time.monotonic()
        done = [t for t in self.pending if t.event.query()]
        late = [t for t in self.pending if t not in done and now - t.submitted > self.request_timeout]
        if late:
            raise TimeoutError(f"KV page transfer {late[0].transfer_id!r} has not completed "
                               f"after {self.request_timeout} s")
        self.pending = [t for t in self.pending if t not in done]
        for t in done:
            self.stats["bytes"] += t.size
            self.stats["transfers"] += 1
            self.stats["seconds"] += now - t.submitted
        return done

    def busy(self, transfer_id) -> bool:
        return transfer_id in {t.transfer_id for t in self.pending}

    def close(self):
        if self.pending:
            raise RuntimeError("transfers are still in flight; poll until they finish before "
                               "closing the transport")
        self.peers.clear()
        self.storage = None

"""GPU-side test utilities: torch <-> numpy storage, and a pool writer that
applies a golden scenario's writes and exit copies through the CUDA kernels."""

from __future__ import annotations

import numpy as np
import torch

import vllm_rlt_b200 as rb

TORCH = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def to_torch(array: np.ndarray, dtype: str, device="cuda") -> torch.Tensor:
    """numpy storage form -> torch tensor of ``dtype`` (bf16 from uint16 bits)."""
    if dtype == "bf16":
        t = torch.from_numpy(np.ascontiguousarray(array).view(np.int16)).view(torch.bfloat16)
    else:
        t = torch.from_numpy(np.ascontiguousarray(array))
    return t.to(device)


def to_numpy(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


class CudaWriter:
    """Replays writes with rb.write_kv and exit copies with rb.finalize."""

    def __init__(self, shape, dtype: str, device="cuda"):
        self.dtype = dtype
        self.key = torch.zeros(shape, dtype=TORCH[dtype], device=device)
        self.value = torch.zeros_like(self.key)
        self.device = torch.device(device)
        self._pending = []  # batched writes (distinct addresses) awaiting one launch
        self._addresses = set()

    def write(self, layer, block, offset, k, v):
        # One launch may not write an address twice (the reference rejects
        # duplicate write addresses in a batch): flush on a repeat.
        if (layer, block, offset) in self._addresses:
            self.flush()
        self._addresses.add((layer, block, offset))
        self._pending.append((layer, block, offset, k, v))

    def flush(self):
        if not self._pending:
            return
        by_layer = {}
        for layer, block, offset, k, v in self._pending:
            by_layer.setdefault(layer, []).append((block, offset, k, v))
        for layer, items in by_layer.items():
            blocks = torch.tensor([i[0] for i in items], dtype=torch.int64, device=self.device)
            offsets = torch.tensor([i[1] for i in items], dtype=torch.int64, device=self.device)
            k = to_torch(np.stack([i[2] for i in items]), self.dtype, self.device)
            v = to_torch(np.stack([i[3] for i in items]), self.dtype, self.device)
            rb.write_kv(self.key, self.value, layer, blocks, offsets, k, v)
        self._pending.clear()
        self._addresses.clear()

    def finalize(self, plane_tables, pos, exit_depth, planes, page):
        # A write batch never holds two writes to one address, and the exit
        # copy reads what the batch wrote: flush first.
        self.flush()
        width = plane_tables.shape[1]
        tables = torch.from_numpy(np.ascontiguousarray(plane_tables, dtype=np.int32)).to(
            self.device).view(1, planes, width)
        desc = torch.tensor([[0, exit_depth, pos]], dtype=torch.int64, device=self.device)
        rb.finalize(desc, tables, self.key, self.value)

    def numpy(self):
        self.flush()
        return to_numpy(self.key), to_numpy(self.value)

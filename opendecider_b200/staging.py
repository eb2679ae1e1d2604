"""Host-to-device staging of one call's inputs: every small host tensor a plan needs (token ids, positions, row
layouts, readout constants) is packed into ONE pinned host buffer and moved by ONE cudaMemcpyAsync on the current
stream, instead of one pageable copy per tensor. Device views are handed out immediately; the kernels that read them
are enqueued after the copy on the same stream, so stream order makes the data visible to them.

A Staging arena is reused call after call: begin() waits for the previous copy out of the pinned buffer to finish
before it is overwritten, so a plan stays valid until the next begin() on the same arena.
"""
from __future__ import annotations

import torch

ALIGN = 256


class Staging:
    def __init__(self, device: torch.device, capacity: int = 1 << 24):
        self.device = torch.device(device)
        self._alloc(capacity)
        self.used = 0
        self.moved = 0
        self.bytes_last = 0
        self._done = []          # (event, pinned buffer) of copies still reading host memory

    def _alloc(self, capacity: int):
        self.capacity = capacity
        self.host = torch.empty(capacity, dtype=torch.uint8, pin_memory=True)
        self.dev = torch.empty(capacity, dtype=torch.uint8, device=self.device)

    def begin(self, reserve: int = 0) -> None:
        """Start packing a new call's tensors (reserve: a lower bound of the bytes this call will stage)."""
        for ev, _ in self._done:
            ev.synchronize()                # earlier copies have finished reading their pinned buffers
        self._done = []
        if reserve > self.capacity:
            self._alloc(1 << (reserve - 1).bit_length())
        self.used = 0
        self.moved = 0

    def put(self, x: torch.Tensor) -> torch.Tensor:
        """Stage host tensor x; returns its device view (valid once commit() has been enqueued)."""
        x = x.contiguous()
        n = x.numel() * x.element_size()
        off = self.used
        end = off + n
        if end > self.capacity:
            # grow: ship what is staged so far from the current buffers (their views stay alive), then continue
            self._flush()
            self._alloc(max(2 * self.capacity, 1 << (n + ALIGN - 1).bit_length()))
            self.used = 0
            off, end = 0, n
        if n:
            self.host[off:end].copy_(x.view(-1).view(torch.uint8))
        self.used = -(-end // ALIGN) * ALIGN
        return self.dev[off:end].view(x.dtype).view(x.shape)

    def _flush(self) -> None:
        if self.used:
            self.dev[: self.used].copy_(self.host[: self.used], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            self._done.append((ev, self.host))
            self.moved += self.used
            self.used = 0

    def commit(self) -> int:
        """One host->device copy of everything staged since begin(). Returns the bytes moved by this call."""
        self._flush()
        self.bytes_last = self.moved
        return self.moved

"""Decode routing trace and routing histograms, recorded on the device.

The reference records each batch-size-1 decode step's raw top-k expert ids into a device
ring with ``index_copy_`` at a device cursor, so a captured decode graph keeps recording
on replay (backends/.../moe/offload_cache.py:225-240, :859-862), accumulates a per-layer
routing histogram the same way (``collect_decode_freq``, :211-224, :853-857), and its
manager dumps routes, request marks and prefill expert counts to an NPZ file
(src/tideway/offload/runtime.py:1037-1066).  ``RouteTrace`` keeps rows of any width (one
row per ensure call: the layer's T x K ids, padded with -1), so it also covers batched
decode.
"""

from __future__ import annotations

import numpy as np
import torch


class RouteTrace:
    """A ring of ``rows`` records of up to ``width`` routed expert ids plus the layer id.

    ``record`` issues only device operations (no host synchronisation, no allocation), so
    calls made while a CUDA graph is captured are replayed with it.
    """

    def __init__(self, rows: int, width: int, device):
        if rows <= 0 or width <= 0:
            raise ValueError("trace rows and width must be positive")
        self.rows, self.width = int(rows), int(width)
        dev = torch.device(device)
        self.ids = torch.full((self.rows, self.width), -1, dtype=torch.int32, device=dev)
        self.layer = torch.full((self.rows,), -1, dtype=torch.int32, device=dev)
        self.pos = torch.zeros((1,), dtype=torch.int64, device=dev)
        self._row = torch.full((1, self.width), -1, dtype=torch.int32, device=dev)

    def record(self, layer_id: int, expert_ids: torch.Tensor) -> None:
        flat = expert_ids.reshape(-1)
        n = flat.numel()
        if n > self.width:
            raise ValueError(f"{n} routed ids do not fit a trace row of {self.width}")
        row = torch.remainder(self.pos, self.rows)
        self._row.fill_(-1)
        self._row[0, :n].copy_(flat)
        self.ids.index_copy_(0, row, self._row)
        self.layer.index_fill_(0, row, int(layer_id))
        self.pos.add_(1)

    def reset(self) -> None:
        self.ids.fill_(-1)
        self.layer.fill_(-1)
        self.pos.zero_()

    def read(self) -> tuple[np.ndarray, np.ndarray, int]:
        """(layers [n], ids [n, width], records ever written) in recording order, the
        oldest first; a full ring keeps the last ``rows`` records.  Synchronises."""
        total = int(self.pos.item())
        n = min(total, self.rows)
        start = total % self.rows if total > self.rows else 0
        order = (start + np.arange(n)) % self.rows
        return (self.layer.cpu().numpy()[order], self.ids.cpu().numpy()[order], total)


def accumulate_histogram(hist: torch.Tensor, layer_id: int, expert_ids: torch.Tensor) -> None:
    """hist[layer_id, e] += number of routes to expert e (negative ids are padding)."""
    ids = expert_ids.reshape(-1).long()
    ones = (ids >= 0).to(hist.dtype)
    hist[layer_id].scatter_add_(0, ids.clamp(min=0), ones)

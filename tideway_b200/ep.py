"""Expert parallelism: a layer's routed experts sharded over the GPUs of a process group.

GPU d owns experts [d*Eg, (d+1)*Eg) of every layer in its own slot cache.  Per layer:

1. ``tw_ep_dispatch`` packs one fixed-size row per (destination GPU, local token): the
   token's input row, the local expert ids of its routes on that GPU (-1 elsewhere) and the
   router weights;
2. one NCCL all-to-all moves the rows (fixed shapes: no host sync, capturable);
3. ``tw_ep_receive`` unpacks them; the owner's slot cache rewrites local expert ids into
   slot ids in place (``ensure_experts``/``copy_missing``) and the slot-indirect tensor-core
   FFN computes one partial sum per received row;
4. a second all-to-all returns the partials; ``tw_ep_combine`` adds them in GPU order.

The reference's MoE path is single-GPU (src/tideway/offload/paged_decode_graph.py:62-63);
this is the expert-parallel sharding the benchmark configuration adds.  With one GPU the
all-to-alls are local copies.
"""

from __future__ import annotations

import torch

from . import _lib, ops
from .offload_cache import OffloadMoeCache


def _dist():
    import torch.distributed as dist

    return dist


class ExpertParallelMoE:
    def __init__(self, num_experts: int, topk: int, hidden: int, inter: int, tokens: int,
                 device, group=None):
        dist = _dist()
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not shard evenly over {self.world} GPUs")
        self.E, self.K, self.H, self.I, self.T = num_experts, topk, hidden, inter, tokens
        self.Eg = num_experts // self.world
        self.device = torch.device(device)
        rb = int(_lib.load().tw_ep_row_bytes(hidden, topk))
        rows = self.world * tokens
        self.row_bytes = rb
        self.send = torch.empty(rows, rb, dtype=torch.uint8, device=self.device)
        self.recv = torch.empty_like(self.send)
        self.x = torch.empty(rows, hidden, dtype=torch.bfloat16, device=self.device)
        self.ids = torch.empty(rows, topk, dtype=torch.int32, device=self.device)
        self.w = torch.empty(rows, topk, dtype=torch.float32, device=self.device)
        self.part = torch.empty(rows, hidden, dtype=torch.bfloat16, device=self.device)
        self.back = torch.empty_like(self.part)
        self.ws = torch.empty(ops.workspace_bytes(rows * topk, hidden, inter), dtype=torch.uint8,
                              device=self.device)

    def static_tensors(self) -> list[torch.Tensor]:
        """The buffers a captured step reads and writes (fixed addresses)."""
        return [self.send, self.recv, self.x, self.ids, self.w, self.part, self.back, self.ws]

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        if self.world == 1:
            out.copy_(inp)
        else:
            _dist().all_to_all_single(out, inp, group=self.group)

    def _dispatch(self, x, topk_w, topk_ids) -> None:
        T, H = x.shape
        if T != self.T or H != self.H or topk_ids.shape != (T, self.K):
            raise ValueError("expert-parallel shapes are fixed at construction")
        st = torch.cuda.current_stream().cuda_stream
        _lib.call("tw_ep_dispatch", x.data_ptr(), topk_w.data_ptr(), topk_ids.data_ptr(), T,
                  self.K, H, self.Eg, self.world, self.send.data_ptr(), st)
        self._a2a(self.recv, self.send)
        _lib.call("tw_ep_receive", self.recv.data_ptr(), self.world * T, self.K, H,
                  self.x.data_ptr(), self.ids.data_ptr(), self.w.data_ptr(), st)

    def _combine(self, out: torch.Tensor) -> torch.Tensor:
        self._a2a(self.back, self.part)
        _lib.call("tw_ep_combine", self.back.data_ptr(), self.T, self.H, self.world,
                  out.data_ptr(), torch.cuda.current_stream().cuda_stream)
        return out

    def forward_resident(self, x: torch.Tensor, topk_w: torch.Tensor, topk_ids: torch.Tensor,
                         banks: tuple, out: torch.Tensor) -> torch.Tensor:
        """Routed expert output when this GPU's expert shard is resident: ``banks`` are the
        shard's NVFP4 banks ((w1 packed, scale, global), (w2 packed, scale, global)) indexed
        by local expert id, or its BF16 banks (w1, w2)."""
        self._dispatch(x, topk_w, topk_ids)
        w1, w2 = banks
        if isinstance(w1, tuple):
            ops.moe_ffn_nvfp4(self.x, w1, w2, self.w, self.ids, out=self.part, ws=self.ws)
        else:
            ops.moe_ffn_bf16(self.x, w1, w2, self.w, self.ids, out=self.part, ws=self.ws)
        return self._combine(out)

    def forward(self, x: torch.Tensor, topk_w: torch.Tensor, topk_ids: torch.Tensor,
                layer_id: int, cache: OffloadMoeCache, out: torch.Tensor) -> torch.Tensor:
        """Routed expert output for this GPU's tokens; ``topk_ids`` are global expert ids."""
        T, H = x.shape
        if T != self.T or H != self.H or topk_ids.shape != (T, self.K):
            raise ValueError("expert-parallel shapes are fixed at construction")
        if cache.num_experts != self.Eg:
            raise ValueError("the slot cache must hold this GPU's expert shard")
        st = torch.cuda.current_stream().cuda_stream
        _lib.call("tw_ep_dispatch", x.data_ptr(), topk_w.data_ptr(), topk_ids.data_ptr(), T,
                  self.K, H, self.Eg, self.world, self.send.data_ptr(), st)
        self._a2a(self.recv, self.send)
        _lib.call("tw_ep_receive", self.recv.data_ptr(), self.world * T, self.K, H,
                  self.x.data_ptr(), self.ids.data_ptr(), self.w.data_ptr(), st)
        cache.ensure_experts(layer_id, self.ids)
        cache.copy_missing()
        gate_up, down = cache.bank_views()
        ops.moe_ffn_bf16(self.x, gate_up, down, self.w, self.ids, out=self.part, ws=self.ws)
        self._a2a(self.back, self.part)
        _lib.call("tw_ep_combine", self.back.data_ptr(), T, H, self.world, out.data_ptr(), st)
        return out

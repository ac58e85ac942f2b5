"""Expert parallelism: a layer's routed experts sharded over the GPUs of a process group.

GPU d owns experts [d*Eg, (d+1)*Eg) of every layer in its own slot cache.  Two transports
move the token rows and the partial outputs; both compute the same numbers.

``transport="p2p"`` (the default): our own kernels write straight into the other GPUs'
memory over NVLink (CUDA IPC mappings of one exchange buffer per GPU, device-side flags,
bounded waits; ``csrc/ep_p2p.cu``).  Per layer:

1. ``tw_ep_p2p_dispatch`` writes every token's local expert ids and router weights into
   each GPU's buffer, and its input row only where it has a route, then waits until every
   GPU's rows for this one have landed;
2. the owner's slot cache rewrites the received local ids into slot ids in place
   (``ensure_experts``/``copy_missing``) and ``tw_moe_ffn_bf16_routes`` computes every
   received route's weighted output (the combine is left to step 3);
3. ``tw_ep_p2p_combine`` sends each received row's partial sum back into its source GPU's
   buffer, waits for the partials of its own tokens, adds them in GPU order and applies the
   next residual RMSNorm when asked.

``transport="nccl"``: ``tw_ep_dispatch`` packs one fixed-size row per (destination, token),
one NCCL all-to-all moves them, ``tw_ep_receive`` unpacks, the FFN computes one partial per
row, a second all-to-all returns them and ``tw_ep_combine`` adds them in GPU order.

The reference's MoE path is single-GPU (src/tideway/offload/paged_decode_graph.py:62-63);
this is the expert-parallel sharding the benchmark configuration adds.  With one GPU the
exchanges stay on that GPU.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib, ops
from .offload_cache import OffloadMoeCache


def _dist():
    import torch.distributed as dist

    return dist


class P2PUnavailable(RuntimeError):
    """Raised on every GPU of the group alike when the peer-memory exchange cannot be set up
    (a buffer that CUDA IPC cannot export, a peer that cannot be mapped)."""


class P2PExchange:
    """One exchange buffer per GPU, mapped into every peer of the group (CUDA IPC): the
    received operands (x, local ids, weights) and the returned partials are views of it."""

    def __init__(self, world: int, rank: int, tokens: int, hidden: int, topk: int, device,
                 group=None):
        lib = _lib.load()
        self.world, self.rank = world, rank
        nbytes = int(lib.tw_ep_p2p_bytes(world, tokens, hidden, topk))
        self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=device)  # flags start at 0
        hb = int(lib.tw_ep_p2p_handle_bytes())
        handle = (C.c_uint8 * hb)()
        off = C.c_uint64()
        ok = lib.tw_ep_p2p_export(self.buf.data_ptr(), C.cast(handle, C.c_void_p),
                                  C.byref(off)) == 0
        # handle bytes, offset, and whether this GPU could export (every GPU learns of all)
        mine = torch.tensor(list(bytes(handle)) + list(off.value.to_bytes(8, "little")) +
                            [int(ok)], dtype=torch.uint8, device=device)
        if world > 1:
            every = [torch.empty_like(mine) for _ in range(world)]
            _dist().all_gather(every, mine, group=group)
        else:
            every = [mine]
        every = [bytes(e.cpu().tolist()) for e in every]
        self.mappings = []
        if not all(e[hb + 8] for e in every):
            raise P2PUnavailable("an exchange buffer could not be exported for CUDA IPC")
        peers = []
        opened = True
        for d in range(world):
            if d == rank:
                peers.append(self.buf.data_ptr())
                continue
            h = (C.c_uint8 * hb).from_buffer_copy(every[d][:hb])
            ptr, mapping = C.c_void_p(), C.c_void_p()
            if lib.tw_ep_p2p_open(C.cast(h, C.c_void_p),
                                  int.from_bytes(every[d][hb:hb + 8], "little"), C.byref(ptr),
                                  C.byref(mapping)) != 0:
                opened = False
                break
            peers.append(ptr.value)
            self.mappings.append(mapping.value)
        if world > 1:  # every GPU must reach every peer, or none uses this transport
            flag = torch.tensor([int(opened)], dtype=torch.int32, device=device)
            _dist().all_reduce(flag, op=_dist().ReduceOp.MIN, group=group)
            opened = bool(flag.item())
        if not opened:
            self.close()
            raise P2PUnavailable("a peer's exchange buffer could not be mapped")
        self.peers = (C.c_void_p * world)(*peers)
        offs = (C.c_size_t * 4)()
        _lib.call("tw_ep_p2p_offsets", world, tokens, hidden, topk, C.cast(offs, C.c_void_p))
        rows = world * tokens

        def view(at, dtype, shape):
            n = shape[0] * shape[1] * torch.tensor([], dtype=dtype).element_size()
            return self.buf[at:at + n].view(dtype).view(*shape)

        self.x = view(offs[0], torch.bfloat16, (rows, hidden))
        self.ids = view(offs[1], torch.int32, (rows, topk))
        self.w = view(offs[2], torch.float32, (rows, topk))
        self.back = view(offs[3], torch.bfloat16, (rows, hidden))

    def error(self) -> int:
        """The buffer's error word (synchronises): 1 = a wait for a peer gave up."""
        err = torch.zeros(1, dtype=torch.int32, device=self.buf.device)
        _lib.call("tw_ep_p2p_error", self.buf.data_ptr(), err.data_ptr(),
                  torch.cuda.current_stream().cuda_stream)
        return int(err.item())

    def close(self) -> None:
        """Unmap the peers' buffers (every GPU of the group must have stopped using them)."""
        for m in self.mappings:
            _lib.call("tw_ep_p2p_close", m)
        self.mappings = []


class ExpertParallelMoE:
    def __init__(self, num_experts: int, topk: int, hidden: int, inter: int, tokens: int,
                 device, group=None, transport: str = "p2p"):
        dist = _dist()
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not shard evenly over {self.world} GPUs")
        if transport not in ("p2p", "nccl"):
            raise ValueError(f"unknown transport {transport!r}")
        self.transport = transport
        self.E, self.K, self.H, self.I, self.T = num_experts, topk, hidden, inter, tokens
        self.Eg = num_experts // self.world
        self.device = torch.device(device)
        rows = self.world * tokens
        self.ws = torch.empty(ops.workspace_bytes(rows * topk, hidden, inter), dtype=torch.uint8,
                              device=self.device)
        if transport == "p2p":
            try:
                self.xc = P2PExchange(self.world, self.rank, tokens, hidden, topk, self.device,
                                      group)
            except P2PUnavailable as e:  # every GPU of the group takes the same branch
                import sys

                print(f"expert parallelism: peer-memory exchange unavailable ({e}); "
                      "using NCCL all-to-alls", file=sys.stderr)
                self.transport = transport = "nccl"
        if transport == "p2p":
            self.x, self.ids, self.w = self.xc.x, self.xc.ids, self.xc.w
            self.part = torch.empty(0, hidden, dtype=torch.bfloat16, device=self.device)
            return
        self.xc = None
        rb = int(_lib.load().tw_ep_row_bytes(hidden, topk))
        self.row_bytes = rb
        self.send = torch.empty(rows, rb, dtype=torch.uint8, device=self.device)
        self.recv = torch.empty_like(self.send)
        self.x = torch.empty(rows, hidden, dtype=torch.bfloat16, device=self.device)
        self.ids = torch.empty(rows, topk, dtype=torch.int32, device=self.device)
        self.w = torch.empty(rows, topk, dtype=torch.float32, device=self.device)
        self.part = torch.empty(rows, hidden, dtype=torch.bfloat16, device=self.device)
        self.back = torch.empty_like(self.part)

    def static_tensors(self) -> list[torch.Tensor]:
        """The buffers a captured step reads and writes (fixed addresses)."""
        if self.xc is not None:
            return [self.xc.buf, self.ws]
        return [self.send, self.recv, self.x, self.ids, self.w, self.part, self.back, self.ws]

    def close(self) -> None:
        if self.xc is not None:
            self.xc.close()

    def error(self) -> int:
        return self.xc.error() if self.xc is not None else 0

    # ------------------------------------------------------------------ p2p
    def _p2p_dispatch(self, x, topk_w, topk_ids) -> None:
        T, H = x.shape
        if T != self.T or H != self.H or topk_ids.shape != (T, self.K):
            raise ValueError("expert-parallel shapes are fixed at construction")
        _lib.call("tw_ep_p2p_dispatch", x.data_ptr(), topk_w.data_ptr(), topk_ids.data_ptr(), T,
                  self.K, H, self.Eg, self.world, self.rank, C.cast(self.xc.peers, C.c_void_p),
                  torch.cuda.current_stream().cuda_stream)

    def _p2p_routes(self, w1, w2) -> None:
        rows = self.world * self.T
        if isinstance(w1, tuple):  # NVFP4 banks
            (w1p, w1s, w1g), (w2p, w2s, w2g) = w1, w2
            _lib.call("tw_moe_ffn_nvfp4_routes", self.xc.x.data_ptr(), rows, self.H, self.I,
                      w1p.data_ptr(), w1s.data_ptr(), w1g.data_ptr(), w2p.data_ptr(),
                      w2s.data_ptr(), w2g.data_ptr(), ops._GLOBAL_DTYPES[w1g.dtype],
                      w1p.shape[0], self.xc.w.data_ptr(), self.xc.ids.data_ptr(), self.K,
                      self.ws.data_ptr(), self.ws.numel(), torch.cuda.current_stream().cuda_stream)
            return
        _lib.call("tw_moe_ffn_bf16_routes", self.xc.x.data_ptr(), rows, self.H, self.I,
                  w1.data_ptr(), w2.data_ptr(), w1.shape[0], self.xc.w.data_ptr(),
                  self.xc.ids.data_ptr(), self.K, self.ws.data_ptr(), self.ws.numel(),
                  torch.cuda.current_stream().cuda_stream)

    def _p2p_combine(self, topk_ids, out=None, residual=None, residual_out=None, norm_w=None,
                     eps: float = 0.0, h_out=None) -> None:
        ptr = (lambda t: None if t is None else t.data_ptr())
        _lib.call("tw_ep_p2p_combine", self.ws.data_ptr(), self.T, self.K, self.H, self.I,
                  self.Eg, topk_ids.data_ptr(), self.world, self.rank,
                  C.cast(self.xc.peers, C.c_void_p), ptr(residual), ptr(residual_out),
                  ptr(norm_w), float(eps), ptr(h_out), ptr(out),
                  torch.cuda.current_stream().cuda_stream)

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
        if self.xc is not None:
            self._p2p_dispatch(x, topk_w, topk_ids)
            self._p2p_routes(banks[0], banks[1])
            self._p2p_combine(topk_ids, out=out)
            return out
        self._dispatch(x, topk_w, topk_ids)
        w1, w2 = banks
        if isinstance(w1, tuple):
            ops.moe_ffn_nvfp4(self.x, w1, w2, self.w, self.ids, out=self.part, ws=self.ws)
        else:
            ops.moe_ffn_bf16(self.x, w1, w2, self.w, self.ids, out=self.part, ws=self.ws)
        return self._combine(out)

    def forward(self, x: torch.Tensor, topk_w: torch.Tensor, topk_ids: torch.Tensor,
                layer_id: int, cache: OffloadMoeCache, out: torch.Tensor | None,
                residual: torch.Tensor | None = None, residual_out: torch.Tensor | None = None,
                norm_w: torch.Tensor | None = None, eps: float = 0.0,
                h_out: torch.Tensor | None = None) -> torch.Tensor | None:
        """Routed expert output for this GPU's tokens; ``topk_ids`` are global expert ids.
        With ``residual``/``norm_w`` (p2p transport) the combine also forms
        residual_out = bf16(routed + residual) and h_out = RMSNorm(residual_out) * norm_w."""
        T, H = x.shape
        if T != self.T or H != self.H or topk_ids.shape != (T, self.K):
            raise ValueError("expert-parallel shapes are fixed at construction")
        if cache.num_experts != self.Eg:
            raise ValueError("the slot cache must hold this GPU's expert shard")
        if self.xc is not None:
            self._p2p_dispatch(x, topk_w, topk_ids)
            cache.ensure_experts(layer_id, self.xc.ids)
            cache.copy_missing()
            gate_up, down = cache.bank_views()
            self._p2p_routes(gate_up, down)
            self._p2p_combine(topk_ids, out=out, residual=residual, residual_out=residual_out,
                              norm_w=norm_w, eps=eps, h_out=h_out)
            return out
        if residual is not None:
            raise NotImplementedError("the fused residual norm needs the p2p transport")
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

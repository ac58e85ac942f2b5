"""A synthetic MoE decoder stack driven through the slot cache (the benchmark workload).

``MoEDecodeStack`` builds L MoE blocks with random-init weights of a named shape (seeded)
and runs the paging-aware decode step exactly as the reference's layer does it
(backends/freetoken_tideway/freetoken/layers/moe.py:261-330), per layer:

    h       = RMSNorm(x)                         (fused with the previous residual add)
    logits  = h . Wr^T                           (fp32)
    w, ids  = softmax top-k, renormalised        (fused_topk; one launch with the logits)
    ids     -> slot ids in place                 (ensure_experts: device LRU)
    misses  -> slot banks from pinned host banks (copy_missing)
    y       = slot-indirect SwiGLU FFN + combine (_expert_gemm)
    x       = x + y

Every step is fixed-shape and host-sync free, so it is captured once as a CUDA graph and
replayed.  The expert banks live in pinned host memory (the offload tier); the device holds
the slot cache (``slot_fraction`` of all experts) plus the router and norm weights.
"""

from __future__ import annotations

import sys
import time

from dataclasses import dataclass

import torch

from . import ops
from .offload_cache import OffloadMoeCache


@dataclass
class StackConfig:
    name: str
    layers: int
    hidden: int
    experts: int
    topk: int
    inter: int
    slot_fraction: float
    renormalize: bool = True
    eps: float = 1e-6
    seed: int = 1
    weight_std: float = 0.02

    @property
    def slots(self) -> int:
        return max(self.experts, int(round(self.slot_fraction * self.layers * self.experts)))

    @property
    def expert_bytes(self) -> int:
        return 3 * self.hidden * self.inter * 2


# Qwen3-A3B-shaped BF16 MoE stack
QWEN3_A3B = StackConfig("qwen3-a3b-bf16", layers=48, hidden=2048, experts=128, topk=8,
                        inter=768, slot_fraction=0.5, seed=1)
# tiny single layer
TINY = StackConfig("tiny-c1", layers=1, hidden=1024, experts=16, topk=2, inter=512,
                   slot_fraction=1.0, seed=0)


def alloc_host_arena(numel: int, register=None, pinned_alloc=None, retry_s: float = 90.0,
                     pause_s: float = 3.0) -> tuple[torch.Tensor, bool]:
    """One page-locked bf16 host arena of ``numel`` elements for every layer's expert banks;
    returns (arena, registered).  Preferred: pageable memory registered in place (exact
    size).  Right after another process has released tens of GB of page-locked memory,
    registering can fail for a while, so each retry takes a fresh range, for up to
    ``retry_s``; then the arena comes from the pinned allocator (cudaHostAlloc through torch,
    which rounds the size up to a power of two) and ``registered`` is False."""
    register = register or ops.host_register
    pinned_alloc = pinned_alloc or (lambda n: torch.empty(n, dtype=torch.bfloat16,
                                                          pin_memory=True))
    deadline = time.monotonic() + retry_s
    while True:
        arena = torch.empty(numel, dtype=torch.bfloat16)
        try:
            register(arena.data_ptr(), numel * 2)
            return arena, True
        except RuntimeError as e:
            print(f"host bank registration: {e}", file=sys.stderr, flush=True)
        del arena
        if time.monotonic() > deadline:
            break
        time.sleep(pause_s)
    return pinned_alloc(numel), False


class StackWeights:
    """Seeded random-init weights of a stack: norms and routers on the device, expert
    banks in pinned host memory (``host_banks=False`` keeps them on the device).

    With ``shard=(rank, world)`` only the rank's expert shard is generated (experts
    [rank*E/world, (rank+1)*E/world) of every layer); norms and routers are identical on
    every rank."""

    def __init__(self, cfg: StackConfig, device="cuda", host_banks: bool = True,
                 shard: tuple[int, int] = (0, 1)):
        self.cfg = cfg
        self.device = torch.device(device)
        self.rank, self.world = shard
        L, H, E, I = cfg.layers, cfg.hidden, cfg.experts, cfg.inter
        gen = torch.Generator(device=self.device).manual_seed(cfg.seed)
        bf = torch.bfloat16
        self.norm_w = [(1 + 0.1 * torch.randn(H, generator=gen, device=self.device)).to(bf)
                       for _ in range(L)]
        self.router_w = [(cfg.weight_std * torch.randn(E, H, generator=gen, device=self.device)
                          ).to(bf) for _ in range(L)]
        self.final_norm_w = torch.ones(H, dtype=bf, device=self.device)
        # expert banks: generated on the device layer by layer, staged to one page-locked
        # host arena (registered in place, so no power-of-two rounding of pinned blocks)
        self.gate_up: list[torch.Tensor] = []
        self.down: list[torch.Tensor] = []
        E = E // self.world  # experts held by this rank
        self.local_experts = E
        if self.world > 1:
            gen = torch.Generator(device=self.device).manual_seed(cfg.seed + 7919 * (self.rank + 1))
        gu_n, dn_n = E * 2 * I * H, E * H * I
        self._arena = None
        self._registered = False
        # bumped when the host banks stop being readable by the device (release()): a graph
        # captured before that must not replay its miss copies
        self.generation = 0
        if host_banks:
            self._alloc_arena(L * (gu_n + dn_n))
        for l in range(L):
            gu = (cfg.weight_std * torch.randn(E, 2 * I, H, generator=gen, device=self.device)
                  ).to(bf)
            dn = (cfg.weight_std * torch.randn(E, H, I, generator=gen, device=self.device)
                  ).to(bf)
            if host_banks:
                base = l * (gu_n + dn_n)
                gu_h = self._arena[base:base + gu_n].view(E, 2 * I, H)
                dn_h = self._arena[base + gu_n:base + gu_n + dn_n].view(E, H, I)
                gu_h.copy_(gu)
                dn_h.copy_(dn)
                gu, dn = gu_h, dn_h
            self.gate_up.append(gu)
            self.down.append(dn)
        torch.cuda.synchronize(self.device)

    def _alloc_arena(self, numel: int) -> None:
        self._arena, self._registered = alloc_host_arena(numel)

    def release(self) -> None:
        """Unregister the host arena (call before dropping the weights)."""
        if self._arena is not None:
            if self._registered:
                ops.host_unregister(self._arena.data_ptr())
            self._registered = False
            self._arena = None
            self.generation += 1


class MoEDecodeStack:
    """The decode step of a stack.  With sharded weights (``world > 1``) the routed experts run
    expert-parallel (``tideway_b200.ep``): each GPU's slot cache holds its own shard, sized
    min(configured slots, shard size)."""

    def __init__(self, weights: StackWeights, batch: int, resident_seed: int | None = None,
                 fused: bool = True, transport: str = "p2p"):
        """``fused``: combine each layer's FFN with the next residual RMSNorm
        (tw_moe_ffn_bf16_residual_norm); False composes tw_moe_ffn_bf16 and tw_rmsnorm (same
        result, one more launch per layer).  ``transport``: how expert parallelism moves rows
        between GPUs ("p2p": NVLink peer stores from our kernels; "nccl": all-to-alls)."""
        cfg = weights.cfg
        self.fused = fused
        self.cfg, self.B, self.wts = cfg, batch, weights
        self.device = weights.device
        L, H, E, I = cfg.layers, cfg.hidden, cfg.experts, cfg.inter
        El = weights.local_experts
        bf = torch.bfloat16
        self.norm_w, self.router_w = weights.norm_w, weights.router_w
        self.final_norm_w = weights.final_norm_w
        slots = min(cfg.slots, L * El) if weights.world > 1 else cfg.slots
        self.cache = OffloadMoeCache(num_layers=L, num_experts=El, cache_size=slots,
                                     device=self.device)
        self.cache.set_bank_sources({"gate_up": weights.gate_up, "down": weights.down})
        # seeded resident subset: slot_fraction of each layer's experts
        rs = torch.Generator().manual_seed(cfg.seed if resident_seed is None else resident_seed)
        per_layer = min(El, slots // L)
        self.resident = {l: torch.randperm(El, generator=rs)[:per_layer].tolist()
                         for l in range(L)}
        self.ep = None
        if weights.world > 1:
            from .ep import ExpertParallelMoE

            self.ep = ExpertParallelMoE(E, cfg.topk, H, I, batch, self.device,
                                        transport=transport)
        self.cache.seed_resident(self.resident)
        torch.cuda.synchronize(self.device)
        # static step buffers (graph-captured)
        T, K = batch, cfg.topk
        self.x_in = torch.zeros(T, H, dtype=bf, device=self.device)
        self.resid = torch.zeros(T, H, dtype=bf, device=self.device)
        self.h = torch.zeros(T, H, dtype=bf, device=self.device)
        self.y = torch.zeros(T, H, dtype=bf, device=self.device)
        self.out = torch.zeros(T, H, dtype=bf, device=self.device)
        self.logits = torch.zeros(T, E, dtype=torch.float32, device=self.device)
        self.router_arrivals = ops.router_arrivals(self.device)
        self.topk_w = [torch.zeros(T, K, dtype=torch.float32, device=self.device) for _ in range(L)]
        self.topk_ids = [torch.zeros(T, K, dtype=torch.int32, device=self.device) for _ in range(L)]
        self.ws = torch.empty(ops.workspace_bytes(T * K, H, I), dtype=torch.uint8,
                              device=self.device)
        self.graph: torch.cuda.CUDAGraph | None = None
        # fail-closed controller state (cf. src/tideway/offload/paged_decode_graph.py:209-213,
        # :411-422): a failed step is not retried; every later step raises
        self.state, self.failure = "installed", None
        self._signature = None

    # kernels this library launches per decode step (for the launch count claim)
    def launches_per_step(self) -> int:
        if self.ep is not None and self.ep.xc is not None and self.fused:
            # router + top-k, dispatch, ensure, copy, grouping, gather (unless the received
            # rows fit one 16-route tile), FFN, combine + next norm
            gather = 0 if self.ep.world * self.B <= 16 else 1
            return self.cfg.layers * (7 + gather) + 1
        if self.ep is not None:
            return self.cfg.layers * 11 + 1
        if not self.fused:
            # per layer: norm, router + top-k, ensure, copy, grouping, (gather: beyond 16
            # tokens), FFN, combine; then the final norm
            return self.cfg.layers * (7 + (0 if self.B <= 16 else 1)) + 1
        # norm (layer 0), then per layer: router + top-k, ensure + grouping, copy, (gather:
        # only beyond 16 tokens), FFN, combine + next norm
        gather = 0 if self.B <= 16 else 1
        return self.cfg.layers * (5 + gather) + 1

    # ---------------------------------------------------------------- one decode step
    def _layer(self, l: int, first: bool) -> None:
        cfg, c = self.cfg, self.cache
        ep_fused = self.ep is not None and self.ep.xc is not None and self.fused
        if first:
            ops.rmsnorm(self.x_in, self.norm_w[l], cfg.eps, out=self.h)
            self.resid.copy_(self.x_in)
        elif (self.ep is not None and not ep_fused) or not self.fused:
            # resid = bf16(resid + y); h = norm(resid)
            ops.rmsnorm(self.y, self.norm_w[l], cfg.eps, residual=self.resid,
                        residual_out=self.resid, out=self.h)
        # (single GPU: the previous layer's FFN call already left h = norm(resid + y))
        # router projection + softmax top-k: one launch (one thread-block cluster per token)
        ops.router_softmax_topk(self.h, self.router_w[l], cfg.topk, cfg.renormalize,
                                out=(self.topk_w[l], self.topk_ids[l]), logits_out=self.logits,
                                arrivals=self.router_arrivals)
        last = l == cfg.layers - 1
        if ep_fused:  # the combine forms the next residual sum and norm (the final one last)
            self.ep.forward(self.h, self.topk_w[l], self.topk_ids[l], l, c, None,
                            residual=self.resid, residual_out=self.out if last else self.resid,
                            norm_w=self.final_norm_w if last else self.norm_w[l + 1],
                            eps=cfg.eps, h_out=self.h)
            return
        if self.ep is not None:
            self.ep.forward(self.h, self.topk_w[l], self.topk_ids[l], l, c, self.y)
            return
        if self.fused:  # the ensure also groups the routes for the FFN (one launch fewer)
            c.ensure_experts_grouped(l, self.topk_ids[l], self.ws, cfg.hidden, cfg.inter)
        else:
            c.ensure_experts(l, self.topk_ids[l])
        c.copy_missing()
        gate_up, down = c.bank_views()
        if not self.fused:
            ops.moe_ffn_bf16(self.h, gate_up, down, self.topk_w[l], self.topk_ids[l],
                             out=self.y, ws=self.ws)
            return
        # the FFN, its combine fused with the next residual add and norm (the final norm
        # after the last layer, whose residual sum is the step's output)
        ops.moe_ffn_bf16_residual_norm(
            self.h, gate_up, down, self.topk_w[l], self.topk_ids[l], self.resid,
            self.out if last else self.resid,
            self.final_norm_w if last else self.norm_w[l + 1], cfg.eps, self.h, ws=self.ws,
            pregrouped=True)

    def step_eager(self) -> None:
        for l in range(self.cfg.layers):
            self._layer(l, l == 0)
        if (self.ep is not None and self.ep.xc is None) or not self.fused:
            ops.rmsnorm(self.y, self.final_norm_w, self.cfg.eps, residual=self.resid,
                        residual_out=self.out, out=self.h)

    def capture(self, verify: bool = False) -> torch.cuda.CUDAGraph:
        """Capture one decode step (all layers) into a CUDA graph (after one eager warm-up
        step outside the capture, which also pages in the first misses).  ``verify``: check
        that a replay reproduces the eager step byte for byte from the same input (cf. the
        reference's capture-time checks, src/tideway/offload/ffn_front_graph.py:323-350)."""
        self._require_ok()
        # a capture that fails leaves the stack usable eagerly (graph None, state unchanged)
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.step_eager()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step_eager()
        self.graph = g
        self._signature = self._static_signature()
        self.state = "ready"
        if verify:
            x0 = self.x_in.clone()
            self.step_eager()
            want = self.out.clone()
            self.x_in.copy_(x0)
            g.replay()
            torch.cuda.synchronize(self.device)
            if not torch.equal(self.out, want):
                self._fail("captured decode step differs from the eager step")
                raise RuntimeError("captured decode step differs from the eager step")
        return g

    # ---------------------------------------------------------------- fail-closed guards
    def _static_signature(self) -> tuple:
        """Addresses and layouts a captured step bakes in: the cache's banks, tables, ensure
        scratch, statistics and trace ring (``OffloadMoeCache.graph_signature``, host source
        pointers included), the step buffers, every layer's routing outputs, the FFN
        workspace, the expert-parallel buffers, and the host banks' generation (a released
        host arena can no longer be read by the miss copies)."""
        ts = [self.x_in, self.out, self.h, self.y, self.resid, self.logits, self.ws,
              self.router_arrivals,
              *self.topk_w, *self.topk_ids, *self.norm_w, *self.router_w, self.final_norm_w]
        if self.ep is not None:
            ts += self.ep.static_tensors()
        own = tuple((t.data_ptr(), tuple(t.shape), tuple(t.stride()), t.dtype) for t in ts)
        return own + self.cache.graph_signature() + (self.wts.generation,)

    def _fail(self, error) -> None:
        self.state, self.failure = "failed", repr(error)

    def _require_ok(self) -> None:
        if self.state == "failed":
            raise RuntimeError(f"decode stack failed earlier and is not retried: {self.failure}")

    def check(self) -> None:
        """Read the FFN's device error word (synchronises); a set word fails the stack."""
        self._require_ok()
        if self.ep is not None:
            rows = self.ep.world * self.B
            err = ops.workspace_error(self.ep.ws, rows * self.cfg.topk, self.cfg.hidden,
                                      self.cfg.inter) or self.ep.error()
        else:
            err = ops.workspace_error(self.ws, self.B * self.cfg.topk, self.cfg.hidden,
                                      self.cfg.inter)
        if err != 0:
            self._fail(f"expert FFN error word {err}")
            raise RuntimeError(f"expert FFN reported error word {err}")

    def capture_ffn_only(self) -> torch.cuda.CUDAGraph:
        """A graph of just the step's 48 expert-FFN launches, on the slot ids and weights the
        last step routed (the roofline region: the FFN launches back to back)."""
        gate_up, down = self.cache.bank_views()

        def run():
            for l in range(self.cfg.layers):
                if self.ep is not None and self.ep.xc is not None:
                    self.ep._p2p_routes(gate_up, down)  # the received rows, slot ids
                elif self.ep is not None:  # the rows this GPU received, already slot ids
                    ops.moe_ffn_bf16(self.ep.x, gate_up, down, self.ep.w, self.ep.ids,
                                     out=self.ep.part, ws=self.ep.ws)
                else:
                    ops.moe_ffn_bf16(self.h, gate_up, down, self.topk_w[l], self.topk_ids[l],
                                     out=self.y, ws=self.ws)

        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            run()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            run()
        return g

    def step(self) -> None:
        self._require_ok()
        try:
            if self.graph is None:
                self.step_eager()
                return
            if self._static_signature() != self._signature:
                raise RuntimeError("a buffer the captured step reads moved or changed layout")
            self.graph.replay()
        except Exception as e:
            self._fail(e)
            raise

    # ---------------------------------------------------------------- public API
    def decode(self, hidden_host: torch.Tensor, out_host: torch.Tensor) -> torch.Tensor:
        """One decode step from host memory to host memory: H2D of the batch's hidden
        states, the captured step, D2H of the step's output (the residual stream after the
        last MoE layer).  Both host tensors should be pinned."""
        self.x_in.copy_(hidden_host, non_blocking=True)
        self.step()
        out_host.copy_(self.out, non_blocking=True)
        return out_host

    # ---------------------------------------------------------------- accounting
    def unique_experts_per_layer(self) -> list[int]:
        """Distinct slots routed per layer in the last step (counted from the actual ids;
        expert-parallel: the distinct local experts this GPU ran in the last layer's call)."""
        if self.ep is not None:
            ids = self.ep.ids
            return [int(torch.unique(ids[ids >= 0]).numel())] * self.cfg.layers
        return [int(torch.unique(t[t >= 0]).numel()) for t in self.topk_ids]

    def step_weight_bytes(self) -> int:
        """Algorithmic expert-weight + router bytes of the last step."""
        cfg = self.cfg
        u = sum(self.unique_experts_per_layer())
        return u * cfg.expert_bytes + cfg.layers * cfg.experts * cfg.hidden * 2

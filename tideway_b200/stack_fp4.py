"""DeepSeek-V4-Flash-shaped NVFP4 MoE decode stack (the benchmark configuration's FP4 workload).

Per layer, as the reference's DSV4 segmented decode composes it
(src/tideway/offload/ffn_front_graph.py:24-30 and :331-336 for the gate contract,
src/tideway/offload/ffn_back_graph.py:29-37 for the routed + shared merge):

    h       = RMSNorm(x)                             (fused with the previous residual add)
    logits  = h . Wr^T                               (fp32)
    w, ids  = sigmoid group-limited top-k            (8 groups, top-4 groups, top-6, x2.5)
    ids     -> slot ids in place                     (ensure_experts: device LRU)
    misses  -> NVFP4 slot banks from pinned host banks (copy_missing)
    y       = slot-indirect NVFP4 SwiGLU FFN + combine  +  shared expert FFN

Expert weights are ~N(0, 0.02) quantised to NVFP4 (e2m1 codes, e4m3 scale per 16 elements,
fp32 per-tensor scale for gate, up and down separately).  Host memory: one pinned host bank
of ``experts`` routed experts backs every layer (layer l's expert e is pool row e), so a
miss copies a full expert's bytes over the host link while the host holds one layer's worth
of distinct experts instead of all 43 (156 GB).  The shared experts stay on the device.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import nvfp4, ops
from .offload_cache import OffloadMoeCache


@dataclass
class Fp4StackConfig:
    name: str = "dsv4-flash-nvfp4"
    layers: int = 43
    hidden: int = 4096
    experts: int = 256
    topk: int = 6
    inter: int = 2048
    n_group: int = 8
    topk_group: int = 4
    routed_scaling: float = 2.5
    slot_fraction: float = 0.25
    eps: float = 1e-6
    seed: int = 3
    weight_std: float = 0.02

    @property
    def slots(self) -> int:
        return max(self.experts, int(round(self.slot_fraction * self.layers * self.experts)))

    @property
    def expert_bytes(self) -> int:
        """Packed codes + e4m3 scales + fp32 row globals of one expert (gate, up, down)."""
        H, I = self.hidden, self.inter
        return 3 * H * I // 2 + 3 * H * I // 16 + (2 * I + H) * 4


DSV4_FLASH = Fp4StackConfig()

_BANKS = ("gate_up_packed", "gate_up_scale", "gate_up_global", "down_packed", "down_scale",
          "down_global")


def _quantize_experts(n: int, H: int, I: int, std: float, gen: torch.Generator, device):
    """n experts quantised on the device: six tensors [n, ...] in bank order."""
    out = {k: [] for k in _BANKS}
    for _ in range(n):
        w1 = std * torch.randn(2 * I, H, generator=gen, device=device)
        w2 = std * torch.randn(H, I, generator=gen, device=device)
        (p1, s1, g1), (p2, s2, g2) = nvfp4.quantize_expert(w1, w2)
        for k, v in zip(_BANKS, (p1, s1, g1, p2, s2, g2)):
            out[k].append(v)
    return {k: torch.stack(v) for k, v in out.items()}


class Fp4StackWeights:
    def __init__(self, cfg: Fp4StackConfig, device="cuda"):
        self.cfg = cfg
        self.device = dev = torch.device(device)
        L, H, E, I = cfg.layers, cfg.hidden, cfg.experts, cfg.inter
        gen = torch.Generator(device=dev).manual_seed(cfg.seed)
        bf = torch.bfloat16
        self.norm_w = [(1 + 0.1 * torch.randn(H, generator=gen, device=dev)).to(bf)
                       for _ in range(L)]
        self.router_w = [(cfg.weight_std * torch.randn(E, H, generator=gen, device=dev)).to(bf)
                         for _ in range(L)]
        self.final_norm_w = torch.ones(H, dtype=bf, device=dev)
        # shared experts: one per layer, resident on the device ([1, ...] banks per layer)
        sh = _quantize_experts(L, H, I, cfg.weight_std, gen, dev)
        self.shared = [tuple(sh[k][l:l + 1] for k in _BANKS) for l in range(L)]
        # routed experts: one pinned host pool of E experts behind every layer
        pool = _quantize_experts(E, H, I, cfg.weight_std, gen, dev)
        self.host_pool = {}
        for k in _BANKS:
            h = torch.empty(pool[k].shape, dtype=pool[k].dtype).pin_memory()
            h.copy_(pool[k])
            self.host_pool[k] = h
        del pool, sh
        torch.cuda.synchronize(dev)
        torch.cuda.empty_cache()

    def bank_sources(self) -> dict[str, list[torch.Tensor]]:
        return {k: [self.host_pool[k]] * self.cfg.layers for k in _BANKS}


class Fp4DecodeStack:
    """The configs[3] decode step for a fixed batch, captured as one CUDA graph."""

    def __init__(self, weights: Fp4StackWeights, batch: int):
        cfg = weights.cfg
        self.cfg, self.B, self.wts = cfg, batch, weights
        self.device = weights.device
        L, H, E, I, K = cfg.layers, cfg.hidden, cfg.experts, cfg.inter, cfg.topk
        bf = torch.bfloat16
        self.cache = OffloadMoeCache(num_layers=L, num_experts=E, cache_size=cfg.slots,
                                     device=self.device, quant_format="nvfp4")
        self.cache.set_bank_sources(weights.bank_sources())
        rs = torch.Generator().manual_seed(cfg.seed)
        per_layer = min(E, cfg.slots // L)
        self.cache.seed_resident({l: torch.randperm(E, generator=rs)[:per_layer].tolist()
                                  for l in range(L)})
        torch.cuda.synchronize(self.device)
        T = batch
        self.x_in = torch.zeros(T, H, dtype=bf, device=self.device)
        self.resid = torch.zeros_like(self.x_in)
        self.h = torch.zeros_like(self.x_in)
        self.y = torch.zeros_like(self.x_in)
        self.y_sh = torch.zeros_like(self.x_in)
        self.out = torch.zeros_like(self.x_in)
        self.logits = torch.zeros(T, E, dtype=torch.float32, device=self.device)
        self.router_arrivals = ops.router_arrivals(self.device)
        self.topk_w = [torch.zeros(T, K, dtype=torch.float32, device=self.device) for _ in range(L)]
        self.topk_ids = [torch.zeros(T, K, dtype=torch.int32, device=self.device) for _ in range(L)]
        self.sh_w = torch.ones(T, 1, dtype=torch.float32, device=self.device)
        self.sh_ids = torch.zeros(T, 1, dtype=torch.int32, device=self.device)
        self.ws = torch.empty(ops.workspace_bytes(T * K, H, I), dtype=torch.uint8,
                              device=self.device)
        # the shared expert runs on a stream of its own, next to the routed path (its FFN is
        # latency-bound at decode sizes: 64 work items), with a workspace of its own
        self.side = torch.cuda.Stream(self.device)
        self.ws_sh = torch.empty(ops.workspace_bytes(T, H, I), dtype=torch.uint8,
                                 device=self.device)
        self.graph: torch.cuda.CUDAGraph | None = None

    def launches_per_step(self) -> int:
        # rmsnorm, router + top-k, ensure + grouping, copy, routed (gather, FFN, combine),
        # shared (group, gather, FFN, combine), add
        return self.cfg.layers * 12 + 1

    def check(self) -> None:
        """Read the routed and shared FFNs' device error words (synchronises); raises when a
        bounded wait inside an FFN launch gave up."""
        cfg = self.cfg
        err = (ops.workspace_error(self.ws, self.B * cfg.topk, cfg.hidden, cfg.inter) or
               ops.workspace_error(self.ws_sh, self.B, cfg.hidden, cfg.inter))
        if err != 0:
            raise RuntimeError(f"NVFP4 expert FFN reported error word {err}")

    def _ffn_routed(self, l: int, pregrouped: bool = False) -> None:
        gp, gs, gg, dp, ds, dg = self.cache.bank_views()
        ops.moe_ffn_nvfp4(self.h, (gp, gs, gg), (dp, ds, dg), self.topk_w[l], self.topk_ids[l],
                          out=self.y, ws=self.ws, pregrouped=pregrouped)

    def _layer(self, l: int, first: bool) -> None:
        cfg, c = self.cfg, self.cache
        if first:
            ops.rmsnorm(self.x_in, self.wts.norm_w[l], cfg.eps, out=self.h)
            self.resid.copy_(self.x_in)
        else:
            ops.rmsnorm(self.y, self.wts.norm_w[l], cfg.eps, residual=self.resid,
                        residual_out=self.resid, out=self.h)
        # router projection + sigmoid group top-k: one launch
        ops.router_sigmoid_group_topk(self.h, self.wts.router_w[l], cfg.topk, cfg.n_group,
                                      cfg.topk_group, cfg.routed_scaling, True,
                                      out=(self.topk_w[l], self.topk_ids[l]),
                                      logits_out=self.logits, arrivals=self.router_arrivals)
        # the shared expert's FFN on the side stream, concurrent with the routed path
        main = torch.cuda.current_stream(self.device)
        self.side.wait_stream(main)
        with torch.cuda.stream(self.side):
            sp, ss, sg, tp, ts, tg = self.wts.shared[l]
            ops.moe_ffn_nvfp4(self.h, (sp, ss, sg), (tp, ts, tg), self.sh_w, self.sh_ids,
                              out=self.y_sh, ws=self.ws_sh)
        # the ensure also groups the routes for the routed FFN (one launch fewer)
        c.ensure_experts_grouped(l, self.topk_ids[l], self.ws, cfg.hidden, cfg.inter)
        c.copy_missing()
        self._ffn_routed(l, pregrouped=True)
        main.wait_stream(self.side)
        ops.add_shared(self.y, self.y_sh, out=self.y)

    def step_eager(self) -> None:
        for l in range(self.cfg.layers):
            self._layer(l, l == 0)
        ops.rmsnorm(self.y, self.wts.final_norm_w, self.cfg.eps, residual=self.resid,
                    residual_out=self.out, out=self.h)

    def _capture(self, fn) -> torch.cuda.CUDAGraph:
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        return g

    def capture(self) -> torch.cuda.CUDAGraph:
        self.graph = self._capture(self.step_eager)
        return self.graph

    def capture_ffn_only(self) -> torch.cuda.CUDAGraph:
        """The step's routed NVFP4 FFN launches back to back, on the last step's slot ids."""
        return self._capture(lambda: [self._ffn_routed(l) for l in range(self.cfg.layers)])

    def step(self) -> None:
        if self.graph is None:
            self.step_eager()
        else:
            self.graph.replay()

    def decode(self, hidden_host: torch.Tensor, out_host: torch.Tensor) -> torch.Tensor:
        self.x_in.copy_(hidden_host, non_blocking=True)
        self.step()
        out_host.copy_(self.out, non_blocking=True)
        return out_host

    def unique_experts_per_layer(self) -> list[int]:
        return [int(torch.unique(t[t >= 0]).numel()) for t in self.topk_ids]

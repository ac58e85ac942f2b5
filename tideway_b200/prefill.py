"""Gemma-shaped MoE prefill stack (the benchmark configuration's prefill workload).

Per layer, as the reference's Gemma decode/prefill blocks compose the MoE operators
(src/tideway/gemma_router_norm_pair.py, src/tideway/gemma_route_copy_kernel.py,
src/tideway/overlap_shared_expert.py:229-294):

    router_in, routed_in, shared_in = router_norm_triple(x)   (one RMSNorm reduction)
    w, ids               = gemma_topk(router_in . Wr^T, per_expert_scale)
    shared               = SwiGLU_shared(shared_in)     (always-active expert, dense FFN)
    routed               = routed experts(routed_in, w, ids)
    x                    = (x + N(N1(shared) + N2(routed))) * scalar   (combine fused in)

All 30 layers' experts live in HBM (46.7 GB at the configured shape): on B200 the two-layer
streaming window of the reference's consumer-GPU setting would only add host-link traffic,
so every layer's experts are resident when its FFN runs (expert id == bank row).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops


@dataclass
class PrefillConfig:
    name: str = "gemma-a4b-bf16-prefill"
    layers: int = 30
    hidden: int = 2816
    experts: int = 128
    topk: int = 8
    inter: int = 704
    shared_inter: int = 2112
    tokens: int = 2048
    eps: float = 1e-6
    seed: int = 2
    weight_std: float = 0.02
    layer_scalar: float = 1.0
    # gate activation of every expert: SwiGLU as the benchmark configuration names it;
    # Gemma 4 checkpoints use "gelu_tanh"
    activation: str = "silu"

    def routed_flops(self) -> float:
        return 6.0 * self.hidden * self.inter * self.tokens * self.topk

    def shared_flops(self) -> float:
        return 6.0 * self.hidden * self.shared_inter * self.tokens

    def router_flops(self) -> float:
        return 2.0 * self.tokens * self.hidden * self.experts


C3 = PrefillConfig()


class GemmaPrefillStack:
    def __init__(self, cfg: PrefillConfig, device="cuda"):
        self.cfg = cfg
        self.device = dev = torch.device(device)
        L, H, E, I, Is, T = (cfg.layers, cfg.hidden, cfg.experts, cfg.inter, cfg.shared_inter,
                             cfg.tokens)
        bf = torch.bfloat16
        g = torch.Generator(device=dev).manual_seed(cfg.seed)

        def rnd(*shape, std=cfg.weight_std):
            return (std * torch.randn(*shape, generator=g, device=dev)).to(bf)

        def norm_w():
            return (1 + 0.1 * torch.randn(H, generator=g, device=dev)).to(bf)

        self.layers = []
        for _ in range(L):
            self.layers.append(dict(
                router=rnd(E, H), router_scale=norm_w(), ones=torch.ones(H, dtype=bf, device=dev),
                expert_scale=(1 + 0.1 * torch.randn(E, generator=g, device=dev)).float(),
                pre_shared=norm_w(), pre_routed=norm_w(), post_shared=norm_w(),
                post_routed=norm_w(), post=norm_w(),
                sh_w1=rnd(1, 2 * Is, H), sh_w2=rnd(1, H, Is),
                w1=rnd(E, 2 * I, H), w2=rnd(E, H, I)))
        self.x = torch.zeros(T, H, dtype=bf, device=dev)
        self.router_in = torch.empty_like(self.x)
        self.routed_in = torch.empty_like(self.x)
        self.shared_in = torch.empty_like(self.x)
        self.shared = torch.empty_like(self.x)
        self.routed = torch.empty_like(self.x)
        self.logits = torch.empty(T, E, dtype=torch.float32, device=dev)
        self.w = torch.empty(T, cfg.topk, dtype=torch.float32, device=dev)
        self.ids = torch.empty(T, cfg.topk, dtype=torch.int32, device=dev)
        self.priv = torch.empty(T, cfg.topk, dtype=torch.int32, device=dev)
        self.ws = torch.empty(ops.workspace_bytes(T * cfg.topk, H, max(I, Is)),
                              dtype=torch.uint8, device=dev)
        self.root = H ** -0.5
        self.graph = None

    def layer(self, p: dict, routed_only: bool = False) -> None:
        cfg = self.cfg
        if not routed_only:
            # the router pair and the shared expert's pre-norm share one reduction of x
            ops.router_norm_triple(self.x, p["ones"], p["pre_routed"], p["router_scale"],
                                   p["pre_shared"], cfg.eps, self.root,
                                   out=(self.router_in, self.routed_in, self.shared_in))
            ops.router_logits(self.router_in, p["router"], out=self.logits)
            ops.gemma_topk(self.logits, p["expert_scale"], cfg.topk,
                           out=(self.w, self.ids, self.priv))
            # the always-active shared expert: a dense FFN over every token
            ops.ffn_dense_bf16(self.shared_in, p["sh_w1"], p["sh_w2"], out=self.shared,
                               ws=self.ws, activation=cfg.activation)
        if routed_only:
            ops.moe_ffn_bf16(self.routed_in, p["w1"], p["w2"], self.w, self.ids,
                             out=self.routed, ws=self.ws, activation=cfg.activation)
        else:
            # the routed experts, their combine fused into the shared/routed merge
            ops.moe_ffn_bf16_dual_merge(self.routed_in, p["w1"], p["w2"], self.w, self.ids,
                                        self.shared, self.x, p["post_shared"], p["post_routed"],
                                        p["post"], cfg.eps, cfg.eps, cfg.eps, cfg.layer_scalar,
                                        out=self.x, ws=self.ws, activation=cfg.activation)

    def step_eager(self) -> None:
        for p in self.layers:
            self.layer(p)

    def capture(self) -> torch.cuda.CUDAGraph:
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
        return g

    def capture_routed_only(self) -> torch.cuda.CUDAGraph:
        """The step's routed-expert launches back to back (on the last step's routing)."""
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for p in self.layers:
                self.layer(p, routed_only=True)
        return g

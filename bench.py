"""Benchmark: MoE decode tokens/s and expert-weight HBM GB/s on B200.

Workload: Qwen3-A3B-shaped BF16 MoE stack, 48 layers,
hidden 2048, 128 routed experts, top-8 softmax with renormalised weights, SwiGLU
intermediate 768, weights ~N(0, 0.02) (seed 1), hidden states ~N(0, 1), slot cache of 50%
of all experts (3072 slots) seeded with a random 50% of each layer's experts, expert banks
in pinned host memory.  One step = one decode step of the whole stack for a fixed batch:
per layer RMSNorm -> router GEMM -> softmax top-k -> device LRU ensure (in-place slot
rewrite) -> miss copy from the host banks -> slot-indirect SwiGLU FFN + combine ->
residual add.  The step is one captured CUDA graph.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--sweep]
    python bench.py --impl reference ...     # the reference path on the host cores

Under torchrun (N > 1) the routed experts run expert-parallel: GPU r holds experts
[r*E/N, (r+1)*E/N) of every layer in its own slot cache, each GPU decodes its own batch of B
tokens (weak scaling) and every layer exchanges token rows and partial outputs with NCCL
all-to-alls; value = N * B / step time, the step time being the max over ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MoE decode tokens/s + expert-weight HBM GB/s vs peak at 1/2/4/8 B200"
WORKLOAD = "configs[1] Qwen3-A3B-shaped BF16 MoE stack, {layers} layers, decode"
PREFILL_METRIC = "MoE prefill tokens/s + routed-expert tensor-pipe utilisation (configs[2])"
C4_METRIC = "MoE decode tokens/s + expert-weight HBM GB/s (configs[3], NVFP4)"
FP4_DTYPE = "nvfp4 weights, f16 x f16 -> f32 tensor-core MMAs"


def c2_config(cfg, B: int, world: int) -> dict:
    """configs[1] config dict, printed identically by both arms."""
    return {"workload": WORKLOAD.format(layers=cfg.layers), "batch": B, "global_batch": B * world,
            "layers": cfg.layers, "hidden": cfg.hidden, "experts": cfg.experts,
            "topk": cfg.topk, "intermediate": cfg.inter, "slots": cfg.slots,
            "parallelism": f"ep{world}" if world > 1 else "single",
            "inputs": "seeded N(0,1) hidden states, distinct on every GPU",
            "l2": "inputs larger than L2 (expert weights streamed per step)"}


def prefill_config(cfg) -> dict:
    return {"workload": f"configs[2] Gemma-A4B-shaped BF16 MoE prefill, {cfg.layers} layers",
            "tokens": cfg.tokens, "hidden": cfg.hidden, "experts": cfg.experts,
            "topk": cfg.topk, "intermediate": cfg.inter, "shared_intermediate": cfg.shared_inter,
            "parallelism": "single",
            "l2": "inputs larger than L2 (1.52 GB of routed experts per layer)"}


def c4_config(cfg, B: int) -> dict:
    return {"workload": f"configs[3] DeepSeek-V4-Flash-shaped NVFP4 MoE decode, "
                        f"{cfg.layers} layers", "batch": B, "hidden": cfg.hidden,
            "experts": cfg.experts, "topk": cfg.topk, "intermediate": cfg.inter,
            "groups": [cfg.n_group, cfg.topk_group], "slots": cfg.slots,
            "parallelism": "single",
            "host_banks": "one pinned pool of 256 NVFP4 experts backs every layer",
            "l2": "inputs larger than L2 (expert weights streamed from HBM)"}


def c5_metric(prefill: bool) -> str:
    return f"expert-parallel MoE layer tokens/s (configs[4], {'prefill' if prefill else 'decode'})"


def c5_config(cfg, prefill: bool, world: int) -> dict:
    T_total = 8192 if prefill else 256
    return {"workload": f"configs[4]: one configs[3]-shaped NVFP4 MoE layer, experts "
                        f"sharded {cfg.experts // world} per GPU, {T_total} tokens "
                        f"({'prefill' if prefill else 'decode'}) split over {world} GPUs",
            "tokens_per_gpu": T_total // world, "hidden": cfg.hidden, "experts": cfg.experts,
            "topk": cfg.topk, "intermediate": cfg.inter, "parallelism": f"ep{world}",
            "routing": "sigmoid group top-k (8 groups, top-4, top-6, x2.5) with a selection "
                       "bias fitted so that route shares follow Zipf(1.2) over a seeded "
                       "popularity order (capped at 1/6: distinct top-6)"}


C5_MODES = {"c5-ep": [False, True], "c5-ep-decode": [False], "c5-ep-prefill": [True]}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--sweep", action="store_true", help="(default on one GPU) other batches")
    ap.add_argument("--no-sweep", action="store_true",
                    help="skip the batch sweep and the paging record (one GPU)")
    ap.add_argument("--sweep-batches", default="1,8,32,64")
    ap.add_argument("--impl", default="tideway", choices=["tideway", "reference"])
    ap.add_argument("--layers", type=int, default=None, help="override layer count (profiling)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="c2-decode",
                    choices=["c2-decode", "c3-prefill", "c4-decode", "c5-ep", "c5-ep-decode",
                             "c5-ep-prefill"],
                    help="c2-decode (the headline) or c3-prefill (configs[2])")
    ap.add_argument("--ep-transport", default="p2p", choices=["p2p", "nccl"],
                    help="expert-parallel row exchange: NVLink peer stores from our kernels "
                         "(p2p) or NCCL all-to-alls")
    ap.add_argument("--ffn-only", action="store_true",
                    help="after set-up, only replay the graph of the step's FFN launches "
                         "(the target for ncu captures of the FFN kernel)")
    return ap.parse_args()


def traffic_per_launch(alg_bytes: float):
    """DRAM bytes per FFN launch: the ratio dram_bytes / algorithmic_bytes measured by ncu on
    the FFN kernel (profiles/expert_ffn_traffic.json) scaled to this launch's algorithmic
    bytes; None when no capture has been summarised."""
    p = ROOT / "profiles" / "expert_ffn_traffic.json"
    if not p.exists():
        return None
    return json.loads(p.read_text())["dram_over_algorithmic"] * alg_bytes


def prefill_traffic():
    """DRAM bytes of one configs[2] routed FFN kernel launch as ncu measured it
    (profiles/prefill_ffn_traffic.json: the same per-layer shape the bench runs); None when
    no capture has been summarised."""
    p = ROOT / "profiles" / "prefill_ffn_traffic.json"
    if not p.exists():
        return None
    return float(json.loads(p.read_text())["dram_bytes_per_launch"])


def grouping_launches(n_routes: int, num_slots: int) -> int:
    """Kernels the FFN's route grouping launches: two (count, then place) for >= 1024 routes
    over <= 1024 slots whose per-slice counts fit shared memory, else one -- the condition
    run_ffn applies (tideway_b200/csrc/moe_ffn.cu)."""
    slices = (n_routes + 127) // 128
    two_pass = n_routes >= 1024 and num_slots <= 1024 and slices * num_slots <= 48 * 1024
    return 2 if two_pass else 1


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


# ---------------------------------------------------------------- clocks

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        try:
            lines = Path(self.path).read_text().strip().splitlines()
        except OSError:
            lines = []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- distributed

def dist_setup():
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- CPU reference path

def _cpu_layer_inputs(cfg, B: int, seed: int):
    """One layer's synthetic inputs for the host-core path (same shapes and distributions)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    H, E, I = cfg.hidden, cfg.experts, cfg.inter
    x = torch.randn(B, H, generator=g).to(torch.bfloat16)
    norm_w = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
    router = (cfg.weight_std * torch.randn(E, H, generator=g)).to(torch.bfloat16)
    gate_up = (cfg.weight_std * torch.randn(E, 2 * I, H, generator=g)).to(torch.bfloat16)
    down = (cfg.weight_std * torch.randn(E, H, I, generator=g)).to(torch.bfloat16)
    return x, norm_w, router, gate_up, down


def cpu_layer_step(cfg, x, norm_w, router, gate_up, down, table, layer):
    """One MoE layer of the decode step on the host cores: the oracle restatement of the
    reference path (norm, router, fused_topk, slot LRU, slot-indirect FFN, combine)."""
    import torch

    from oracle import ffn as off
    from oracle import routing as orouting
    from oracle import slot_cache as osc

    h = off.rmsnorm(x, norm_w, cfg.eps)
    logits = h.float() @ router.float().t()
    w, ids = orouting.softmax_topk(logits, cfg.topk, cfg.renormalize)
    slots = osc.lru_ensure(table, ids.numpy(), layer)
    # slot s holds expert id_of_slot[s] - layer*E: the FFN reads the experts through it
    expert_of = torch.from_numpy(table.id_of_slot.astype("int64") - layer * cfg.experts)
    eids = expert_of[torch.from_numpy(slots).long()].to(torch.int32)
    y = off.moe_decode(h, gate_up, down, w, eids)
    return (x.float() + y.float()).to(torch.bfloat16)


def cpu_c2_layer(cfg, B: int, seed: int = 1):
    """Host-core path of one configs[1] layer at batch B (the oracle restatement of the
    reference path): inputs and one layer's 128 experts drawn once, a slot table that keeps
    them resident (the GPU run's steady state has no misses either).  Returns a callable that
    runs the layer once and returns its seconds."""
    import torch

    from oracle import slot_cache as osc

    torch.set_num_threads(os.cpu_count() or 1)
    x, norm_w, router, gate_up, down = _cpu_layer_inputs(cfg, B, seed)
    table = osc.SlotTable(1, cfg.experts, cfg.slots)
    state = {"x": x}

    def layer() -> float:
        t0 = time.perf_counter()
        state["x"] = cpu_layer_step(cfg, state["x"], norm_w, router, gate_up, down, table, 0)
        return time.perf_counter() - t0

    return layer


def cpu_c2_timed(cfg, B: int, warmup: int, steps: int) -> tuple[float, int]:
    """Mean seconds per layer over ``steps`` timed samples after ``warmup`` untimed ones (the
    protocol of both the reference arm and the cpu_baseline leg); returns (sec, threads)."""
    import torch

    layer = cpu_c2_layer(cfg, B)
    per = [layer() for _ in range(warmup + steps)][warmup:]
    return statistics.mean(per), torch.get_num_threads()


def cpu_c2_baseline(cfg, B: int, sec: float, cores: int, warmup: int, steps: int) -> dict:
    return {"value": B / (sec * cfg.layers), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"1 of {cfg.layers} layers at batch {B} (norm, router, softmax top-k, "
                      f"slot LRU, expert FFN, combine: the oracle restatement of the reference "
                      f"path) on {cores} host threads, mean of {steps} samples after {warmup} "
                      f"warm-up, scaled x{cfg.layers}"}


def _reference_line(args, world: int, metric: str, value: float, ms: float, scaling: str,
                    dtype: str, config: dict, cpu: dict) -> None:
    """The reference arm's JSON line: the host-core port of the path, timed on the same
    workload as the tideway arm (its cpu_baseline describes the run; e2e = value)."""
    print(json.dumps({
        "impl": "reference", "metric": metric, "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": dtype,
        "data": "synthetic", "config": config, "cpu_baseline": cpu,
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }))


def run_reference_other(args, world: int) -> None:
    """Reference arm of configs[2], configs[3] and configs[4]: the same host-core port as
    their cpu_baseline, W untimed + K timed samples, the mean of the timed ones."""
    import torch

    if args.workload == "c3-prefill":
        from tideway_b200.prefill import C3 as cfg

        layer = cpu_prefill_layer(cfg, cfg.seed + 7)
        per = [layer() for _ in range(args.warmup + args.steps)][args.warmup:]
        sec = statistics.mean(per)
        cpu = cpu_prefill_baseline(cfg, sec, torch.get_num_threads())
        _reference_line(args, world, PREFILL_METRIC, cpu["value"], sec * cfg.layers * 1e3,
                        "weak", "bf16", prefill_config(cfg), cpu)
        return
    from tideway_b200.stack_fp4 import DSV4_FLASH as cfg

    if args.workload == "c4-decode":
        B = args.batch
        layer = cpu_fp4_decode_layer(cfg, B, cfg.seed + 7)
        per = [layer() for _ in range(args.warmup + args.steps)][args.warmup:]
        sec = statistics.mean(r[0] for r in per)
        cpu = cpu_fp4_decode_baseline(cfg, B, sec, per[-1][1], torch.get_num_threads())
        _reference_line(args, world, C4_METRIC, cpu["value"], sec * cfg.layers * 1e3, "weak",
                        FP4_DTYPE, c4_config(cfg, B), cpu)
        return
    for prefill in C5_MODES[args.workload]:
        Ts = c5_cpu_sample(prefill)
        layer = cpu_ep_layer(cfg, Ts, 4 + 7)
        per = [layer() for _ in range(args.warmup + args.steps)][args.warmup:]
        sec = statistics.mean(r[0] for r in per)
        cpu = cpu_ep_baseline(Ts, sec, per[-1][1], torch.get_num_threads(), prefill)
        T_total = 8192 if prefill else 256
        _reference_line(args, world, c5_metric(prefill), cpu["value"],
                        T_total / cpu["value"] * 1e3, "strong", FP4_DTYPE,
                        c5_config(cfg, prefill, world), cpu)


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.workload != "c2-decode":
        return run_reference_other(args, world)
    from tideway_b200.stack import QWEN3_A3B as cfg

    B = args.batch
    # the whole job's tokens: every GPU of the tideway arm decodes its own batch of B
    sec_layer, cores = cpu_c2_timed(cfg, B * world, args.warmup, args.steps)
    cpu = cpu_c2_baseline(cfg, B * world, sec_layer, cores, args.warmup, args.steps)
    _reference_line(args, world, METRIC, cpu["value"], sec_layer * cfg.layers * 1e3,
                    "weak", "bf16", c2_config(cfg, B, world), cpu)


# ---------------------------------------------------------------- GPU path

def _events():
    import torch

    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def _time_replays(fn, n: int) -> float:
    """Mean ms of ``fn()`` over n calls, CUDA events on the current stream."""
    import torch

    st = torch.cuda.current_stream()
    a, b = _events()
    a.record(st)
    for _ in range(n):
        fn()
    b.record(st)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / n


def gather_floats(vals: list[float], world: int) -> list[list[float]]:
    """Every rank's ``vals`` (same length on all ranks), rank order."""
    if world == 1:
        return [list(vals)]
    import torch
    import torch.distributed as dist

    t = torch.tensor(vals, dtype=torch.float64, device="cuda")
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [o.tolist() for o in out]


def ep_parity(stack, weights, world: int, rank: int, layer: int = 0) -> dict:
    """Outside the timed region: one layer's expert-parallel output on fresh rank-distinct
    tokens against the same layer run through the 1-GPU FFN entry over the whole layer's
    experts (every rank's shard gathered), max over ranks of max|ep - ref| / max|ref|."""
    import torch
    import torch.distributed as dist

    from tideway_b200 import ops

    cfg, dev = weights.cfg, weights.device
    B = stack.B
    g = torch.Generator(device=dev).manual_seed(cfg.seed + 4242 + 7919 * rank)
    x = torch.randn(B, cfg.hidden, generator=g, device=dev).to(torch.bfloat16)
    logits = ops.router_logits(x, stack.router_w[layer])
    w, ids = ops.softmax_topk(logits, cfg.topk, cfg.renormalize)
    y_ep = torch.empty_like(x)
    stack.ep.forward(x, w, ids.clone(), layer, stack.cache, y_ep)
    full = []
    for bank in (weights.gate_up[layer], weights.down[layer]):
        mine = bank.to(dev)
        parts = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine)
        full.append(torch.cat(parts))
    ref = ops.moe_ffn_bf16(x, full[0], full[1], w, ids)
    err = float((y_ep.float() - ref.float()).abs().max() / ref.float().abs().max())
    err = max_over_ranks(err, world)
    del full
    torch.cuda.empty_cache()
    return {"layer": layer, "max_rel": err, "tolerance": 2e-2, "ok": err <= 2e-2,
            "against": "1-GPU slot-indirect FFN over the gathered expert shards"}


def copy_rows_gbs(stack, rows: int = 32) -> float:
    """Host-link GB/s of the miss copy: ``rows`` whole experts from the pinned host banks into
    slot rows [0, rows) through the step's own copy kernel (device-side count), CUDA events.
    Leaves those slots holding other experts than the tables say: run last on a stack."""
    import torch

    from tideway_b200 import ops

    c = stack.cache
    n = min(rows, c.num_experts, c.cache_size)
    idx = torch.arange(n, dtype=torch.int32, device=c.device)
    num = torch.tensor([n], dtype=torch.int64, device=c.device)
    plan = c._copy_plans[0]
    ops.copy_rows(plan, idx, idx, num, n)
    torch.cuda.synchronize()
    ms = _time_replays(lambda: ops.copy_rows(plan, idx, idx, num, n), 3)
    return n * stack.cfg.expert_bytes / (ms * 1e-3) / 1e9


def run_batch(weights, B: int, steps: int, warmup: int, world: int, rank: int, clock_idx: int,
              e2e: bool, ffn_only: bool = False, sustained: bool = False,
              parity: bool = False, transport: str = "p2p") -> dict:
    import torch

    from tideway_b200.stack import MoEDecodeStack

    cfg = weights.cfg
    stack = MoEDecodeStack(weights, B, transport=transport)
    # every GPU decodes its own tokens (weak scaling): the seed includes the rank
    g = torch.Generator().manual_seed(cfg.seed + 1000 + B + 7919 * rank)
    x_host = torch.randn(B, cfg.hidden, generator=g).to(torch.bfloat16).pin_memory()
    out_host = torch.empty(B, cfg.hidden, dtype=torch.bfloat16).pin_memory()
    stack.x_in.copy_(x_host)
    try:
        stack.capture()
    except Exception as e:  # collectives that refuse capture: replay the step eagerly
        torch.cuda.synchronize()
        stack.graph = None
        print(f"[bench] step not captured ({type(e).__name__}: {e}); running eagerly",
              file=sys.stderr)
    for _ in range(warmup):
        stack.step()
    torch.cuda.synchronize()
    if ffn_only:  # profiling target: nothing but the FFN launches of a routed step
        g = stack.capture_ffn_only()
        for _ in range(steps):
            g.replay()
        torch.cuda.synchronize()
        return {"B": B, "uniq": stack.unique_experts_per_layer()}

    st = torch.cuda.current_stream()
    e0, e1 = _events()
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(clock_idx) as clk:
        e0.record(st)
        for _ in range(steps):
            stack.step()
        e1.record(st)
        torch.cuda.synchronize()
    barrier(world)
    stack.check()  # a bounded wait that gave up would void the timed steps
    ms = e0.elapsed_time(e1) / steps
    ms = max_over_ranks(ms, world)
    res = {"B": B, "ms_per_step": ms, "tokens_per_s": B / (ms * 1e-3), "clocks": clk.summary(),
           "launches": stack.launches_per_step() * steps}
    if sustained:
        # the same replays for at least a second, clocks sampled throughout (the step count
        # comes from the max-over-ranks step time, so every rank runs the same number)
        n_long = max(steps, int(1.2 / (ms * 1e-3)) + 1)
        barrier(world)
        torch.cuda.synchronize()
        with ClockSampler(clock_idx) as clk2:
            e0.record(st)
            for _ in range(n_long):
                stack.step()
            e1.record(st)
            torch.cuda.synchronize()
        barrier(world)
        lms = max_over_ranks(e0.elapsed_time(e1) / n_long, world)
        res["sustained"] = {"steps": n_long, "ms_per_step": lms,
                            "tokens_per_s": world * B / (lms * 1e-3), "clocks": clk2.summary()}

    # roofline region: the step's FFN launches replayed back to back from their own graph,
    # timed with CUDA events on the launching stream
    ffn_graph = stack.capture_ffn_only()
    ffn_graph.replay()
    torch.cuda.synchronize()
    ffn_total_ms = _time_replays(ffn_graph.replay, max(steps, 3))
    uniq = stack.unique_experts_per_layer()
    ffn_bytes = [u * cfg.expert_bytes + 2 * B * cfg.hidden * 2 for u in uniq]
    ffn_gbs = sum(ffn_bytes) / (ffn_total_ms * 1e-3) / 1e9
    step_bytes = stack.step_weight_bytes()
    res.update({"ffn_ms_per_step": ffn_total_ms, "ffn_gbs": ffn_gbs,
                "ffn_bytes_per_launch": sum(ffn_bytes) / len(ffn_bytes),
                "ffn_ms_per_launch": ffn_total_ms / cfg.layers,
                "expert_weight_gbs_step": step_bytes / (ms * 1e-3) / 1e9,
                "unique_experts_per_layer": sum(uniq) / len(uniq)})
    if world > 1:
        # per GPU: distinct local experts, FFN GB/s, and the row exchange of a layer (the two
        # NCCL all-to-alls, or the p2p dispatch + combine launches), every GPU in step
        ep = stack.ep
        if ep.xc is not None:
            def exchange():
                ep._p2p_dispatch(stack.h, stack.topk_w[0], stack.topk_ids[0])
                ep._p2p_combine(stack.topk_ids[0], out=stack.y)

            exchange()
            torch.cuda.synchronize()
            barrier(world)
            ex_us = _time_replays(exchange, max(steps, 20)) * 1e3
        else:
            torch.cuda.synchronize()
            barrier(world)
            ex_us = 2 * _time_replays(lambda: ep._a2a(ep.recv, ep.send), max(steps, 20)) * 1e3
        rows = gather_floats([sum(uniq) / len(uniq), ffn_gbs, ex_us], world)
        res["per_gpu"] = [{"rank": r, "distinct_experts_per_layer": v[0], "ffn_gbs": v[1],
                           "exchange_us_per_layer": v[2]} for r, v in enumerate(rows)]
    # misses in the steady state: one more step with the LRU statistics on
    stack.cache.collect_stats = True
    stack.cache.reset_stats()
    stack.step_eager()
    torch.cuda.synchronize()
    miss = stack.cache.decode_miss_stats()
    stack.cache.collect_stats = False
    res["misses_per_layer"] = miss["missing_per_layer"]
    res["paged_bytes_per_step"] = miss["missing_per_layer"] * cfg.layers * cfg.expert_bytes
    if e2e:
        torch.cuda.synchronize()
        a, b = _events()
        a.record(st)
        for _ in range(steps):
            stack.decode(x_host, out_host)
        b.record(st)
        torch.cuda.synchronize()
        ems = max_over_ranks(a.elapsed_time(b) / steps, world)
        res["e2e_ms_per_step"] = ems
        res["e2e_tokens_per_s"] = B / (ems * 1e-3)
        res["h2d"] = B * cfg.hidden * 2
        res["d2h"] = B * cfg.hidden * 2
    if parity and stack.ep is not None:
        res["parity"] = ep_parity(stack, weights, world, rank)
    if stack.ep is not None:
        res["transport"] = stack.ep.transport
        res["ep_error_word"] = max_over_ranks(float(stack.ep.error()), world)
        torch.cuda.synchronize()
        barrier(world)  # every GPU is done with the peers' exchange buffers
        stack.ep.close()
    del stack, ffn_graph
    torch.cuda.empty_cache()
    return res


def run_paging(weights, B: int, steps: int, warmup: int, pool: int = 16) -> dict:
    """Paging record (one GPU): every step decodes a fresh batch drawn from a pool of
    pre-generated device batches, so routing changes and the misses are real; the misses are
    counted by the LRU kernel and copied over the host link inside the captured step."""
    import torch

    from tideway_b200.stack import MoEDecodeStack

    cfg = weights.cfg
    stack = MoEDecodeStack(weights, B)
    g = torch.Generator(device=weights.device).manual_seed(cfg.seed + 5000 + B)
    xs = torch.randn(pool, B, cfg.hidden, generator=g, device=weights.device).to(torch.bfloat16)
    stack.cache.collect_stats = True  # the captured ensures count hits and misses
    stack.x_in.copy_(xs[0])
    stack.capture()
    it = [0]

    def step():
        it[0] += 1
        stack.x_in.copy_(xs[it[0] % pool])
        stack.step()

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    stack.cache.reset_stats()
    ms = _time_replays(step, steps)
    miss = stack.cache.decode_miss_stats()
    paged = miss["missing_per_layer"] * cfg.layers * cfg.expert_bytes
    out = {"B": B, "steps": steps, "ms_per_step": ms, "tokens_per_s": B / (ms * 1e-3),
           "misses_per_layer": miss["missing_per_layer"],
           "hit_rate": 1.0 - miss["miss_rate"], "paged_bytes_per_step": paged,
           "paged_gbs": paged / (ms * 1e-3) / 1e9,
           "copy_rows_gbs": copy_rows_gbs(stack),
           "inputs": f"a fresh batch each step from a pool of {pool} seeded batches"}
    del stack
    torch.cuda.empty_cache()
    return out


def run_prefill(args) -> None:
    """Gemma-A4B-shaped prefill, 30 layers, 2048 tokens, all experts resident."""
    import torch

    import tideway_b200
    from tideway_b200.prefill import C3, GemmaPrefillStack, PrefillConfig

    world, rank, local = dist_setup()
    tideway_b200.load()
    cfg = C3 if not args.layers else PrefillConfig(layers=args.layers)
    stack = GemmaPrefillStack(cfg, device=f"cuda:{local}")
    g = torch.Generator(device=stack.device).manual_seed(cfg.seed + 1)
    x0 = torch.randn(cfg.tokens, cfg.hidden, generator=g, device=stack.device).to(torch.bfloat16)
    x_host = x0.cpu().pin_memory()
    stack.x.copy_(x0)
    stack.capture()
    for _ in range(args.warmup):
        stack.x.copy_(x0)
        stack.graph.replay()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    clock_idx = int(vis.split(",")[local]) if vis else local
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    with ClockSampler(clock_idx) as clk:
        a.record(st)
        for _ in range(args.steps):
            stack.x.copy_(x0)
            stack.graph.replay()
        b.record(st)
        torch.cuda.synchronize()
    ms = max_over_ranks(a.elapsed_time(b) / args.steps, world)
    # routed-expert roofline region: the step's routed FFN launches back to back
    rg = stack.capture_routed_only()
    rg.replay()
    torch.cuda.synchronize()
    a.record(st)
    for _ in range(args.steps):
        rg.replay()
    b.record(st)
    torch.cuda.synchronize()
    routed_ms = a.elapsed_time(b) / args.steps / cfg.layers
    pk = peaks()
    sustained = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()).get(
        "bf16_tflops_sustained", pk["bf16_tflops"]) if pk["source"] == "measured" else 1400.0
    tflops = cfg.routed_flops() / (routed_ms * 1e-3) / 1e12
    wbytes = 3 * cfg.hidden * cfg.inter * 2 * cfg.experts
    # e2e: host input -> step -> host output
    out_host = torch.empty_like(x_host).pin_memory()
    a.record(st)
    for _ in range(args.steps):
        stack.x.copy_(x_host, non_blocking=True)
        stack.graph.replay()
        out_host.copy_(stack.x, non_blocking=True)
    b.record(st)
    torch.cuda.synchronize()
    e2e_ms = a.elapsed_time(b) / args.steps
    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu_layer = cpu_prefill_layer(cfg, cfg.seed + 7)
        cpu = cpu_prefill_baseline(cfg, cpu_layer(), torch.get_num_threads())
    print(json.dumps({
        "metric": PREFILL_METRIC,
        "value": cfg.tokens * world / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": prefill_config(cfg),
        "cpu_baseline": cpu,
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": sustained, "unit": "TFLOP/s",
                     "frac": tflops / sustained, "traffic": prefill_traffic(),
                     "kernel": "routed expert FFN launch per layer (tcgen05), 30 back to back",
                     "ms_per_launch": routed_ms,
                     "hbm_gbs": wbytes / (routed_ms * 1e-3) / 1e9,
                     "hbm_frac": wbytes / (routed_ms * 1e-3) / 1e9 / pk["hbm_gbs"],
                     "peak_source": pk["source"] + " (sustained)"},
        "clocks": clk.summary(),
        "gpu_launches": cfg.layers * 10 * args.steps,
        "e2e": {"value": cfg.tokens / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": cfg.tokens * cfg.hidden * 2,
                "d2h_bytes_per_step": cfg.tokens * cfg.hidden * 2},
    }))


def cpu_fp4_decode_layer(cfg, B: int, seed: int):
    """Host-core path of one configs[3] layer at batch B (the oracle restatement): norm,
    router, sigmoid group top-k, per routed expert and the shared expert a
    dequantise-then-matmul SwiGLU FFN, combine, residual.  Each expert is dequantised when
    its routes run.  One quantised expert's codes stand in for every expert (the cost of
    dequantising and multiplying does not depend on the values; quantising each expert would
    dominate the set-up).  Returns a callable that runs the layer once and returns
    (seconds, experts run including the shared one)."""
    import torch

    from oracle import ffn as off
    from oracle import nvfp4 as onv
    from oracle import routing as orouting
    from tideway_b200 import nvfp4

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(seed)
    H, E, I, K = cfg.hidden, cfg.experts, cfg.inter, cfg.topk
    x = torch.randn(B, H, generator=g).to(torch.bfloat16)
    norm_w = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
    router = (cfg.weight_std * torch.randn(E, H, generator=g)).to(torch.bfloat16)
    (p1, s1, g1), (p2, s2, g2) = nvfp4.quantize_expert(
        cfg.weight_std * torch.randn(2 * I, H, generator=g),
        cfg.weight_std * torch.randn(H, I, generator=g))

    def layer() -> tuple[float, int]:
        t0 = time.perf_counter()
        h = off.rmsnorm(x, norm_w, cfg.eps)
        logits = h.float() @ router.float().t()
        w, ids = orouting.sigmoid_group_topk(logits, K, cfg.n_group, cfg.topk_group,
                                             cfg.routed_scaling, True)
        c3 = torch.zeros(B, K, H, dtype=torch.bfloat16)
        experts = torch.unique(ids).tolist()
        for e in experts:
            t_idx, k_idx = torch.nonzero(ids == e, as_tuple=True)
            c3[t_idx, k_idx] = off.expert_ffn_routes(h[t_idx], onv.dequantize(p1, s1, g1),
                                                     onv.dequantize(p2, s2, g2),
                                                     w[t_idx, k_idx])
        y = c3.float().sum(dim=1).to(torch.bfloat16)
        ysh = off.shared_expert(h, onv.dequantize(p1, s1, g1), onv.dequantize(p2, s2, g2))
        (x.float() + (y.float() + ysh.float()).to(torch.bfloat16).float()).to(torch.bfloat16)
        return time.perf_counter() - t0, len(experts) + 1

    return layer


def cpu_fp4_decode_baseline(cfg, B: int, sec: float, experts: int, cores: int) -> dict:
    return {"value": B / (sec * cfg.layers), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"1 of {cfg.layers} layers at batch {B}: oracle norm, router, sigmoid "
                      f"group top-k, dequantise-then-matmul of {experts} NVFP4 experts (routed "
                      f"+ shared), combine, on {cores} host threads; scaled x{cfg.layers}"}


def cpu_prefill_layer(cfg, seed: int):
    """Host-core path of one configs[2] layer over all ``cfg.tokens`` tokens (the oracle
    restatement): router norm pair + the shared expert's pre-norm, router GEMM, Gemma top-k,
    shared expert, routed experts, dual-norm merge.  Weights and inputs are drawn here; the
    returned callable runs the layer once and returns its seconds."""
    import torch

    from oracle import ffn as off
    from oracle import routing as orouting

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(seed)
    H, E, I, Is, T = cfg.hidden, cfg.experts, cfg.inter, cfg.shared_inter, cfg.tokens
    bf = torch.bfloat16

    def rnd(*shape):
        return (cfg.weight_std * torch.randn(*shape, generator=g)).to(bf)

    def norm_w():
        return (1 + 0.1 * torch.randn(H, generator=g)).to(bf)

    x = torch.randn(T, H, generator=g).to(bf)
    router, router_scale, ones = rnd(E, H), norm_w(), torch.ones(H, dtype=bf)
    expert_scale = (1 + 0.1 * torch.randn(E, generator=g)).float()
    pre_shared, pre_routed = norm_w(), norm_w()
    post_shared, post_routed, post = norm_w(), norm_w(), norm_w()
    sh_w1, sh_w2 = rnd(2 * Is, H), rnd(H, Is)
    w1, w2 = rnd(E, 2 * I, H), rnd(E, H, I)
    root, eps = H ** -0.5, cfg.eps

    def layer() -> float:
        t0 = time.perf_counter()
        router_in, routed_in = off.router_norm_pair(x, ones, pre_routed, router_scale, eps, root)
        shared_in = off.rmsnorm(x, pre_shared, eps)
        logits = router_in.float() @ router.float().t()
        w, ids, _ = orouting.gemma_topk(logits, expert_scale, cfg.topk)
        shared = off.shared_expert(shared_in, sh_w1, sh_w2)
        routed = off.moe_prefill(routed_in, w1, w2, w, ids)
        off.dual_norm_merge(shared, routed, x, post_shared, post_routed, post, eps, eps, eps,
                            cfg.layer_scalar)
        return time.perf_counter() - t0

    return layer


def cpu_prefill_baseline(cfg, layer_s: float, cores: int) -> dict:
    return {"value": cfg.tokens / (layer_s * cfg.layers), "unit": "tokens/s", "cores": cores,
            "kind": "port",
            "sample": f"1 of {cfg.layers} layers over all {cfg.tokens} tokens: oracle norms, "
                      f"router, Gemma top-k, shared expert, {cfg.experts}-expert routed FFN, "
                      f"dual-norm merge on {cores} host threads; scaled x{cfg.layers}"}


def zipf_targets(order, s: float = 1.2, k: int = 6):
    """configs[4]'s expert popularity: Zipf(s) over the popularity ranks (expert order[r] has
    rank r), capped at 1/k because every token routes to k distinct experts (no expert can
    carry more than 1/k of the routes), the capped mass spread over the others in proportion
    to their Zipf weight.  Route shares per expert, summing to 1."""
    import torch

    E = order.numel()
    zipf = 1.0 / torch.arange(1, E + 1, dtype=torch.float64).pow(s)
    capped = torch.zeros(E, dtype=torch.bool)
    p = zipf / zipf.sum()
    while True:
        over = (p > 1.0 / k + 1e-12) & ~capped
        if not bool(over.any()):
            break
        capped |= over
        free = 1.0 - capped.sum().item() / k
        p = torch.where(capped, torch.full_like(p, 1.0 / k), zipf / zipf[~capped].sum() * free)
    target = torch.empty(E, dtype=torch.float64)
    target[order.cpu()] = p
    return target


def fit_zipf_bias(route, target, iters: int = 300, step: float = 0.05, decay: float = 0.995):
    """Selection bias of the sigmoid gate (the DeepSeek correction-bias slot: it changes which
    experts are chosen, not their weights) fitted so that the route shares that ``route(bias)``
    measures (ids [T, K]) follow ``target``: round i adds step * decay^i * log(target_e /
    share_e) (clipped) to bias_e; the decaying step lets the discrete top-k selection settle
    instead of oscillating.  Returns (bias fp32 on the routing device, measured shares)."""
    import torch

    ids = route(None)
    dev = ids.device
    tgt = target.to(dev)
    bias = torch.zeros(target.numel(), dtype=torch.float64, device=dev)
    share = None
    for i in range(iters):
        ids = route(bias.float())
        share = torch.bincount(ids.flatten().long(), minlength=tgt.numel()).double() / ids.numel()
        bias += step * decay ** i * torch.log((tgt + 1e-7) / (share + 1e-7)).clamp(-2.0, 2.0)
    ids = route(bias.float())
    share = torch.bincount(ids.flatten().long(), minlength=tgt.numel()).double() / ids.numel()
    return bias.float(), share


def zipf_report(target, share, order) -> dict:
    """Measured route shares next to the Zipf(1.2) targets, by popularity rank."""
    ranks = [0, 1, 2, 3, 7, 15, 31, 63, 127, 255]
    o = order.cpu()
    t, m = target.cpu()[o], share.cpu()[o]
    return {"ranks": [r + 1 for r in ranks if r < len(o)],
            "target_share": [round(float(t[r]), 5) for r in ranks if r < len(o)],
            "measured_share": [round(float(m[r]), 5) for r in ranks if r < len(o)],
            "top16_target": round(float(t[:16].sum()), 4),
            "top16_measured": round(float(m[:16].sum()), 4),
            "total_variation": round(0.5 * float((t - m).abs().sum()), 4)}


def c5_routing_cpu(cfg, T_fit: int = 8192, seed: int = 4):
    """configs[4] router and fitted Zipf bias on the host (the reference arm's routing): router
    weights, the popularity order and the fit tokens drawn from one CPU generator."""
    import torch

    from oracle import routing as orouting

    g = torch.Generator().manual_seed(seed)
    H, E, K = cfg.hidden, cfg.experts, cfg.topk
    router = (cfg.weight_std * torch.randn(E, H, generator=g)).to(torch.bfloat16)
    order = torch.randperm(E, generator=g)
    x = torch.randn(T_fit, H, generator=g).to(torch.bfloat16)
    logits = x.float() @ router.float().t()
    target = zipf_targets(order, 1.2, K)

    def route(bias):
        return orouting.sigmoid_group_topk(logits, K, cfg.n_group, cfg.topk_group,
                                           cfg.routed_scaling, True, bias=bias)[1]

    bias, share = fit_zipf_bias(route, target)
    return router, bias, zipf_report(target, share, order)


def cpu_ep_layer(cfg, T: int, seed: int, router=None, bias=None):
    """Host-core path of one configs[4] layer over a T-token sample (the oracle
    restatement): router GEMM, sigmoid group top-k with the fitted Zipf selection bias, per
    routed expert dequantise-then-matmul SwiGLU FFN, combine.  Each expert is dequantised when
    its routes run.  One quantised expert's codes stand in for every expert: the cost of
    dequantising and multiplying does not depend on the values, and quantising 256 experts
    would take minutes of set-up.  ``router``/``bias``: the routing to use (default: the
    host-fitted one of ``c5_routing_cpu``).  Returns a callable that runs the layer once and
    returns (seconds, distinct experts)."""
    import torch

    from oracle import ffn as off
    from oracle import nvfp4 as onv
    from oracle import routing as orouting
    from tideway_b200 import nvfp4

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(seed)
    H, E, I, K = cfg.hidden, cfg.experts, cfg.inter, cfg.topk
    if router is None or bias is None:
        router, bias, _ = c5_routing_cpu(cfg)
    router, bias = router.cpu(), bias.cpu()
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    (p1, s1, g1), (p2, s2, g2) = nvfp4.quantize_expert(
        cfg.weight_std * torch.randn(2 * I, H, generator=g),
        cfg.weight_std * torch.randn(H, I, generator=g))

    def layer() -> tuple[float, int]:
        t0 = time.perf_counter()
        logits = x.float() @ router.float().t()
        w, ids = orouting.sigmoid_group_topk(logits, K, cfg.n_group, cfg.topk_group,
                                             cfg.routed_scaling, True, bias=bias)
        c3 = torch.zeros(T, K, H, dtype=torch.bfloat16)
        experts = torch.unique(ids).tolist()
        for e in experts:
            t_idx, k_idx = torch.nonzero(ids == e, as_tuple=True)
            c3[t_idx, k_idx] = off.expert_ffn_routes(x[t_idx], onv.dequantize(p1, s1, g1),
                                                     onv.dequantize(p2, s2, g2),
                                                     w[t_idx, k_idx])
        c3.float().sum(dim=1).to(torch.bfloat16)
        return time.perf_counter() - t0, len(experts)

    return layer


def c5_cpu_sample(prefill: bool) -> int:
    """Tokens in one host-core configs[4] sample (about 10-30 s of CPU work)."""
    return 64 if prefill else 16


def cpu_ep_baseline(T: int, layer_s: float, experts: int, cores: int, prefill: bool) -> dict:
    return {"value": T / layer_s, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"one layer over {T} of the {8192 if prefill else 256} tokens "
                      f"({experts} distinct experts): oracle router, sigmoid group top-k "
                      "with the Zipf bias, dequantise-then-matmul NVFP4 FFN per expert, "
                      f"combine, on {cores} host threads"}


def run_c4(args) -> None:
    """DeepSeek-V4-Flash-shaped NVFP4 decode, 43 layers, 25% slot cache."""
    import torch

    import tideway_b200
    from tideway_b200.stack_fp4 import DSV4_FLASH, Fp4DecodeStack, Fp4StackConfig, Fp4StackWeights

    world, rank, local = dist_setup()
    if world > 1:
        raise SystemExit("c4-decode runs on one GPU (the expert-parallel workload is c2-decode)")
    tideway_b200.load()
    cfg = DSV4_FLASH if not args.layers else Fp4StackConfig(layers=args.layers)
    weights = Fp4StackWeights(cfg, device=f"cuda:{local}")
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    clock_idx = int(vis.split(",")[local]) if vis else local
    B = args.batch
    stack = Fp4DecodeStack(weights, B)
    g = torch.Generator().manual_seed(cfg.seed + 1000 + B)
    x_host = torch.randn(B, cfg.hidden, generator=g).to(torch.bfloat16).pin_memory()
    out_host = torch.empty_like(x_host).pin_memory()
    stack.x_in.copy_(x_host)
    stack.capture()
    for _ in range(args.warmup):
        stack.step()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(clock_idx) as clk:
        a.record(st)
        for _ in range(args.steps):
            stack.step()
        b.record(st)
        torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.steps
    stack.check()  # a bounded wait that gave up would void the timed steps
    uniq = stack.unique_experts_per_layer()
    fg = stack.capture_ffn_only()
    fg.replay()
    torch.cuda.synchronize()
    a.record(st)
    for _ in range(args.steps):
        fg.replay()
    b.record(st)
    torch.cuda.synchronize()
    ffn_ms = a.elapsed_time(b) / args.steps
    ffn_bytes = sum(u * cfg.expert_bytes + 2 * B * cfg.hidden * 2 for u in uniq)
    ffn_gbs = ffn_bytes / (ffn_ms * 1e-3) / 1e9
    # misses of one more step, counted by the slot table
    stack.cache.collect_stats = True
    stack.cache.reset_stats()
    stack.step_eager()
    torch.cuda.synchronize()
    miss = stack.cache.decode_miss_stats()
    stack.cache.collect_stats = False
    a.record(st)
    for _ in range(args.steps):
        stack.decode(x_host, out_host)
    b.record(st)
    torch.cuda.synchronize()
    e2e_ms = a.elapsed_time(b) / args.steps
    cpu = None
    if not args.no_cpu_baseline:
        sec, n_exp = cpu_fp4_decode_layer(cfg, B, cfg.seed + 7)()
        cpu = cpu_fp4_decode_baseline(cfg, B, sec, n_exp, torch.get_num_threads())
    pk = peaks()
    step_bytes = sum((u + 1) * cfg.expert_bytes for u in uniq) + \
        cfg.layers * cfg.experts * cfg.hidden * 2
    print(json.dumps({
        "metric": C4_METRIC,
        "value": B / (ms * 1e-3), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": FP4_DTYPE, "data": "synthetic",
        "config": c4_config(cfg, B),
        "roofline": {"bound": "hbm", "achieved": ffn_gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": ffn_gbs / pk["hbm_gbs"], "traffic": None,
                     "kernel": f"routed NVFP4 expert FFN launches of a step ({cfg.layers}), "
                               "back to back", "ms_per_launch": ffn_ms / cfg.layers,
                     "peak_source": pk["source"]},
        "unique_experts_per_layer": sum(uniq) / len(uniq),
        "misses_per_layer": miss["missing_per_layer"],
        "expert_weight_gbs_step": step_bytes / (ms * 1e-3) / 1e9,
        "clocks": clk.summary(),
        "gpu_launches": stack.launches_per_step() * args.steps,
        "cpu_baseline": cpu,
        "e2e": {"value": B / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": B * cfg.hidden * 2, "d2h_bytes_per_step": B * cfg.hidden * 2},
    }))


def run_c5(args) -> None:
    """expert parallelism at configs[3] layer shapes.  256 NVFP4 experts sharded
    256/G per GPU (resident, no paging), router logits with a seeded Zipf(1.2) popularity bias
    (applied as the sigmoid gate's selection bias), one MoE layer per step: router GEMM,
    sigmoid group top-k, dispatch, NCCL all-to-all, local NVFP4 FFN, all-to-all back, combine.
    Strong scaling: 256 decode tokens or 8192 prefill tokens in total, split over the G GPUs;
    time = max over ranks (CUDA events)."""
    import torch

    import tideway_b200
    from tideway_b200 import ops
    from tideway_b200.ep import ExpertParallelMoE
    from tideway_b200.stack_fp4 import DSV4_FLASH as cfg
    from tideway_b200.stack_fp4 import _BANKS, _quantize_experts

    world, rank, local = dist_setup()
    tideway_b200.load()
    dev = torch.device("cuda", local)
    if 8192 % world or cfg.experts % world:
        raise SystemExit(f"tokens / {cfg.experts} experts do not split over {world}")
    H, E, I, K = cfg.hidden, cfg.experts, cfg.inter, cfg.topk
    Eg = E // world
    g = torch.Generator(device=dev).manual_seed(4)  # shared: router, bias, inputs
    router = (cfg.weight_std * torch.randn(E, H, generator=g, device=dev)).to(torch.bfloat16)
    order = torch.randperm(E, generator=g, device=dev)
    x_all = torch.randn(8192, H, generator=g, device=dev).to(torch.bfloat16)
    # Zipf(1.2) popularity: the selection bias fitted on these 8192 tokens so that their
    # measured route shares follow the (1/6-capped) targets; identical on every rank
    target = zipf_targets(order, 1.2, K)
    fit_logits = ops.router_logits(x_all, router)

    def route(b):
        return ops.sigmoid_group_topk(fit_logits, K, cfg.n_group, cfg.topk_group,
                                      cfg.routed_scaling, True, bias=b)[1]

    bias, share = fit_zipf_bias(route, target)
    popularity = zipf_report(target, share, order)
    del fit_logits
    gl = torch.Generator(device=dev).manual_seed(4 + 1000 * (rank + 1))
    sh = _quantize_experts(Eg, H, I, cfg.weight_std, gl, dev)
    banks = (tuple(sh[k] for k in _BANKS[:3]), tuple(sh[k] for k in _BANKS[3:]))
    for prefill in C5_MODES[args.workload]:
        T_total = 8192 if prefill else 256
        T = T_total // world
        x = x_all[rank * T:(rank + 1) * T].contiguous()
        # decode rows fit one resident wave of the peer-store combine; prefill's 8192 rows
        # take the all-to-alls
        transport = "nccl" if prefill else "p2p"
        ep = ExpertParallelMoE(E, K, H, I, T, dev, transport=transport)
        logits = torch.empty(T, E, dtype=torch.float32, device=dev)
        w = torch.empty(T, K, dtype=torch.float32, device=dev)
        ids = torch.empty(T, K, dtype=torch.int32, device=dev)
        out = torch.empty_like(x)

        def layer():
            ops.router_logits(x, router, out=logits)
            ops.sigmoid_group_topk(logits, K, cfg.n_group, cfg.topk_group, cfg.routed_scaling,
                                   True, bias=bias, out=(w, ids))
            ep.forward_resident(x, w, ids, banks, out)

        layer()
        torch.cuda.synchronize()
        graph = None
        try:
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):
                layer()
            torch.cuda.current_stream(dev).wait_stream(s)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                layer()
        except Exception as e:  # collectives that refuse capture: run eagerly
            torch.cuda.synchronize()
            graph = None
            print(f"[bench] c5 layer not captured ({type(e).__name__}: {e}); running eagerly",
                  file=sys.stderr)
        step = graph.replay if graph is not None else layer
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        st = torch.cuda.current_stream()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        clock_idx = int(vis.split(",")[local]) if vis else local
        barrier(world)
        with ClockSampler(clock_idx) as clk:
            a.record(st)
            for _ in range(args.steps):
                step()
            b.record(st)
            torch.cuda.synchronize()
        barrier(world)
        ms = max_over_ranks(a.elapsed_time(b) / args.steps, world)
        # routing statistics: routes per expert over all ranks, and this rank's received load
        cnt = torch.bincount(ids.flatten().long(), minlength=E).to(torch.int64)
        if world > 1:
            import torch.distributed as dist

            dist.all_reduce(cnt)
        local_ids = ep.ids[ep.ids >= 0]
        uniq_local = int(torch.unique(local_ids).numel())
        routes_local = float(local_ids.numel())
        per_gpu = gather_floats([routes_local, float(uniq_local), ms], world)
        routes_max = max(r[0] for r in per_gpu)
        uniq_max = max(r[1] for r in per_gpu)
        busiest = max(range(world), key=lambda r: per_gpu[r][0])
        top = torch.sort(cnt, descending=True).values.float() / cnt.sum()
        torch.cuda.synchronize()
        barrier(world)
        if rank != 0:
            if graph is not None:
                del graph
            ep.close()
            continue
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            Ts = c5_cpu_sample(prefill)
            sec, n_exp = cpu_ep_layer(cfg, Ts, 4 + 7, router=router, bias=bias)()
            cpu = cpu_ep_baseline(Ts, sec, n_exp, torch.get_num_threads(), prefill)
        print(json.dumps({
            "metric": c5_metric(prefill),
            "value": T_total / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": FP4_DTYPE, "data": "synthetic",
            "config": {**c5_config(cfg, prefill, world), "ep_transport": ep.transport},
            "cpu_baseline": cpu,
            "route_share_top1": float(top[0]), "route_share_top16": float(top[:16].sum()),
            "popularity_fit": popularity,
            "busiest_rank_routes": routes_max, "busiest_rank_distinct_experts": uniq_max,
            "busiest_rank": busiest,
            "per_gpu": [{"rank": r, "routes_received": v[0], "distinct_experts": v[1]}
                        for r, v in enumerate(per_gpu)],
            "clocks": clk.summary(),
            # router, top-k, dispatch, receive, grouping, gather, FFN, combine, EP combine
            "gpu_launches": (8 + grouping_launches(world * T * K, Eg)) * args.steps,
        }))
        if graph is not None:
            del graph
        ep.close()


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "c3-prefill":
        return run_prefill(args)
    if args.workload == "c4-decode":
        return run_c4(args)
    if args.workload.startswith("c5-"):
        return run_c5(args)
    import torch

    import tideway_b200
    from tideway_b200.stack import QWEN3_A3B, StackConfig, StackWeights

    world, rank, local = dist_setup()
    tideway_b200.load()
    cfg = QWEN3_A3B
    if args.layers:
        cfg = StackConfig(**{**cfg.__dict__, "layers": args.layers})
    weights = StackWeights(cfg, device=f"cuda:{local}", shard=(rank, world))
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    clock_idx = int(vis.split(",")[local]) if vis else local

    head = run_batch(weights, args.batch, args.steps, args.warmup, world, rank, clock_idx,
                     not args.no_e2e, args.ffn_only, sustained=True, parity=world > 1,
                     transport=args.ep_transport)
    if args.ffn_only:
        if rank == 0:
            print(json.dumps({"ffn_only": True, "batch": args.batch, "layers": cfg.layers,
                              "unique_experts_per_layer": head["uniq"],
                              "expert_bytes": cfg.expert_bytes}))
        return
    sweep, paging = [], None
    if world == 1 and not args.no_sweep:
        # the other configs[1] batch sizes: the step (paging included: from batch 32 on the
        # step's working set exceeds the slot cache, so every step re-pages), and the FFN
        # launches on the experts the last step left resident (the HBM roofline)
        for B in [int(b) for b in args.sweep_batches.split(",")]:
            if B == args.batch:
                sweep.append(head)
            else:
                n = args.steps if B <= 16 else min(args.steps, 3)
                sweep.append(run_batch(weights, B, n, min(args.warmup, 2), world, rank,
                                       clock_idx, False))
        paging = run_paging(weights, args.batch, min(args.steps, 5), 2)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sec, cores = cpu_c2_timed(cfg, args.batch, 2, 5)
        cpu = cpu_c2_baseline(cfg, args.batch, sec, cores, 2, 5)
    if rank != 0:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    pk = peaks()
    value = head["tokens_per_s"] * world
    out = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {**c2_config(cfg, args.batch, world),
                   **({"ep_transport": head["transport"]} if world > 1 else {})},
        "expert_weight_hbm_gbs": head["expert_weight_gbs_step"],
        "expert_weight_hbm_frac": head["expert_weight_gbs_step"] / pk["hbm_gbs"],
        "roofline": {"bound": "hbm", "achieved": head["ffn_gbs"], "peak": pk["hbm_gbs"],
                     "unit": "GB/s", "frac": head["ffn_gbs"] / pk["hbm_gbs"],
                     "traffic": traffic_per_launch(head["ffn_bytes_per_launch"]),
                     "kernel": "slot-indirect expert FFN launch (grouping, tcgen05 up/down "
                               "kernel, combine) per layer, the step's launches replayed back "
                               "to back",
                     "bytes_per_launch": head["ffn_bytes_per_launch"],
                     "ms_per_launch": head["ffn_ms_per_launch"],
                     "peak_source": pk["source"]},
        "unique_experts_per_layer": head["unique_experts_per_layer"],
        "misses_per_layer": head["misses_per_layer"],
        "clocks": head["clocks"],
        "sustained": head.get("sustained"),
        "gpu_launches": head["launches"],
    }
    if "e2e_tokens_per_s" in head:
        out["e2e"] = {"value": head["e2e_tokens_per_s"] * world, "unit": "tokens/s",
                      "h2d_bytes_per_step": head["h2d"], "d2h_bytes_per_step": head["d2h"]}
    if cpu:
        out["cpu_baseline"] = cpu
    if "per_gpu" in head:
        out["per_gpu"] = head["per_gpu"]
    if "parity" in head:
        out["parity"] = head["parity"]
    if "ep_error_word" in head:
        out["ep_error_word"] = head["ep_error_word"]
    if sweep:
        out["sweep"] = [{"B": r["B"], "tokens_per_s": r["tokens_per_s"],
                         "ms_per_step": r["ms_per_step"], "ffn_gbs": r["ffn_gbs"],
                         "ffn_frac": r["ffn_gbs"] / pk["hbm_gbs"],
                         "ffn_ms_per_launch": r["ffn_ms_per_launch"],
                         "unique_experts_per_layer": r["unique_experts_per_layer"],
                         "misses_per_layer": r["misses_per_layer"],
                         "paged_bytes_per_step": r["paged_bytes_per_step"],
                         "expert_weight_gbs_step": r["expert_weight_gbs_step"]}
                        for r in sweep]
    if paging:
        out["paging"] = paging
    print(json.dumps(out))
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()

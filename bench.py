#!/usr/bin/env python
"""RefineKV decode attention phase on B200: microseconds per decode step at 128K.

Workload (attention phase): Llama-3.1-8B attention
geometry -- 32 layers, 8 KV heads, GQA group 4, head_dim 128 -- over a
131072-token synthetic bf16 prompt per layer (seeded generator, see
refinekv_b200/synthetic.py), block_size 32, eps 0.01, GQA "any", 32 prompt
anchors.  Following the reference's speed protocol (128 generated tokens,
timing the last 125), the default run decodes W=3 warm-up steps and times
K=125 steps.  A step is one decode step of all 32 layers: for each layer the
selector (2 kernels), the split attention (1 kernel) and its combine (1
kernel), replayed from a per-step CUDA graph with the device-side suffix
length.

Every layer's KV (512 MiB) is larger than L2, so no flush is needed between
steps.  value = device time per step (CUDA events, max over ranks).  e2e =
the same step through the public Python API (sparse_attention) with the
step's queries and new K/V tokens copied from pinned host memory and the
outputs copied back inside the timed region, the host waiting for each
step: one captured CUDA graph per step (copies included) for `value`, the
same calls issued eagerly for `eager_value`.

--gpus N shards the KV heads across N ranks (one process per GPU, torchrun);
with N dividing the 8 KV heads there is no per-step collective (strong
scaling: fixed total work).  When N does not divide the heads, or with
--seq-ranks S, each head's prompt blocks are split over S ranks, which
exchange the selector normalisers and the (max, sum, output) rows of each
step over NCCL (refinekv_b200.parallel).

--impl reference times the reference algorithm on the host CPU (the oracle
restatement of the reference PyTorch backend, all host threads): every step
runs all 32 layers, unless that would exceed a few minutes of CPU time, in
which case each step runs a rotating subset of the layers and the line says
how many.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import pathlib
import statistics
import sys
import threading
import time

REPO = pathlib.Path(__file__).resolve().parent
for _p in (REPO, REPO / "refinekv-release_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import torch  # noqa: E402

METRIC = "attention-phase µs/decode step at 128K; achieved HBM GB/s vs B200 peak"
FALLBACK_HBM_GBS = 6650.0


# Whole-decoder shapes for --model (random init: no checkpoints are available).
# RefineKV settings: Llama follows the reference's speed protocol
# (examples/benchmark_decode.py:128-130: B 32, eps 0.01, GQA mean, no anchors);
# Qwen follows BASELINE config 3 (B 64, eps 0.005, GQA max, 64 anchors, the
# first 2 layers dense, static YaRN x4).
MODELS = {
    "llama8b": dict(family="llama", layers=32, hidden=4096, heads=32, kv_heads=8,
                    intermediate=14336, vocab=128256,
                    rope={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                          "high_freq_factor": 4.0, "original_max_position_embeddings": 8192,
                          "rope_theta": 500000.0},
                    refinekv=dict(block_size=32, eps=0.01, gqa_reduction="mean", anchor_tokens=0,
                                  full_attention_layers=0)),
    "qwen7b": dict(family="qwen2", layers=28, hidden=3584, heads=28, kv_heads=4,
                   intermediate=18944, vocab=152064,
                   rope={"rope_type": "yarn", "factor": 4.0,
                         "original_max_position_embeddings": 32768, "rope_theta": 1000000.0},
                   refinekv=dict(block_size=64, eps=0.005, gqa_reduction="max", anchor_tokens=64,
                                 full_attention_layers=2)),
}


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--seq-ranks", type=int, default=None,
                    help="ranks per sequence group (default: split heads first)")
    ap.add_argument("--steps", type=int, default=125)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--tokens", type=int, default=131072)
    ap.add_argument("--kv-heads", type=int, default=8)
    ap.add_argument("--group", type=int, default=4)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--block-size", type=int, default=32)
    ap.add_argument("--eps", type=float, default=0.01)
    ap.add_argument("--reduction", default="any")
    ap.add_argument("--anchors", type=int, default=32)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--query-scale", type=float, default=1.0,
                    help="extra, not the headline workload: scale the queries (sharper "
                         "attention, fewer refined blocks)")
    ap.add_argument("--batch", type=int, default=1,
                    help="extra, not the headline workload: prompts that decode together, "
                         "stacked on the KV-head axis (one GPU)")
    ap.add_argument("--model", choices=sorted(MODELS), default=None,
                    help="extra line, not the headline: a whole random-init decoder of this "
                         "shape decoding through RefineKV(model, config, cuda_graph=True) against "
                         "dense attention on the same model and cache (BASELINE configs 2 and 3)")
    ap.add_argument("--model-layers", type=int, default=None,
                    help="--model: keep only the first N decoder layers (a quick check of the "
                         "flow, not the configuration)")
    ap.add_argument("--new-tokens", type=int, default=128,
                    help="--model: generated tokens (the last new-tokens - 3 are timed)")
    ap.add_argument("--four-kernel-decode", action="store_true",
                    help="run each layer-step as the four kernels (selector stats and final, "
                         "attention, combine) instead of the one-kernel decode (A/B)")
    ap.add_argument("--skip-e2e", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-dense", action="store_true")
    ap.add_argument("--cpu-samples", type=int, default=12)
    args = ap.parse_args()
    if args.warmup < 0 or args.steps < 1:
        ap.error("--steps must be >= 1 and --warmup >= 0")
    if args.batch < 1 or (args.batch > 1 and args.gpus > 1):
        ap.error("--batch must be >= 1, and a batch runs on one GPU")
    if args.model is not None and (args.gpus > 1 or args.new_tokens < 4):
        ap.error("--model runs on one GPU with --new-tokens >= 4")
    return args


def geometry_name(args):
    """The model whose attention geometry the arguments describe."""
    if (args.kv_heads, args.group, args.head_dim) == (4, 7, 128):
        return "qwen2.5-7b", 28
    return "llama3.1-8b", 32


def workload_config(args, world, plan=None):
    """The `config` object; identical in both arms for the same arguments."""
    if plan is None:
        from refinekv_b200 import parallel

        plan = parallel.plan_shards(args.kv_heads * args.batch, args.tokens, args.block_size,
                                    world, 0, args.seq_ranks)
    model, full_layers = geometry_name(args)
    size = f"{args.tokens // 1024}k" if args.tokens % 1024 == 0 else str(args.tokens)
    return {
        "workload": (f"{model}-attention-phase-{size}" if args.layers == full_layers
                     else f"{model}-attention-phase-{args.layers}L-{size}")
                    + ("" if args.query_scale == 1.0 else f"-q{args.query_scale:g}")
                    + ("" if args.batch == 1 else f"-batch{args.batch}"),
        "batch": args.batch,
        "layers": args.layers,
        "prompt_tokens": args.tokens,
        "kv_heads": args.kv_heads,
        "group": args.group,
        "head_dim": args.head_dim,
        "block_size": args.block_size,
        "eps": args.eps,
        "gqa_reduction": args.reduction,
        "anchor_tokens": args.anchors,
        "decode_steps": args.warmup + args.steps,
        "parallelism": f"kv-head shard x{plan.head_shards}, sequence split x{plan.seq_ranks}",
        "cache_flush": "none needed: every layer's KV (heads x tokens x 256 B x 2) exceeds L2",
        "seed": args.seed,
        "query_scale": args.query_scale,
    }


def measured_hbm_peak():
    path = REPO / "MEASURED_PEAKS.json"
    try:
        peaks = json.loads(path.read_text())
        return float(peaks["hbm_gbs"]), "of measured (MEASURED_PEAKS.json hbm_gbs)"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "of fallback (6.65 TB/s pool measurement)"


def profiled_traffic(kernel_file: str):
    """dram bytes per launch and the pages it covered, from a committed ncu figure (JSON)."""
    path = REPO / "profiles" / kernel_file
    try:
        figures = json.loads(path.read_text())
        return float(figures["dram_bytes_per_launch"]), float(figures["pages_per_launch"])
    except (OSError, KeyError, ValueError):
        return None


# ---------------------------------------------------------------------------
# clocks during the timed region (NVML, read-only)
# ---------------------------------------------------------------------------
_REASONS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
    0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
}


class ClockSampler:
    def __init__(self, device: torch.device, period_s: float = 0.01):
        self.samples = []
        self.period = period_s
        self._stop = threading.Event()
        self._thread = None
        self.handle = None
        self.max_mhz = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            try:
                self.handle = pynvml.nvmlDeviceGetHandleByUUID(
                    uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(device.index or 0)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception as error:  # NVML missing: report no clocks rather than fail
            self.error = str(error)

    def _reasons(self):
        nv = self.nvml
        for name in ("nvmlDeviceGetCurrentClocksEventReasons",
                     "nvmlDeviceGetCurrentClocksThrottleReasons"):
            fn = getattr(nv, name, None)
            if fn is not None:
                try:
                    return int(fn(self.handle))
                except Exception:
                    continue
        return 0

    def _run(self):
        nv = self.nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                self.samples.append((mhz, self._reasons()))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.handle is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        if self.handle is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "note": getattr(self, "error", "nvml unavailable")}
        busy = [(m, r) for m, r in self.samples if not r & 0x1] or self.samples
        reasons = 0
        for _, r in busy:
            reasons |= r
        return {
            "sm_mhz": statistics.median(m for m, _ in busy) if busy else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(name for bit, name in _REASONS.items() if reasons & bit),
            "samples": len(self.samples),
        }


# ---------------------------------------------------------------------------
# distributed plumbing (one process per GPU)
# ---------------------------------------------------------------------------
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        torch.cuda.synchronize()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ---------------------------------------------------------------------------
# reference arm: the reference algorithm on the host CPU
# ---------------------------------------------------------------------------
REFERENCE_BUDGET_S = 240.0  # timed CPU work of the reference arm, warm-up included


def run_reference(args):
    """The reference algorithm on the host CPU, one decode step = every layer of the step.

    Each layer's prompt K/V comes from the same generator as the B200 arm
    (drawn on the GPU when there is one, then copied to host memory), is
    summarised by the CPU oracle (the reference PyTorch backend restated,
    ``summary.py:46-113``) and gets its 32-anchor union; every step then
    runs ``reference.py:50-73`` (selection and the mixed softmax) for each
    layer with that step's query and the suffix so far.  When the requested
    steps of all layers would exceed REFERENCE_BUDGET_S of timed work, each
    step runs a rotating subset of the layers and the line says so
    (``layers_timed_per_step``; ``value`` is then that subset's time scaled
    to all layers).
    """
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import refinekv_oracle as ora
    from refinekv_b200 import synthetic

    torch.set_num_threads(max(torch.get_num_threads(), os.cpu_count() or 1))
    cores = torch.get_num_threads()
    gen_dev = "cuda" if torch.cuda.is_available() else "cpu"
    cap = args.warmup + args.steps
    H, D, B, G, N = args.kv_heads * args.batch, args.head_dim, args.block_size, args.group, args.tokens
    layers = []
    for li in range(args.layers):
        seqs = []
        for b in range(args.batch):
            seed = args.seed + 7919 * b if args.batch > 1 else args.seed
            data = synthetic.make_layer(seed, li, args.kv_heads, N, D, B, device=gen_dev)
            seqs.append((seed, data.keys.cpu(), data.values.cpu(), data.planted_mean))
            del data
        L = Layer()
        L.keys = torch.cat([k for _, k, _, _ in seqs])
        L.values = torch.cat([v for _, _, v, _ in seqs])
        L.summary = ora.build_summary(L.keys, L.values, B)

        def queries(step, count, seqs=seqs, li=li):
            return torch.cat([(synthetic.make_queries(seed, li, step, mean, G, count, torch.float32)
                               * args.query_scale).to(torch.bfloat16).cpu()
                              for seed, _, _, mean in seqs], dim=1)

        L.anchor = (ora.anchor_union(queries(-1, args.anchors), L.summary, args.eps,
                                     args.reduction) if args.anchors else None)
        L.q = [queries(s, 1)[0] for s in range(cap)]
        toks = [[synthetic.make_decode_token(seed, li, s, args.kv_heads, D, N + s, device=gen_dev)
                 for seed, _, _, _ in seqs] for s in range(cap)]
        L.suffix_k = torch.cat([torch.cat([k for k, _ in t]) for t in toks], 1).cpu()
        L.suffix_v = torch.cat([torch.cat([v for _, v in t]) for t in toks], 1).cpu()
        layers.append(L)

    def run_layer(L, step):
        ora.sparse_attention(L.q[step], L.summary, L.suffix_k[:, :step + 1],
                             L.suffix_v[:, :step + 1], args.eps, args.reduction,
                             anchor_mask=L.anchor)

    t0 = time.perf_counter()
    run_layer(layers[0], 0)  # untimed: sizes the sample
    per_layer_s = time.perf_counter() - t0
    per_step = len(layers)
    if cap * len(layers) * per_layer_s > REFERENCE_BUDGET_S:
        per_step = max(1, min(len(layers), int(REFERENCE_BUDGET_S / (cap * per_layer_s))))
    times = []
    for step in range(cap):
        chosen = [layers[(step * per_step + j) % len(layers)] for j in range(per_step)]
        t0 = time.perf_counter()
        for L in chosen:
            run_layer(L, step)
        dt = time.perf_counter() - t0
        if step >= args.warmup:
            times.append(dt)
    timed_ms = statistics.median(times) * 1e3
    value_us = timed_ms * 1e3 * len(layers) / per_step
    full = per_step == len(layers)
    sample = (f"every step runs all {len(layers)} layers ({H} KV-head rows x {N} tokens each) "
              "through the CPU oracle (the reference PyTorch backend restated); median over the "
              f"{len(times)} timed steps" if full else
              f"{per_step} of {len(layers)} layers per step (rotating), scaled x{len(layers)}/"
              f"{per_step}: all layers' {cap} steps would exceed {REFERENCE_BUDGET_S:.0f} s")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value_us, 1),
        "unit": "us/step",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(timed_ms, 3),
        "layers_timed_per_step": per_step,
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32 math on bf16 data",
        "data": "synthetic",
        "config": workload_config(args, 1),
        "execution": {"device": "cpu", "threads": cores, "cuda_graph": False},
        "cpu_baseline": {"value": round(value_us, 1), "unit": "us/step", "cores": cores,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value_us, 1), "unit": "us/step", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    emit(line)


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------
class Layer:
    pass


def build_layers(args, plan, group, dev):
    from refinekv_b200 import RefineKVConfig, build_summary, parallel, synthetic

    H = args.kv_heads
    h0, h1 = plan.head_lo, plan.head_hi
    world = plan.world
    cfg = RefineKVConfig(block_size=args.block_size, eps=args.eps,
                         gqa_reduction=args.reduction, anchor_tokens=args.anchors)
    cap = args.warmup + args.steps
    layers = []
    summarize_ms = []
    for li in range(args.layers):
        if args.batch > 1:
            L, ms = build_batch_layer(args, li, cfg, dev)
            layers.append(L)
            summarize_ms.append(ms)
            continue
        data = synthetic.make_layer(args.seed, li, H, args.tokens, args.head_dim,
                                    args.block_size, device=dev)
        L = Layer()
        L.keys, L.values = parallel.shard_prompt(data.keys, data.values, plan)
        if world > 1:  # keep only this rank's share resident
            L.keys, L.values = L.keys.contiguous(), L.values.contiguous()
        del data.keys, data.values
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        # A few ms of spin ahead of the events keep the host's launch time of
        # the summary call out of its measured device time.
        torch.cuda._sleep(10_000_000)
        start.record()
        L.summary = build_summary(L.keys, L.values, cfg)  # the kernel alone; merged below
        end.record()
        end.synchronize()
        summarize_ms.append(start.elapsed_time(end))
        parallel.merge_max_value_norm(L.summary.max_value_norm, group)
        anchors = (synthetic.make_queries(args.seed, li, -1, data.planted_mean, args.group,
                                          args.anchors, torch.float32)[:, h0:h1]
                   * args.query_scale).to(torch.bfloat16)
        L.anchor = (parallel.select_blocks_union_split(anchors.contiguous(), L.summary, cfg, plan,
                                                       group) if args.anchors else None)
        L.q = torch.stack([(synthetic.make_queries(args.seed, li, s, data.planted_mean,
                                                   args.group, 1, torch.float32)[0, h0:h1]
                            * args.query_scale).to(torch.bfloat16)
                           for s in range(cap)]).contiguous()
        L.suffix_k = L.suffix_v = None  # the generated tokens live on the group's last rank
        if plan.holds_suffix:
            ks, vs = [], []
            for s in range(cap):
                k, v = synthetic.make_decode_token(args.seed, li, s, H, args.head_dim,
                                                   args.tokens + s, device=dev)
                ks.append(k[h0:h1])
                vs.append(v[h0:h1])
            L.suffix_k = torch.cat(ks, 1).contiguous()
            L.suffix_v = torch.cat(vs, 1).contiguous()
        L.workspace = {}
        layers.append(L)
    return layers, cfg, summarize_ms


def build_batch_layer(args, li, cfg, dev):
    """One layer of `--batch` prompts (sequence b seeded seed + 7919 b), stacked on the
    KV-head axis in one batched cache whose pages the batched summary aliases."""
    from refinekv_b200 import build_summary_batch, synthetic
    from refinekv_b200.attention import select_blocks_union

    B, H, T, D = args.batch, args.kv_heads, args.tokens, args.head_dim
    cap = args.warmup + args.steps
    keys = torch.empty(B, H, T, D, device=dev, dtype=torch.bfloat16)
    values = torch.empty_like(keys)
    means = []
    for b in range(B):
        data = synthetic.make_layer(args.seed + 7919 * b, li, H, T, D, args.block_size, device=dev)
        keys[b].copy_(data.keys)
        values[b].copy_(data.values)
        means.append(data.planted_mean)
        del data
    L = Layer()
    L.keys, L.values = keys.view(B * H, T, D), values.view(B * H, T, D)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(10_000_000)
    start.record()
    L.summary = build_summary_batch(list(keys), list(values), cfg)
    end.record()
    end.synchronize()

    def queries(step, count):
        return torch.cat([
            (synthetic.make_queries(args.seed + 7919 * b, li, step, means[b], args.group, count,
                                    torch.float32) * args.query_scale).to(torch.bfloat16)
            for b in range(B)], dim=1)

    L.anchor = (select_blocks_union(queries(-1, args.anchors).contiguous(), L.summary, cfg)
                if args.anchors else None)
    L.q = torch.stack([queries(s, 1)[0] for s in range(cap)]).contiguous()
    ks, vs = [], []
    for s in range(cap):
        toks = [synthetic.make_decode_token(args.seed + 7919 * b, li, s, H, D, T + s, device=dev)
                for b in range(B)]
        ks.append(torch.cat([k for k, _ in toks]))
        vs.append(torch.cat([v for _, v in toks]))
    L.suffix_k = torch.cat(ks, 1).contiguous()
    L.suffix_v = torch.cat(vs, 1).contiguous()
    L.workspace = {}
    return L, start.elapsed_time(end)


def run_b200(args):
    rank, world, local = dist_setup()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    from refinekv_b200 import _native, parallel

    if args.four_kernel_decode:
        _native.load().rkv_set_fused_selector(0)
    plan = parallel.plan_shards(args.kv_heads * args.batch, args.tokens, args.block_size, world,
                                rank, args.seq_ranks)
    group = parallel.new_seq_group(plan)
    decode = parallel.SplitDecode(plan, group)
    lib = _native.load()
    layers, cfg, summarize_ms = build_layers(args, plan, group, dev)
    cap = args.warmup + args.steps
    # One tensor per step-wide quantity, each layer's a view of it (as a
    # serving engine lays out its decode buffers): the suffix caches and the
    # attention outputs, so a step moves its inputs and outputs in one copy.
    G, D = args.group, args.head_dim
    out_all = torch.empty(args.layers, plan.heads, G, D, device=dev, dtype=torch.bfloat16)
    for li, L in enumerate(layers):
        L.workspace["output"] = out_all[li]
    sk_all = sv_all = None
    if plan.holds_suffix:
        sk_all = torch.stack([L.suffix_k for L in layers])  # (layers, heads, cap, dim)
        sv_all = torch.stack([L.suffix_v for L in layers])
        for li, L in enumerate(layers):
            L.suffix_k, L.suffix_v = sk_all[li], sv_all[li]
    length = torch.zeros((), device=dev, dtype=torch.int32)
    heads_local = plan.heads
    split = plan.seq_ranks > 1

    # one CUDA graph per decode step: bump the visible suffix, then all layers
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for L in layers:  # allocate every workspace before capture
            decode(L.q[0], L.summary, L.suffix_k, L.suffix_v, cfg, anchor_mask=L.anchor,
                   workspace=L.workspace, suffix_length=length)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    graphs = []
    for s in range(cap):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            length.add_(1)
            for L in layers:
                decode(L.q[s], L.summary, L.suffix_k, L.suffix_v, cfg, anchor_mask=L.anchor,
                       workspace=L.workspace, suffix_length=length)
        graphs.append(g)

    length.zero_()
    barrier(world)
    for s in range(args.warmup):
        graphs[s].replay()
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clocks:
        start.record()
        for s in range(args.warmup, cap):
            graphs[s].replay()
        end.record()
        end.synchronize()
    barrier(world)
    local_ms = start.elapsed_time(end)
    total_ms = max_over_ranks(local_ms, world)
    us_per_step = total_ms * 1e3 / args.steps
    for L in layers:
        from refinekv_b200.attention import device_status

        if device_status(L.workspace):
            raise RuntimeError("device status word set during the timed run")
    del graphs, g  # graphs that hold NCCL calls must go before the process group

    # ---- per-phase timing (CUDA graphs, same steps) for the roofline -------
    # Without a sequence split, each timed step's selector launches (stats +
    # final) and attention launches (attend + combine) for all layers are
    # captured as two graphs and replayed between CUDA events, so the phase
    # times hold no host launch gaps.  With a split, the unit is the whole
    # split step of a layer, taken from the timed run above; one untimed
    # eager pass then counts the selected pages.
    from refinekv_b200 import sparse_attention

    # tokens per (row, page): a batch's counts are per sequence, rows sequence-major
    counts_all = [L.summary.counts.repeat_interleave(plan.heads // L.summary.counts.shape[0], 0)
                  if L.summary.counts.ndim == 2 else L.summary.counts for L in layers]
    sel_tokens = torch.zeros((), device=dev, dtype=torch.int64)
    sel_pages = torch.zeros((), device=dev, dtype=torch.int64)
    # Anchored blocks of all layers (fixed for the whole decode; the one-kernel
    # decode streams them before its decisions).
    anchored_pages = sum(int(L.anchor.sum()) for L in layers if L.anchor is not None)
    fused = (not split and lib.rkv_decode_kernel_count(
        plan.heads, args.group, plan.blocks, args.head_dim, args.block_size) == 1)

    def count_selected():
        nonlocal sel_pages, sel_tokens
        for L, counts in zip(layers, counts_all):
            sel = L.workspace["selected"]
            sel_pages += sel.sum()
            sel_tokens += (sel.to(torch.int64) * counts).sum()

    select_ms, attend_ms = [], []
    if split:
        for s in range(args.warmup, cap):
            length.fill_(s + 1)
            for L in layers:
                decode(L.q[s], L.summary, L.suffix_k, L.suffix_v, cfg, anchor_mask=L.anchor,
                       workspace=L.workspace, suffix_length=length)
            count_selected()
        attend_ms = [us_per_step / 1e3 / args.layers]
    elif fused:
        # One kernel per layer: the per-step graph of all layers' launches,
        # replayed between CUDA events (no host launch gaps).
        step_graphs = []
        for s in range(args.warmup, cap):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for L in layers:
                    sparse_attention(L.q[s], L.summary, L.suffix_k, L.suffix_v, cfg,
                                     anchor_mask=L.anchor, workspace=L.workspace,
                                     suffix_length=length)
            step_graphs.append((s, graph))
        del graph
        events = []
        for s, graph in step_graphs:
            length.fill_(s + 1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            events.append((e0, e1))
            count_selected()
        torch.cuda.synchronize(dev)
        attend_ms = [a.elapsed_time(b) / args.layers for a, b in events]
        del step_graphs
    else:
        phase_graphs = []
        for s in range(args.warmup, cap):
            pair = (torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph())
            for graph, phases in zip(pair, (_native.PHASE_STATS | _native.PHASE_FINAL,
                                            _native.PHASE_ATTEND | _native.PHASE_COMBINE)):
                with torch.cuda.graph(graph):
                    for L in layers:
                        sparse_attention(L.q[s], L.summary, L.suffix_k, L.suffix_v, cfg,
                                         anchor_mask=L.anchor, workspace=L.workspace,
                                         suffix_length=length, _phases=phases)
            phase_graphs.append((s, pair))
        del pair, graph
        events = []
        for s, (g_sel, g_att) in phase_graphs:
            length.fill_(s + 1)
            e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            e0.record()
            g_sel.replay()
            e1.record()
            g_att.replay()
            e2.record()
            events.append((e0, e1, e2))
            count_selected()
        torch.cuda.synchronize(dev)
        select_ms = [a.elapsed_time(b) / args.layers for a, b, _ in events]
        attend_ms = [b.elapsed_time(c) / args.layers for _, b, c in events]
        del phase_graphs, g_sel, g_att
    torch.cuda.synchronize(dev)
    launches = args.steps * args.layers
    pages = int(sel_pages.item())
    tokens_refined = int(sel_tokens.item())
    D, G, B = args.head_dim, args.group, args.block_size
    nb = plan.blocks
    # algorithmic bytes (our formats, workspace scratch excluded)
    suffix_total = (args.layers * heads_local * sum(s + 1 for s in range(args.warmup, cap))
                    if plan.holds_suffix else 0)
    qo_bytes = 2 * heads_local * G * D * 2
    unselected = launches * heads_local * nb - pages
    summary_bytes = (heads_local * nb * D * 2 * 2 + nb * 8 + heads_local * nb * 4 + heads_local * 4
                     + heads_local * nb * (2 if args.anchors else 1))

    def statistics_rows(L, counts):
        # The one-kernel decode reads no statistics (key means, ellipsoids,
        # norms, counts) for a row whose every real block is anchored: none of
        # its blocks is decided or represented.
        if not fused or L.anchor is None:
            return heads_local
        real = (counts if counts.ndim == 2 else counts.expand(heads_local, -1)) > 0
        return heads_local - int((L.anchor | ~real).all(dim=1).sum())

    stat_rows_layers = [statistics_rows(L, c) for L, c in zip(layers, counts_all)]
    mask_bytes = heads_local * nb * (2 if args.anchors else 1)
    stat_bytes_layers = [
        summary_bytes if r == heads_local else
        r * nb * (D * 2 * 2 + 4) + (nb * 8 + heads_local * 4 if r else 0) + mask_bytes
        for r in stat_rows_layers]
    step_bytes = sum(stat_bytes_layers) + args.layers * qo_bytes + (
        tokens_refined * D * 4 + unselected * D * 2 + suffix_total * D * 4) / args.steps
    # Per launch.  One-kernel decode: the whole layer-step (summaries, value
    # means of the unselected blocks, every selected page, the suffix, q and
    # the output).  Four kernels: the attention launch (+ combine) streams the
    # selected pages and the suffix; the selector reads the summaries.
    attend_avg_ms = statistics.mean(attend_ms)
    select_avg_ms = statistics.mean(select_ms) if select_ms else None
    if fused:
        attend_bytes = step_bytes / args.layers
    else:
        attend_bytes = (tokens_refined + suffix_total) * D * 2 * 2 / launches + qo_bytes
    select_bytes = summary_bytes + heads_local * G * D * 2 + unselected * D * 2 / launches
    peak, peak_note = measured_hbm_peak()
    attend_gbs = attend_bytes / (attend_avg_ms * 1e-3) / 1e9
    select_gbs = select_bytes / (select_avg_ms * 1e-3) / 1e9 if select_avg_ms else None
    traffic = profiled_traffic("decode_llama8b_128k.json" if fused
                               else "attend_llama8b_128k.json")
    traffic_per_launch = None
    # A committed capture is of one 128K layer of 8 KV heads in 32-token pages
    # of 128 channels; its DRAM bytes scale with the pages a launch reads only
    # for that workload.
    if (traffic is not None and not split and (args.block_size, args.head_dim) == (32, 128)
            and args.tokens == 131072 and heads_local == 8 and args.batch == 1):
        dram_bytes, pages_profiled = traffic
        traffic_per_launch = dram_bytes * (pages / launches) / pages_profiled
    step_bytes_all = sum_over_ranks(step_bytes, world)  # every rank joins the collective
    step_gbs = step_bytes_all / (us_per_step * 1e-6) / 1e9  # whole job
    step_gbs_per_gpu = step_gbs / world

    # ---- dense decode attention over the same prompt KV (reference point) --
    # The dense alternative RefineKV competes with: one query token against
    # every prompt K/V row of each layer, PyTorch SDPA (GQA), replayed from a
    # CUDA graph over all layers.
    dense = None
    if not split and not args.skip_dense:
        import torch.nn.functional as F

        qd = [L.q[cap - 1].reshape(1, heads_local * args.group, 1, args.head_dim) for L in layers]
        kd = [L.keys.unsqueeze(0) for L in layers]
        vd = [L.values.unsqueeze(0) for L in layers]

        def dense_step():
            for q_, k_, v_ in zip(qd, kd, vd):
                F.scaled_dot_product_attention(q_, k_, v_, enable_gqa=True)

        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            dense_step()
        torch.cuda.current_stream(dev).wait_stream(side)
        dense_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(dense_graph):
            dense_step()
        for _ in range(3):
            dense_graph.replay()
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        d0.record()
        for _ in range(reps):
            dense_graph.replay()
        d1.record()
        d1.synchronize()
        del dense_graph
        dense_layer_us = d0.elapsed_time(d1) * 1e3 / (reps * args.layers)
        dense = {"us_per_layer": round(dense_layer_us, 2),
                 "us_per_step": round(dense_layer_us * args.layers, 1),
                 "impl": "torch.nn.functional.scaled_dot_product_attention (enable_gqa), bf16, "
                         "prompt K/V only, CUDA graph over all layers"}

    # ---- end to end through the public API with host buffers ---------------
    # Each step copies its inputs -- every layer's query and new K/V token,
    # packed in one pinned host buffer -- to the device in one copy, places the
    # new tokens in the suffix caches, runs every layer's decode through the
    # public call and copies all layers' outputs back in one copy; the host
    # waits for them before the next step.  As in the adapter's CUDA-graph
    # decode, each step is one captured graph (copies included); the same
    # steps issued eagerly, call by call, are reported beside it.
    e2e = None
    if not args.skip_e2e:
        pin = dict(pin_memory=True)
        q_words = plan.heads * G * D
        kv_words = 2 * plan.heads * D if plan.holds_suffix else 0
        host_in = torch.empty(cap, args.layers, q_words + kv_words, dtype=torch.bfloat16, **pin)
        for li, L in enumerate(layers):
            host_in[:, li, :q_words] = L.q.reshape(cap, q_words).cpu()
            if plan.holds_suffix:
                kv = torch.stack([L.suffix_k, L.suffix_v]).permute(2, 0, 1, 3)  # (cap, 2, H, D)
                host_in[:, li, q_words:] = kv.reshape(cap, kv_words).cpu()
        dev_in = torch.empty(args.layers, q_words + kv_words, device=dev, dtype=torch.bfloat16)
        q_dev = [dev_in[li, :q_words].view(plan.heads, G, 1, D) for li in range(args.layers)]
        kv_new = dev_in[:, q_words:].view(args.layers, 2, plan.heads, D) if kv_words else None
        reads_output = plan.seq_rank == 0  # every rank of a sequence group gets the output
        out_host = torch.empty(cap, args.layers, plan.heads, G, D, dtype=torch.bfloat16, **pin)

        def e2e_step(s, *, graph_mode):
            dev_in.copy_(host_in[s], non_blocking=True)
            if kv_new is not None:
                sk_all[:, :, s].copy_(kv_new[:, 0])
                sv_all[:, :, s].copy_(kv_new[:, 1])
            if graph_mode:
                length.fill_(s + 1)
            for li, L in enumerate(layers):
                if graph_mode:
                    decode(q_dev[li], L.summary, L.suffix_k, L.suffix_v, cfg,
                           anchor_mask=L.anchor, workspace=L.workspace, suffix_length=length)
                else:
                    decode(q_dev[li], L.summary,
                           L.suffix_k[:, :s + 1] if plan.holds_suffix else None,
                           L.suffix_v[:, :s + 1] if plan.holds_suffix else None, cfg,
                           anchor_mask=L.anchor, workspace=L.workspace)
            if reads_output:
                out_host[s].copy_(out_all, non_blocking=True)

        def timed(run_step):
            barrier(world)
            e_start = torch.cuda.Event(enable_timing=True)
            e_end = torch.cuda.Event(enable_timing=True)
            for s in range(cap):
                if s == args.warmup:
                    barrier(world)
                    e_start.record()
                run_step(s)
                torch.cuda.current_stream(dev).synchronize()  # the host reads the step's outputs
            e_end.record()
            e_end.synchronize()
            return max_over_ranks(e_start.elapsed_time(e_end), world) * 1e3 / args.steps

        eager_us = timed(lambda s: e2e_step(s, graph_mode=False))
        e2e_graphs = []
        for s in range(cap):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                e2e_step(s, graph_mode=True)
            e2e_graphs.append(graph)
        # The first launch of an instantiated graph uploads it to the device;
        # a server replays one uploaded graph every step, so every step graph
        # is launched once before timing (each step rewrites the same suffix
        # slot and length, so a repeated step leaves the same state).
        for graph in e2e_graphs:
            graph.replay()
        del graph
        torch.cuda.synchronize()
        graph_us = timed(lambda s: e2e_graphs[s].replay())
        del e2e_graphs
        h2d = host_in[0].numel() * 2
        d2h = out_all.numel() * 2 if reads_output else 0
        api = "refinekv_b200.parallel.SplitDecode" if split else "refinekv_b200.sparse_attention"
        e2e = {"value": round(graph_us, 1), "unit": "us/step",
               "h2d_bytes_per_step": int(sum_over_ranks(h2d, world)),
               "d2h_bytes_per_step": int(sum_over_ranks(d2h, world)),
               "path": f"{api} via the C ABI, one CUDA graph per step: one pinned-host copy of "
                       "all layers' queries and new K/V tokens in, one copy of all outputs out, "
                       "host waits for each step's outputs",
               "eager_value": round(eager_us, 1),
               "eager_path": f"{api}, eager call per layer, same copies and waits"}

    # ---- CPU baseline: the reference algorithm on the host (rank 0, N=1) ---
    # A bounded sample: `cpu_samples` (layer, step) pairs spread over the
    # layers, each one layer's decode step through the CPU oracle (the
    # reference PyTorch backend restated), timed, median scaled to all
    # layers.  The same pairs double as a parity record: the GPU's mask and
    # output for that layer and step (one eager call, untimed) against the
    # oracle's, masks compared outside the eps margin.
    cpu = parity = None
    if rank == 0 and world == 1 and args.batch == 1 and not args.skip_cpu:
        from oracle import refinekv_oracle as ora

        torch.set_num_threads(os.cpu_count() or 1)
        times = []
        parity = {"layer_steps": 0, "mask_mismatch_outside_margin": 0, "margin_blocks": 0,
                  "max_abs_out_err": 0.0, "tolerance_max_abs": 2e-2,
                  "judge": "the CPU oracle on the GPU's summary; margin = blocks whose "
                           "decisive risk lies within 1e-3 (relative) of eps"}
        check_ws = {}
        for i in range(args.cpu_samples):
            L = layers[i * args.layers // args.cpu_samples]
            s = args.warmup + i % args.steps
            s_cpu = ora.as_cpu_summary(L.summary)
            anchor = L.anchor.cpu() if L.anchor is not None else None
            q = L.q[s].cpu()
            ks, vs = L.suffix_k[:, :s + 1].cpu(), L.suffix_v[:, :s + 1].cpu()
            t0 = time.perf_counter()
            want_out, want_mask = ora.sparse_attention(q, s_cpu, ks, vs, args.eps,
                                                       args.reduction, anchor_mask=anchor)
            times.append(time.perf_counter() - t0)
            got = sparse_attention(L.q[s], L.summary, L.suffix_k[:, :s + 1],
                                   L.suffix_v[:, :s + 1], cfg, anchor_mask=L.anchor,
                                   workspace=check_ws, return_selected=True)
            margin = ora.margin_blocks(q, s_cpu, args.eps, args.reduction)
            if anchor is not None:
                margin &= ~anchor
            parity["layer_steps"] += 1
            parity["margin_blocks"] += int(margin.sum())
            parity["mask_mismatch_outside_margin"] += int(
                ((got.selected.cpu() != want_mask) & ~margin).sum())
            parity["max_abs_out_err"] = max(parity["max_abs_out_err"], float(
                (got.output.float().cpu() - want_out.float()).abs().max()))
            del s_cpu
        cpu_us = statistics.median(times[1:] or times) * 1e6 * args.layers
        cpu = {"value": round(cpu_us, 1), "unit": "us/step", "cores": torch.get_num_threads(),
               "kind": "port",
               "sample": f"{args.cpu_samples} (layer, decode step) pairs spread over the layers, "
                         "each one layer's step through the CPU oracle (reference PyTorch "
                         f"algorithm), median x{args.layers} layers"}

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(us_per_step, 2),
            "unit": "us/step",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(us_per_step / 1e3, 4),
            "higher_is_better": False,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded: LogNormal-scaled RoPE keys, N(0,1) values, 6 planted "
                    "blocks per layer; stands in for the paper's LongBench prompts)",
            "config": workload_config(args, world, plan),
            "execution": {"device": "cuda", "cuda_graph": True},
            "hbm": {"achieved_gbs": round(step_gbs, 1),
                    "achieved_gbs_per_gpu": round(step_gbs_per_gpu, 1), "peak_gbs": peak,
                    "frac": round(step_gbs_per_gpu / peak, 4),
                    "bytes_per_step": int(step_bytes_all),
                    "note": peak_note + "; frac is per GPU (job bytes / GPUs / step time "
                                        "/ one GPU's peak)"},
            "roofline": {"bound": "hbm", "achieved": round(attend_gbs, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(attend_gbs / peak, 4),
                         "traffic": (None if traffic_per_launch is None
                                     else int(traffic_per_launch)),
                         "kernel": ("rkv split decode step (selector, attention, exchanges, "
                                    "merge)" if split else
                                    f"rkv fused_kernel<{D},{B}> (one kernel per layer-step)"
                                    if fused else
                                    f"rkv attend_kernel<{B},{D},{1 if G <= 8 else 2}> + combine"),
                         "algorithmic_bytes_per_launch": int(attend_bytes),
                         "avg_launch_us": round(attend_avg_ms * 1e3, 2),
                         "peak_note": peak_note},
            "phase_us_per_layer": (
                {"split_step": round(attend_avg_ms * 1e3, 2)} if split else
                {"decode_kernel": round(attend_avg_ms * 1e3, 2)} if fused else
                {"select": round(select_avg_ms * 1e3, 2),
                 "select_achieved_gbs": round(select_gbs, 1),
                 "attend_and_combine": round(attend_avg_ms * 1e3, 2),
                 "attend_achieved_gbs": round(attend_gbs, 1)}),
            "one_kernel_decode": fused,
            "anchored_fraction": round(anchored_pages / (args.layers * heads_local * nb), 5),
            # layer-rows decoded without statistics (every block anchored)
            "rows_without_statistics": round(
                1.0 - sum(stat_rows_layers) / (args.layers * heads_local), 4),
            "selected_fraction": round(pages / (launches * heads_local * nb), 5),
            # median over layers (layer 0 carries one-time module loading)
            "summarize_us_per_layer": round(statistics.median(summarize_ms) * 1e3, 1),
            # our kernels per layer-step: 4 (stats, final, attend, combine), or 5 under a
            # sequence split (the same four plus the rank merge; NCCL's kernels not counted)
            # our kernels per layer-step: 1 with the one-kernel decode, 4 with the
            # selector, attention and combine kernels, 5 under a sequence split (+ the
            # rank merge; NCCL's kernels not counted)
            "gpu_launches": args.steps * args.layers * (
                (1 if fused else lib.rkv_decode_launch_count(_native.PHASE_ALL))
                + (1 if split else 0)),
            "clocks": clocks.summary(),
            "e2e": e2e,
            "dense_attention": dense,
            "cpu_baseline": cpu,
            "parity": parity,
        }
        emit(line)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# whole random-init decoder (--model): BASELINE configs 2 and 3
# ---------------------------------------------------------------------------
def build_model(name, dev, seed=0, layers=None):
    """A random-init decoder of the named shape in bf16 on `dev` (initialised on the GPU)."""
    import transformers

    spec = dict(MODELS[name])
    if layers is not None:
        spec["layers"] = layers
    config_type, model_type = (
        (transformers.LlamaConfig, transformers.LlamaForCausalLM) if spec["family"] == "llama"
        else (transformers.Qwen2Config, transformers.Qwen2ForCausalLM))
    config = config_type(
        vocab_size=spec["vocab"], hidden_size=spec["hidden"],
        intermediate_size=spec["intermediate"], num_hidden_layers=spec["layers"],
        num_attention_heads=spec["heads"], num_key_value_heads=spec["kv_heads"],
        max_position_embeddings=131072, rope_parameters=dict(spec["rope"]), pad_token_id=0,
        bos_token_id=None, eos_token_id=None, tie_word_embeddings=False)
    config._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    default = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(dev):
            model = model_type(config)
    finally:
        torch.set_default_dtype(default)
    return model.eval()


def run_model(args):
    """Decode ms/token of a whole random-init decoder at a 128K prompt (reference protocol).

    The reference's speed protocol (examples/benchmark_decode.py:17-100,
    speed/README.md:109): greedy generation of `new_tokens` tokens after a
    synthetic prompt, the last `new_tokens - 3` decode steps timed.  Arms, all
    on the same model, prompt and cache capacity:
    * refinekv_graph -- RefineKV(model, config, cuda_graph=True): dense SDPA
      prefill fused with the summary write, then one captured decode step
      replayed (the clock starts when the capture ends, as the reference's);
    * dense_graph -- the same session with every layer in
      full_attention_layers: dense decode attention over the same static
      cache from the same captured-graph shell (a like-for-like dense arm);
    * full_attention_eager -- the reference's own "Full Attention" arm:
      Transformers' generate over make_visible_static_cache with native SDPA,
      eager, timed from the third forward.
    Times are CUDA events on the generating stream (wall clock beside them).
    """
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    from refinekv_b200 import RefineKV, RefineKVConfig, _native, make_visible_static_cache
    from refinekv_b200.integrations import transformers as adapter

    spec = dict(MODELS[args.model])
    if args.model_layers is not None:
        spec["layers"] = args.model_layers
    model = build_model(args.model, dev, args.seed, spec["layers"])
    gen = torch.Generator(device=dev).manual_seed(args.seed + 12345)
    ids = torch.randint(3, spec["vocab"], (1, args.tokens), device=dev, generator=gen)
    n_new = args.new_tokens
    timed_steps = n_new - 3
    options = dict(input_ids=ids, attention_mask=torch.ones_like(ids), max_new_tokens=n_new,
                   min_new_tokens=n_new, eos_token_id=None, forced_eos_token_id=None,
                   do_sample=False, num_beams=1)
    rk_cfg = dict(spec["refinekv"])

    class Marks:
        """CUDA events + wall times at the boundaries the reference's benchmark marks."""

        def __init__(self):
            self.events, self.walls = {}, {}

        def mark(self, name):
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            torch.cuda.synchronize(dev)
            self.events[name], self.walls[name] = e, time.perf_counter()

        def ms(self, a, b, steps):
            return (self.events[a].elapsed_time(self.events[b]) / steps,
                    (self.walls[b] - self.walls[a]) * 1e3 / steps)

    def graph_arm(config):
        marks = Marks()
        original_graph = torch.cuda.CUDAGraph
        calls = [0]

        class TimedGraph(original_graph):
            def capture_end(self, *a, **k):
                result = super().capture_end(*a, **k)
                marks.mark("replay")
                return result

        def on_forward(module, a, out):
            calls[0] += 1
            if calls[0] == 1:
                marks.mark("prefill_end")

        summarize = []
        real_into, real_summary = adapter.build_summary_into, adapter.build_summary

        def timed(fn):
            def call(*a, **k):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                out = fn(*a, **k)
                e1.record()
                summarize.append((e0, e1))
                return out
            return call

        handle = model.register_forward_hook(on_forward)
        torch.cuda.CUDAGraph = TimedGraph
        adapter.build_summary_into, adapter.build_summary = timed(real_into), timed(real_summary)
        try:
            marks.mark("start")
            with RefineKV(model, RefineKVConfig(**config), cuda_graph=True):
                out = model.generate(**options)
                marks.mark("end")  # before the context's exit, which the GPU would idle through
        finally:
            handle.remove()
            torch.cuda.CUDAGraph = original_graph
            adapter.build_summary_into, adapter.build_summary = real_into, real_summary
        steady, steady_wall = marks.ms("replay", "end", timed_steps)
        prefill_ms = marks.events["start"].elapsed_time(marks.events["prefill_end"])
        summ = [a.elapsed_time(b) * 1e3 for a, b in summarize]
        return dict(ms_per_token=round(steady, 3), wall_ms_per_token=round(steady_wall, 3),
                    prefill_s=round(prefill_ms / 1e3, 2),
                    summarize_us_per_layer=round(statistics.median(summ), 1) if summ else None,
                    summarized_layers=len(summ)), out[0, -n_new:]

    def eager_full_attention():
        marks = Marks()
        calls = [0]

        def on_forward(module, a, out):
            calls[0] += 1
            if calls[0] in (1, 3):
                marks.mark(f"call{calls[0]}")

        cache = make_visible_static_cache(model, args.tokens + n_new)
        handle = model.register_forward_hook(on_forward)
        try:
            with torch.inference_mode():
                marks.mark("start")
                out = model.generate(**options, past_key_values=cache)
                marks.mark("end")
        finally:
            handle.remove()
        del cache
        steady, steady_wall = marks.ms("call3", "end", timed_steps)
        return dict(ms_per_token=round(steady, 3), wall_ms_per_token=round(steady_wall, 3)), \
            out[0, -n_new:]

    def eager_refinekv_stats():
        """Eager RefineKV decode with the reference's access counters (selected fraction)."""
        config = RefineKVConfig(**rk_cfg, collect_stats=True)
        with RefineKV(model, config) as session:
            out = model.generate(**options)
            stats = session.stats
        return stats, out[0, -n_new:]

    dense_cfg = dict(rk_cfg, full_attention_layers=spec["layers"])
    results = {}
    with ClockSampler(dev) as clocks:
        graph_arm(rk_cfg)  # warm-up: module loading, cuBLAS and SDPA plans, first captures
        results["refinekv_graph"], rk_tokens = graph_arm(rk_cfg)
        graph_arm(dense_cfg)
        results["dense_graph"], dense_tokens = graph_arm(dense_cfg)
        results["full_attention_eager"], full_tokens = eager_full_attention()
    stats, eager_tokens = eager_refinekv_stats()
    rk = results["refinekv_graph"]["ms_per_token"]
    layers_sparse = spec["layers"] - rk_cfg["full_attention_layers"]
    line = {
        "metric": "whole-decoder decode ms/token at a 128K prompt (steady: last "
                  f"{timed_steps} of {n_new} generated tokens)",
        "value": rk,
        "unit": "ms/token",
        "n_gpus": 1,
        "steps": timed_steps,
        "warmup": 3,
        "ms_per_step": rk,
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: uniform random token ids, random-init weights (no checkpoints "
                "are available)",
        "config": {"workload": f"{args.model}-random-init-decoder-{args.tokens // 1024}k"
                               + (f"-{spec['layers']}L" if args.model_layers else ""),
                   "model": args.model, "layers": spec["layers"], "hidden": spec["hidden"],
                   "query_heads": spec["heads"], "kv_heads": spec["kv_heads"],
                   "intermediate": spec["intermediate"], "vocab": spec["vocab"],
                   "rope": spec["rope"], "prompt_tokens": args.tokens,
                   "generated_tokens": n_new, "refinekv": rk_cfg, "seed": args.seed},
        "arms": results,
        "speedup_vs_dense_graph": round(results["dense_graph"]["ms_per_token"] / rk, 3),
        "speedup_vs_full_attention_eager": round(
            results["full_attention_eager"]["ms_per_token"] / rk, 3),
        "equivalent_access_ratio": stats["equivalent_access_ratio"],
        "refinekv_decode_calls_per_token": stats["decode_attention_calls"] / max(1, n_new - 1),
        "sparse_layers": layers_sparse,
        "graph_tokens_equal_eager_tokens": bool(torch.equal(rk_tokens, eager_tokens)),
        "tokens_equal_to_dense": round(float((rk_tokens == dense_tokens).float().mean()), 4),
        "dense_graph_tokens_equal_full_attention_tokens": bool(
            torch.equal(dense_tokens, full_tokens)),
        # this build's kernels in the timed replays: the decode kernels of every
        # sparse layer of every timed step
        "gpu_launches": timed_steps * layers_sparse * _native.load().rkv_decode_kernel_count(
            spec["kv_heads"], spec["heads"] // spec["kv_heads"], -(-args.tokens // rk_cfg["block_size"]),
            spec["hidden"] // spec["heads"], rk_cfg["block_size"]),
        "clocks": clocks.summary(),
    }
    emit(line)


# The result line goes to the process's original stdout; everything else the
# process writes to file descriptor 1 (NCCL's version banner, library
# messages) is sent to stderr, so stdout holds exactly the one JSON line.
_RESULT_FD = None


def emit(line: dict) -> None:
    os.write(_RESULT_FD if _RESULT_FD is not None else 1, (json.dumps(line) + "\n").encode())


def main():
    global _RESULT_FD
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)
    args = parse_args()
    if args.model is not None:
        if args.impl == "reference":
            emit({"impl": "reference", "unavailable": "the --model line carries its own dense "
                  "arms on the same model (dense_graph, full_attention_eager); the reference's "
                  "CPU path cannot decode an 8B model at a 128K prompt in a bench run"})
            return
        if "--tokens" not in sys.argv:
            args.tokens = 131072
        run_model(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    run_b200(args)


if __name__ == "__main__":
    main()

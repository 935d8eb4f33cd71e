"""Two-rank worker for tests/test_gpu_split.py::test_two_gpu_nccl_split (run under torchrun).

Both ranks build the same seeded layer (Qwen2.5-7B attention geometry: 4 KV
heads, GQA group 7, block 64, ragged prompt), keep only their half of the
prompt blocks, and decode through ``refinekv_b200.parallel.SplitDecode`` over
NCCL -- eagerly, then from a captured CUDA graph with a device-side suffix
length.  Each rank compares its output with the one-GPU decode of the full
prompt and its mask slice with the oracle outside the eps margin, and prints
``split-ok`` on success.
"""

from __future__ import annotations

import datetime
import os
import pathlib
import sys

REPO = pathlib.Path(__file__).resolve().parents[1]
for _p in (REPO, REPO / "refinekv-release_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from oracle import refinekv_oracle as ora  # noqa: E402
from refinekv_b200 import RefineKVConfig, build_summary, parallel, sparse_attention, synthetic  # noqa: E402
from refinekv_b200.attention import select_blocks_union  # noqa: E402


def main() -> None:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    heads, group, dim, block, tokens, cap = 4, 7, 128, 64, 6000, 16
    cfg = RefineKVConfig(block_size=block, eps=0.3, gqa_reduction="max")
    data = synthetic.make_layer(21, 0, heads, tokens, dim, block, device=dev)
    q = (synthetic.make_queries(21, 0, 0, data.planted_mean, group, 1, torch.float32)[0]
         * 32.0).to(torch.bfloat16)
    gen = torch.Generator(device=dev).manual_seed(22)
    ks = torch.randn(heads, cap, dim, device=dev, generator=gen).to(torch.bfloat16)
    vs = torch.randn(heads, cap, dim, device=dev, generator=gen).to(torch.bfloat16)

    plan = parallel.plan_shards(heads, tokens, block, world, rank, seq_ranks=world)
    seq_group = parallel.new_seq_group(plan)
    k, v = parallel.shard_prompt(data.keys, data.values, plan)
    summary = parallel.build_shard_summary(k, v, cfg, plan, seq_group)
    anchors = (synthetic.make_queries(21, 0, -1, data.planted_mean, group, 8, torch.float32)
               * 32.0).to(torch.bfloat16)
    anchor = parallel.select_blocks_union_split(anchors, summary, cfg, plan, seq_group)
    decode = parallel.SplitDecode(plan, seq_group)
    mine_k = ks if plan.holds_suffix else None
    mine_v = vs if plan.holds_suffix else None

    full = build_summary(data.keys, data.values, cfg)
    s_cpu = ora.as_cpu_summary(full)
    margin = ora.margin_blocks(q.cpu(), s_cpu, cfg.eps, cfg.gqa_reduction)
    failures = []
    full_anchor = select_blocks_union(anchors, full, cfg)
    anchor_margin = torch.zeros_like(margin)
    for a in anchors.cpu():
        anchor_margin |= ora.margin_blocks(a, s_cpu, cfg.eps, cfg.gqa_reduction)
    lo, hi = plan.block_lo, plan.block_hi
    if ((anchor.cpu() != full_anchor[:, lo:hi].cpu()) & ~anchor_margin[:, lo:hi]).any():
        failures.append("anchor union differs outside the margin")

    def check(out, selected, n, what):
        want = sparse_attention(q, full, ks[:, :n], vs[:, :n], cfg, anchor_mask=full_anchor,
                                return_selected=True)
        lo, hi = plan.block_lo, plan.block_hi
        bad = (selected.cpu() != want.selected[:, lo:hi].cpu()) & ~margin[:, lo:hi]
        if bad.any():
            failures.append(f"{what}: {int(bad.sum())} blocks differ outside the margin")
        err = float((out.float() - want.output.float()).abs().max())
        if err > 2e-2:
            failures.append(f"{what}: max abs error {err}")

    workspace = {}
    res = decode(q, summary, mine_k, mine_v, cfg, anchor_mask=anchor, workspace=workspace,
                 return_selected=True)
    check(res.output, res.selected, cap, "eager")

    length = torch.tensor(cap, device=dev, dtype=torch.int32)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        decode(q, summary, mine_k, mine_v, cfg, anchor_mask=anchor, workspace=workspace,
               suffix_length=length)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = decode(q, summary, mine_k, mine_v, cfg, anchor_mask=anchor, workspace=workspace,
                     suffix_length=length).output
    for n in (3, 11):
        length.fill_(n)
        graph.replay()
        torch.cuda.synchronize(dev)
        check(out, workspace["selected"].bool(), n, f"graph n={n}")
    del graph  # a graph holding NCCL calls goes before the process group
    dist.barrier()
    dist.destroy_process_group()
    if failures:
        print(f"rank {rank} FAILED: " + "; ".join(failures), flush=True)
        sys.exit(1)
    print(f"rank {rank} split-ok", flush=True)


if __name__ == "__main__":
    main()

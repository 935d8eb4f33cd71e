"""Sequence-split decode (rkv_decode_split) against the one-GPU decode and the oracle.

One GPU plays every rank of a sequence group: each rank's summary covers its
own blocks, all ranks write their slabs into one exchange buffer (which is
what the all-gathers produce on real ranks), and the three stages run in
order for all ranks.  The concatenated masks must equal the one-GPU masks
outside the eps margin (the only difference is the summation order of the
row normalisers) and every rank's merged output must match the one-GPU
output and the oracle within the usual tolerances.  The two-GPU NCCL run of
the same path is ``test_two_gpu_nccl_split`` (skipped with fewer GPUs).
"""

from __future__ import annotations

import os
import pathlib
import socket
import subprocess
import sys

import pytest
import torch

from oracle import refinekv_oracle as ora
from refinekv_b200 import RefineKVConfig, _native, build_summary, parallel, sparse_attention, synthetic
from refinekv_b200.attention import _query_code

pytestmark = pytest.mark.gpu
DEV = "cuda"
REPO = pathlib.Path(__file__).resolve().parents[1]


def _emulate(q, keys, values, ks, vs, cfg, seq_ranks, *, anchor=None, suffix_length=None):
    """All ranks of one sequence group on this GPU; returns (per-rank outputs, mask, summaries)."""
    heads, group, _, dim = q.shape
    tokens = keys.shape[1]
    plans = [parallel.plan_shards(heads, tokens, cfg.block_size, seq_ranks, r, seq_ranks=seq_ranks)
             for r in range(seq_ranks)]
    summaries = [build_summary(*parallel.shard_prompt(keys, values, p), cfg) for p in plans]
    vmax = torch.stack([s.max_value_norm for s in summaries]).amax(0)
    for s in summaries:
        s.max_value_norm.copy_(vmax)
    stats_slab, out_slab = parallel.exchange_slabs(heads, group, plans[0].max_blocks, dim)
    exchange = torch.zeros(seq_ranks * (stats_slab + out_slab), device=DEV, dtype=torch.uint8)
    lib = _native.load()
    qc = q.reshape(heads, group, dim).contiguous()
    outs, masks, calls = [], [], []
    for p, s in zip(plans, summaries):
        ws = torch.zeros(lib.rkv_decode_workspace_size(heads, group, s.num_blocks, dim,
                                                       cfg.block_size), device=DEV,
                         dtype=torch.uint8)
        out = torch.full((heads, group, dim), float("nan"), device=DEV, dtype=q.dtype)
        sel = torch.full((heads, s.num_blocks), 7, device=DEV, dtype=torch.uint8)
        cap = ks.shape[1] if p.holds_suffix else 0
        anc = anchor[:, p.block_lo:p.block_hi].contiguous() if anchor is not None else None
        args = (s.abi(), qc.data_ptr(), _query_code(qc), group,
                ks.data_ptr() if cap else None, vs.data_ptr() if cap else None, cap,
                ks.stride(0), ks.stride(1), vs.stride(0), vs.stride(1),
                suffix_length.data_ptr() if (cap and suffix_length is not None) else None, cap,
                anc.data_ptr() if anc is not None else None, cfg.eps,
                _native.GQA_CODES[cfg.gqa_reduction], out.data_ptr(), sel.data_ptr(),
                ws.data_ptr(), ws.numel(), seq_ranks, p.seq_rank, p.max_blocks,
                exchange.data_ptr(), exchange.numel())
        calls.append((args, ws, anc))
        outs.append(out)
        masks.append(sel)
    stream = torch.cuda.current_stream().cuda_stream
    for stage in (_native.SPLIT_STATS, _native.SPLIT_ATTEND, _native.SPLIT_MERGE):
        for args, _, _ in calls:
            _native.check(lib.rkv_decode_split(*args, stage, stream))
    torch.cuda.synchronize()
    for _, ws, _ in calls:
        assert int(ws[:4].view(torch.int32).item()) == 0  # device status word
    return outs, torch.cat(masks, 1).bool(), summaries


def _case(seed, heads, group, dim, block, tokens, suffix, sharpness=1.0, qdtype=torch.bfloat16):
    data = synthetic.make_layer(seed, 0, heads, tokens, dim, block, device=DEV)
    q = (synthetic.make_queries(seed, 0, 0, data.planted_mean, group, 1, torch.float32)[0]
         * sharpness).to(qdtype)
    gen = torch.Generator(device=DEV).manual_seed(seed + 1)
    ks = torch.randn(heads, suffix, dim, device=DEV, generator=gen).to(torch.bfloat16)
    vs = torch.randn(heads, suffix, dim, device=DEV, generator=gen).to(torch.bfloat16)
    return data, q, ks, vs


def _check(outs, mask, q, data, ks, vs, cfg, *, anchor=None):
    full = build_summary(data.keys, data.values, cfg)
    want = sparse_attention(q, full, ks, vs, cfg, anchor_mask=anchor, return_selected=True)
    s_cpu = ora.as_cpu_summary(full)
    margin = ora.margin_blocks(q.cpu(), s_cpu, cfg.eps, cfg.gqa_reduction)
    diff = (mask.cpu() != want.selected.cpu()) & ~margin
    assert not diff.any(), f"{int(diff.sum())} blocks differ outside the eps margin"
    fp32 = q.dtype == torch.float32
    tol = dict(atol=1e-4, rtol=0) if fp32 else dict(atol=4e-3, rtol=2e-2)
    for out in outs[1:]:
        assert torch.equal(out, outs[0])  # every rank gets the same merged output
    if bool((mask.cpu() == want.selected.cpu()).all()):
        torch.testing.assert_close(outs[0], want.output.reshape(outs[0].shape), **tol)
        # and against the oracle directly
        _, z = ora.select_blocks(q.cpu(), s_cpu, cfg.eps, cfg.gqa_reduction)
        oracle = ora.mixed_attention(q.cpu(), s_cpu, ks.cpu(), vs.cpu(), mask.cpu(), z)
        limit = 1e-4 if fp32 else 2e-2
        assert float((outs[0].cpu().float() - oracle[:, :, 0]).abs().max()) <= limit
    return want


SPLIT_CASES = [
    # seed, heads, group, dim, block, tokens, suffix, reduction, eps, sharpness, ranks
    (1, 8, 4, 128, 32, 8192, 5, "any", 0.01, 1.0, 2),
    (2, 8, 4, 128, 32, 8192, 5, "any", 0.3, 16.0, 4),
    (3, 4, 7, 128, 64, 5000, 9, "max", 0.005, 1.0, 2),   # Qwen2.5-7B geometry, ragged tail
    (4, 4, 7, 128, 64, 5000, 9, "max", 0.3, 32.0, 3),
    (5, 2, 16, 64, 16, 1000, 40, "mean", 0.3, 16.0, 2),
    (6, 1, 2, 256, 32, 300, 0, "any", 0.3, 16.0, 4),     # no suffix at all
]


@pytest.mark.parametrize("case", SPLIT_CASES)
@pytest.mark.parametrize("qdtype", [torch.bfloat16, torch.float32])
def test_emulated_split_matches_one_gpu(case, qdtype):
    seed, heads, group, dim, block, tokens, suffix, reduction, eps, sharp, ranks = case
    cfg = RefineKVConfig(block_size=block, eps=eps, gqa_reduction=reduction)
    data, q, ks, vs = _case(seed, heads, group, dim, block, tokens, suffix, sharp, qdtype)
    outs, mask, _ = _emulate(q, data.keys, data.values, ks, vs, cfg, ranks)
    _check(outs, mask, q, data, ks, vs, cfg)


def test_emulated_split_with_anchors_and_device_suffix_length():
    heads, group, dim, block, tokens = 4, 7, 128, 64, 6000
    cfg = RefineKVConfig(block_size=block, eps=0.3, gqa_reduction="max")
    data, q, ks, vs = _case(9, heads, group, dim, block, tokens, 16, 32.0)
    anchor = torch.zeros(heads, -(-tokens // block), device=DEV, dtype=torch.bool)
    anchor[:, ::7] = True
    length = torch.tensor(11, device=DEV, dtype=torch.int32)
    outs, mask, _ = _emulate(q, data.keys, data.values, ks, vs, cfg, 2, anchor=anchor,
                             suffix_length=length)
    assert bool(mask[anchor].all())
    _check(outs, mask, q, data, ks[:, :11], vs[:, :11], cfg, anchor=anchor)


@pytest.mark.parametrize("ranks", [2, 3])
def test_emulated_anchor_union_split(ranks):
    """rkv_select_split over several anchor queries equals the one-GPU union outside the margin."""
    from refinekv_b200.attention import select_blocks_union

    heads, group, dim, block, tokens, count = 4, 7, 128, 64, 7000, 4
    cfg = RefineKVConfig(block_size=block, eps=3.0, gqa_reduction="max")
    data = synthetic.make_layer(13, 0, heads, tokens, dim, block, device=DEV)
    anchors = (synthetic.make_queries(13, 0, -1, data.planted_mean, group, count, torch.float32)
               * 32.0).to(torch.bfloat16)
    full = build_summary(data.keys, data.values, cfg)
    want = select_blocks_union(anchors, full, cfg)
    plans = [parallel.plan_shards(heads, tokens, block, ranks, r, seq_ranks=ranks)
             for r in range(ranks)]
    summaries = [build_summary(*parallel.shard_prompt(data.keys, data.values, p), cfg)
                 for p in plans]
    vmax = torch.stack([x.max_value_norm for x in summaries]).amax(0)
    for x in summaries:
        x.max_value_norm.copy_(vmax)
    lib = _native.load()
    slab = lib.rkv_select_split_slab(heads, group, plans[0].max_blocks, count)
    exchange = torch.zeros(ranks * slab, device=DEV, dtype=torch.uint8)
    q = anchors.reshape(count, heads, group, dim).contiguous()
    calls, masks = [], []
    for p, x in zip(plans, summaries):
        ws = torch.zeros(lib.rkv_select_workspace_size(heads, group, x.num_blocks, dim, count),
                         device=DEV, dtype=torch.uint8)
        m = torch.full((heads, x.num_blocks), 7, device=DEV, dtype=torch.uint8)
        calls.append((x.abi(), q.data_ptr(), 0, count, group, cfg.eps, 1, m.data_ptr(), 0,
                      ws.data_ptr(), ws.numel(), ranks, p.seq_rank, p.max_blocks,
                      exchange.data_ptr(), exchange.numel(), ws))
        masks.append(m)
    stream = torch.cuda.current_stream().cuda_stream
    for stage in (_native.SPLIT_STATS, _native.SPLIT_FINAL):
        for c in calls:
            _native.check(lib.rkv_select_split(*c[:-1], stage, stream))
    torch.cuda.synchronize()
    got = torch.cat(masks, 1).bool().cpu()
    s_cpu = ora.as_cpu_summary(full)
    margin = torch.zeros_like(got)
    for a in anchors.cpu():
        margin |= ora.margin_blocks(a, s_cpu, cfg.eps, cfg.gqa_reduction)
    assert 0 < int(want.sum()) < want.numel()
    assert not ((got != want.cpu()) & ~margin).any()


def test_split_rejects_bad_geometry():
    lib = _native.load()
    cfg = RefineKVConfig(eps=0.01)
    data, q, ks, vs = _case(7, 2, 4, 128, 32, 2048, 0)
    s = build_summary(data.keys, data.values, cfg)
    qc = q.reshape(2, 4, 128).contiguous()
    out = torch.empty_like(qc)
    sel = torch.empty(2, s.num_blocks, device=DEV, dtype=torch.uint8)
    ws = torch.zeros(lib.rkv_decode_workspace_size(2, 4, s.num_blocks, 128, 32), device=DEV,
                     dtype=torch.uint8)
    stats_slab, out_slab = parallel.exchange_slabs(2, 4, s.num_blocks, 128)
    ex = torch.zeros(2 * (stats_slab + out_slab), device=DEV, dtype=torch.uint8)

    def call(ranks, rank, max_blocks, exchange_bytes, stage=_native.SPLIT_STATS):
        return lib.rkv_decode_split(s.abi(), qc.data_ptr(), 0, 4, None, None, 0, 0, 0, 0, 0,
                                    None, 0, None, 0.01, 2, out.data_ptr(), sel.data_ptr(),
                                    ws.data_ptr(), ws.numel(), ranks, rank, max_blocks,
                                    ex.data_ptr(), exchange_bytes, stage,
                                    torch.cuda.current_stream().cuda_stream)

    assert call(2, 2, s.num_blocks, ex.numel()) == _native.RKV_ERR_INVALID_ARGUMENT
    assert call(2, 0, s.num_blocks - 1, ex.numel()) == _native.RKV_ERR_INVALID_ARGUMENT
    assert call(2, 0, s.num_blocks, ex.numel() - 1) == _native.RKV_ERR_WORKSPACE
    assert call(2, 0, s.num_blocks, ex.numel(), stage=8) == _native.RKV_ERR_INVALID_ARGUMENT
    assert call(2, 0, s.num_blocks, ex.numel()) == _native.RKV_OK
    torch.cuda.synchronize()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_nccl_split():
    """SplitDecode over NCCL on two GPUs (eager and CUDA-graph replay) vs the one-GPU decode."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=os.pathsep.join(
        [str(REPO), str(REPO / "refinekv-release_b200"), os.environ.get("PYTHONPATH", "")]))
    cmd = ["timeout", "-k", "60", "420", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1",
           f"--master-port={_free_port()}", str(REPO / "tests" / "split_nccl_worker.py")]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=540)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    assert proc.stdout.count("split-ok") == 2, proc.stdout[-3000:]

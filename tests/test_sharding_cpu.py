"""Multi-GPU host logic on the CPU: shard plans, the slab exchange and the split decode math.

The GPU path (``refinekv_b200.parallel``) shards KV heads over ranks and,
when ranks outnumber heads, splits each head's prompt blocks over a sequence
group that exchanges two small slabs per step.  Here, without GPUs:

* every plan tiles the (head, block) grid exactly once with one suffix owner
  per sequence group;
* ``all_gather_slabs`` and ``merge_max_value_norm`` -- the same helpers the
  CUDA path calls over NCCL -- run on ``gloo`` ranks (world size 2 and 4);
* the split decode, written with the oracle's per-rank pieces and exchanged
  through those helpers, reproduces the one-GPU oracle: masks equal outside
  the eps margin, outputs within 1e-5.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import refinekv_oracle as ref
from refinekv_b200 import parallel


# ---------------------------------------------------------------------------
# plans
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("heads", [1, 4, 8, 28])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("tokens,block", [(8192, 32), (1000, 64), (131072, 32), (70, 16)])
def test_plan_tiles_the_head_block_grid_once(heads, world, tokens, block):
    blocks = -(-tokens // block)
    seq = parallel.default_seq_ranks(heads, world)
    if blocks < seq:
        with pytest.raises(ValueError):
            parallel.plan_shards(heads, tokens, block, world, 0)
        return
    plans = [parallel.plan_shards(heads, tokens, block, world, r) for r in range(world)]
    cover = torch.zeros(heads, blocks, dtype=torch.int32)
    for p in plans:
        assert p.seq_ranks == seq and p.head_shards * p.seq_ranks == world
        assert p.blocks >= 1 and p.blocks <= p.max_blocks
        assert p.token_lo == p.block_lo * block
        assert p.token_hi - p.token_lo <= p.blocks * block
        assert p.rank in p.seq_group and len(p.seq_group) == seq
        cover[p.head_lo:p.head_hi, p.block_lo:p.block_hi] += 1
    assert bool((cover == 1).all())
    for shard in range(plans[0].head_shards):
        owners = [p for p in plans if p.head_shard == shard and p.holds_suffix]
        assert len(owners) == 1 and owners[0].block_hi == blocks and owners[0].token_hi == tokens
    if world <= heads and heads % world == 0:
        assert seq == 1  # heads are split before the sequence


def test_plan_forced_grid_and_errors():
    p = parallel.plan_shards(8, 8192, 32, 8, 5, seq_ranks=2)  # 4 head shards x 2
    assert (p.head_shards, p.head_shard, p.seq_rank) == (4, 2, 1)
    assert (p.head_lo, p.head_hi, p.block_lo, p.block_hi) == (4, 6, 128, 256)
    assert p.holds_suffix and p.seq_group == (4, 5)
    with pytest.raises(ValueError):
        parallel.plan_shards(8, 8192, 32, 8, 0, seq_ranks=3)  # does not divide the world
    with pytest.raises(ValueError):
        parallel.plan_shards(6, 8192, 32, 4, 0, seq_ranks=1)  # 4 head shards of 6 heads
    with pytest.raises(ValueError):
        parallel.plan_shards(8, 8192, 32, 2, 2)
    with pytest.raises(ValueError):
        parallel.plan_shards(1, 40, 32, 4, 0)  # 2 blocks over 4 ranks


# ---------------------------------------------------------------------------
# split decode on one process (oracle pieces, no exchange)
# ---------------------------------------------------------------------------

def _layer(seed, heads, group, tokens, dim, suffix, sharpness=1.0):
    """Seeded layer; `sharpness` scales the query so that short prompts get a sparse mask."""
    g = torch.Generator().manual_seed(seed)
    scales = torch.exp(0.5 * torch.randn(heads, 1, dim, generator=g))
    keys = (torch.randn(heads, tokens, dim, generator=g) * scales).to(torch.bfloat16)
    values = torch.randn(heads, tokens, dim, generator=g).to(torch.bfloat16)
    planted = keys[:, :min(tokens, 64)].float().mean(1, keepdim=True)
    query = sharpness * (0.7 * planted.unsqueeze(1).expand(heads, group, 1, dim)
                         + 0.3 * torch.randn(heads, group, 1, dim, generator=g))
    ks = torch.randn(heads, suffix, dim, generator=g).to(torch.bfloat16)
    vs = torch.randn(heads, suffix, dim, generator=g).to(torch.bfloat16)
    return keys, values, query, ks, vs


def _decode_split_local(keys, values, query, ks, vs, block, seq_ranks, eps, reduction):
    plans = [parallel.plan_shards(keys.shape[0], keys.shape[1], block, seq_ranks, r,
                                  seq_ranks=seq_ranks) for r in range(seq_ranks)]
    summaries = []
    for p in plans:
        k, v = parallel.shard_prompt(keys, values, p)
        summaries.append(ref.build_summary(k, v, block_size=block))
    vmax = torch.stack([s.max_value_norm for s in summaries]).amax(0)
    for s in summaries:
        s.max_value_norm = vmax.clone()
    partials = torch.stack([ref.normalizer_partials(query, s) for s in summaries])
    log_z, log_c = ref.merge_normalizers(partials)
    masks, ms, ls, os_ = [], [], [], []
    for p, s in zip(plans, summaries):
        sel, z = ref.select_blocks_given(query, s, log_z, log_c, eps, reduction)
        sk = ks if p.holds_suffix else ks[:, :0]
        sv = vs if p.holds_suffix else vs[:, :0]
        m, l, o = ref.mixed_attention_partial(query, s, sk, sv, sel, z)
        masks.append(sel)
        ms.append(m)
        ls.append(l)
        os_.append(o)
    out = ref.merge_rank_outputs(torch.stack(ms), torch.stack(ls), torch.stack(os_))
    return out, torch.cat(masks, 1)


@pytest.mark.parametrize("seq_ranks", [2, 3, 4])
@pytest.mark.parametrize("heads,group,tokens,block,reduction,sharpness", [
    (2, 4, 2048, 32, "any", 16.0),
    (2, 7, 1000, 64, "max", 32.0),  # Qwen2.5-7B group, ragged last page
    (1, 4, 777, 16, "mean", 16.0),
])
def test_split_pieces_match_the_one_piece_oracle(seq_ranks, heads, group, tokens, block,
                                                 reduction, sharpness):
    eps = 0.3
    keys, values, query, ks, vs = _layer(7, heads, group, tokens, 64, 5, sharpness)
    full = ref.build_summary(keys, values, block_size=block)
    want, want_mask = ref.sparse_attention(query, full, ks, vs, eps, reduction)
    out, mask = _decode_split_local(keys, values, query, ks, vs, block, seq_ranks, eps,
                                    reduction)
    margin = ref.margin_blocks(query, full, eps, reduction)
    assert bool(((mask == want_mask) | margin).all())
    assert 0 < int(want_mask.sum()) < want_mask.numel()  # selection is not trivial here
    if bool((mask == want_mask).all()):
        torch.testing.assert_close(out, want.float(), atol=1e-5, rtol=1e-5)


# ---------------------------------------------------------------------------
# gloo ranks
# ---------------------------------------------------------------------------

def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port, case, results):
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        results[rank] = _CASES[case](rank, world)
    finally:
        dist.destroy_process_group()


def _case_exchange(rank, world):
    # Two regions of different slab sizes in one flat buffer, as rkv_decode_split lays them out.
    stats_slab, out_slab = 48, 80
    buf = torch.zeros(world * (stats_slab + out_slab), dtype=torch.uint8)
    buf[rank * stats_slab:(rank + 1) * stats_slab] = rank + 1
    off = world * stats_slab
    buf[off + rank * out_slab:off + (rank + 1) * out_slab] = 100 + rank
    parallel.all_gather_slabs(buf[:off], stats_slab, rank, None)
    parallel.all_gather_slabs(buf[off:], out_slab, rank, None)
    want = torch.cat([torch.full((stats_slab,), r + 1, dtype=torch.uint8) for r in range(world)]
                     + [torch.full((out_slab,), 100 + r, dtype=torch.uint8) for r in range(world)])
    vmax = torch.tensor([float(rank), 10.0 - rank])
    parallel.merge_max_value_norm(vmax, dist.group.WORLD)
    return bool(torch.equal(buf, want)) and vmax.tolist() == [world - 1.0, 10.0]


def _case_split_decode(rank, world):
    """A (world/2) head x 2 sequence grid; per-rank oracle pieces, exchanged with gloo."""
    heads, group, tokens, block, eps, reduction = 4, 7, 1500, 64, 0.3, "max"
    keys, values, query, ks, vs = _layer(11, heads, group, tokens, 64, 4, 32.0)
    seq = 2
    plan = parallel.plan_shards(heads, tokens, block, world, rank, seq_ranks=seq)
    seq_group = parallel.new_seq_group(plan)
    k, v = parallel.shard_prompt(keys, values, plan)
    s = ref.build_summary(k, v, block_size=block)
    parallel.merge_max_value_norm(s.max_value_norm, seq_group)
    q = query[plan.head_lo:plan.head_hi]
    # stats exchange: one flat fp32 slab per rank
    part = ref.normalizer_partials(q, s).contiguous().view(-1)
    region = torch.zeros(seq * part.numel())
    region[plan.seq_rank * part.numel():(plan.seq_rank + 1) * part.numel()] = part
    parallel.all_gather_slabs(region, part.numel(), plan.seq_rank, seq_group)
    log_z, log_c = ref.merge_normalizers(region.view(seq, plan.heads, group, 4))
    sel, z = ref.select_blocks_given(q, s, log_z, log_c, eps, reduction)
    hs = slice(plan.head_lo, plan.head_hi)
    sk = ks[hs] if plan.holds_suffix else ks[hs, :0]
    sv = vs[hs] if plan.holds_suffix else vs[hs, :0]
    m, l, o = ref.mixed_attention_partial(q, s, sk, sv, sel, z)
    slab = torch.cat([m.view(-1), l.view(-1), o.reshape(-1)])
    region = torch.zeros(seq * slab.numel())
    region[plan.seq_rank * slab.numel():(plan.seq_rank + 1) * slab.numel()] = slab
    parallel.all_gather_slabs(region, slab.numel(), plan.seq_rank, seq_group)
    rows = plan.heads * group
    r = region.view(seq, -1)
    out = ref.merge_rank_outputs(r[:, :rows].view(seq, plan.heads, group),
                                 r[:, rows:2 * rows].view(seq, plan.heads, group),
                                 r[:, 2 * rows:].view(seq, plan.heads, group, -1))
    # one-process oracle of the same heads
    full = ref.build_summary(keys[hs], values[hs], block_size=block)
    want, want_mask = ref.sparse_attention(q, full, ks[hs], vs[hs], eps, reduction)
    margin = ref.margin_blocks(q, full, eps, reduction)
    mask_ok = bool(((sel == want_mask[:, plan.block_lo:plan.block_hi])
                    | margin[:, plan.block_lo:plan.block_hi]).all())
    exact = bool((sel == want_mask[:, plan.block_lo:plan.block_hi]).all())
    out_err = float((out - want.float()).abs().max())
    sparse = 0 < int(want_mask.sum()) < want_mask.numel()
    return mask_ok, exact, out_err, sparse


_CASES = {"exchange": _case_exchange, "split_decode": _case_split_decode}


def _run(case, world):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        mp.start_processes(_gloo_worker, args=(world, _free_port(), case, results), nprocs=world,
                           join=True, start_method="spawn")
        return [results[r] for r in range(world)]


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_slab_exchange_and_value_norm_merge(world):
    assert all(_run("exchange", world))


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_split_decode_matches_one_process(world):
    for mask_ok, exact, out_err, sparse in _run("split_decode", world):
        assert mask_ok and sparse
        if exact:
            assert out_err <= 1e-5

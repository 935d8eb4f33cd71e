"""Multi-GPU decode: KV heads sharded over ranks, prompt blocks split when GPUs outnumber heads.

The reference decodes one sequence on one GPU (``integrations/transformers.py:448-449``).
Every part of its decode step is independent per KV head -- summaries,
selection, anchors and attention all grid over ``kv_head`` -- so ranks that
own disjoint KV heads run the single-GPU path on their heads with no
collective at all.

When there are more ranks than KV heads (Qwen2.5-7B's 4 KV heads on 8 GPUs,
or a forced head x sequence grid), each head's prompt blocks are cut into
contiguous ranges over the ranks of a *sequence group*, and the decode step
then has two row-global reductions to exchange:

1. the selector normalisers log Z and log C (``reference.py:15-17``), which
   are log-sum-exps over all blocks of a head: each rank writes its phase-A
   (max, sum) partials into its slab of an exchange buffer and an all-gather
   gives every rank all slabs before the risks are evaluated, so masks are
   exactly the single-GPU masks up to the summation order of those sums;
2. the softmax over representatives, refined pages and the suffix: each rank
   combines its own sources into one (max, sum, normalised output) row per
   query row, a second all-gather shares the rows and an LSE merge gives
   every rank of the group the full output.

Both all-gathers move a few KB in place (``all_gather_into_tensor`` on slices
of one flat buffer), over NCCL on GPUs; the same helper runs on ``gloo`` CPU
tensors, which is how the host logic is tested without GPUs.  The generated
-token suffix lives on the last rank of each sequence group (the one holding
the prompt's tail).  Rank layout: ``rank = head_shard * seq_ranks + seq_rank``.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _native
from .attention import (AttentionResult, _buffer, _check_backend, _query_code, _scratch,
                        _validate, sparse_attention)
from .config import RefineKVConfig
from .summary import BlockSummary, build_summary


@dataclass(frozen=True)
class ShardPlan:
    """What one rank owns: a range of KV heads and, within them, a range of prompt blocks."""

    world: int
    rank: int
    head_shards: int  # groups of ranks that own disjoint KV heads
    seq_ranks: int    # ranks per head shard (1: no sequence split)
    head_shard: int
    seq_rank: int
    head_lo: int
    head_hi: int
    block_lo: int
    block_hi: int
    token_lo: int
    token_hi: int
    max_blocks: int   # largest block range of any rank of the group (sizes the exchange)
    holds_suffix: bool

    @property
    def heads(self) -> int:
        return self.head_hi - self.head_lo

    @property
    def blocks(self) -> int:
        return self.block_hi - self.block_lo

    @property
    def seq_group(self) -> tuple[int, ...]:
        """Global ranks that share this rank's heads, in sequence order."""
        first = self.head_shard * self.seq_ranks
        return tuple(range(first, first + self.seq_ranks))


def default_seq_ranks(kv_heads: int, world: int) -> int:
    """Ranks per sequence group: as few as possible, so that heads are split first."""
    return world // math.gcd(kv_heads, world)


def plan_shards(kv_heads: int, prompt_tokens: int, block_size: int, world: int, rank: int,
                seq_ranks: int | None = None) -> ShardPlan:
    """Place ``rank`` of ``world`` on a (head shard, sequence rank) grid.

    ``world = head_shards * seq_ranks``; ``head_shards`` must divide the KV
    heads.  Blocks are split as evenly as possible (``lo = r * blocks //
    seq_ranks``), so every rank gets at least one block when there are at
    least ``seq_ranks`` blocks.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError("need world >= 1 and 0 <= rank < world")
    if kv_heads < 1 or prompt_tokens < 1 or block_size < 1:
        raise ValueError("kv_heads, prompt_tokens and block_size must be positive")
    if seq_ranks is None:
        seq_ranks = default_seq_ranks(kv_heads, world)
    if seq_ranks < 1 or world % seq_ranks:
        raise ValueError(f"seq_ranks={seq_ranks} must divide world={world}")
    head_shards = world // seq_ranks
    if kv_heads % head_shards:
        raise ValueError(f"{head_shards} head shards must divide the {kv_heads} KV heads")
    blocks = -(-prompt_tokens // block_size)
    if blocks < seq_ranks:
        raise ValueError(f"{blocks} prompt blocks cannot be split over {seq_ranks} ranks")
    head_shard, seq_rank = divmod(rank, seq_ranks)
    per_shard = kv_heads // head_shards
    block_lo = seq_rank * blocks // seq_ranks
    block_hi = (seq_rank + 1) * blocks // seq_ranks
    return ShardPlan(
        world=world, rank=rank, head_shards=head_shards, seq_ranks=seq_ranks,
        head_shard=head_shard, seq_rank=seq_rank,
        head_lo=head_shard * per_shard, head_hi=(head_shard + 1) * per_shard,
        block_lo=block_lo, block_hi=block_hi,
        token_lo=block_lo * block_size, token_hi=min(block_hi * block_size, prompt_tokens),
        max_blocks=-(-blocks // seq_ranks), holds_suffix=seq_rank == seq_ranks - 1)


def new_seq_group(plan: ShardPlan, backend: str | None = None):
    """Create every sequence group (a collective call on all ranks) and return this rank's.

    Returns None when there is no sequence split.  ``torch.distributed``
    requires all ranks to create all groups in the same order.
    """
    if plan.seq_ranks == 1:
        return None
    mine = None
    for shard in range(plan.head_shards):
        ranks = list(range(shard * plan.seq_ranks, (shard + 1) * plan.seq_ranks))
        group = dist.new_group(ranks, backend=backend)
        if shard == plan.head_shard:
            mine = group
    return mine


def shard_prompt(keys: torch.Tensor, values: torch.Tensor, plan: ShardPlan):
    """This rank's (heads, tokens, dim) slices of the full prompt K/V (views, no copy)."""
    sl = (slice(plan.head_lo, plan.head_hi), slice(plan.token_lo, plan.token_hi))
    return keys[sl], values[sl]


def all_gather_slabs(region: torch.Tensor, slab: int, rank: int, group) -> None:
    """In-place all-gather of equal slabs: slab ``rank`` of the flat ``region`` goes to every rank."""
    if region.ndim != 1 or region.numel() % slab:
        raise ValueError("region must be a flat whole number of slabs")
    dist.all_gather_into_tensor(region, region[rank * slab:(rank + 1) * slab], group=group)


def merge_max_value_norm(max_value_norm: torch.Tensor, group) -> None:
    """All-reduce MAX of the per-head largest value norm over a sequence group (in place).

    The selector's distortion bound uses the head's largest value norm over
    the whole prompt (``summary.py:110``), not over one rank's blocks.
    """
    if group is not None:
        dist.all_reduce(max_value_norm, op=dist.ReduceOp.MAX, group=group)


def build_shard_summary(keys: torch.Tensor, values: torch.Tensor, config: RefineKVConfig,
                        plan: ShardPlan, group) -> BlockSummary:
    """Summaries of this rank's prompt blocks (``keys``/``values`` already sliced by ``shard_prompt``)."""
    if keys.shape[0] != plan.heads or keys.shape[1] != plan.token_hi - plan.token_lo:
        raise ValueError("keys must be this rank's slice of the prompt")
    summary = build_summary(keys, values, config)
    merge_max_value_norm(summary.max_value_norm, group)
    return summary


def exchange_slabs(heads: int, group: int, max_blocks: int, head_dim: int) -> tuple[int, int]:
    """Byte sizes of one rank's stats slab and output slab (``rkv_split_exchange_slabs``)."""
    lib = _native.load()
    stats, output = ctypes.c_size_t(), ctypes.c_size_t()
    _native.check(lib.rkv_split_exchange_slabs(heads, group, max_blocks, head_dim,
                                               ctypes.byref(stats), ctypes.byref(output)))
    return stats.value, output.value


@torch.no_grad()
def select_blocks_union_split(queries, summary: BlockSummary, config: RefineKVConfig,
                              plan: ShardPlan, group, *, workspace=None) -> torch.Tensor:
    """``select_blocks_union`` on a rank of a sequence group: this rank's blocks of the OR mask.

    ``queries`` is (anchors, kv_heads, group, 1, head_dim), the same on every
    rank of the group; the selector normalisers are merged over the group
    (``rkv_select_split``), so the mask equals the one-GPU mask's slice.
    """
    from .attention import select_blocks_union

    if plan.seq_ranks == 1:
        return select_blocks_union(queries, summary, config, workspace=workspace)
    if queries.ndim != 5 or queries.shape[3] != 1:
        raise ValueError("queries must have shape (anchors, kv_heads, group_size, 1, head_dim)")
    _validate(queries[0], summary, config)
    _check_backend(queries[0], config)
    count, heads, group_size, _, dim = queries.shape
    dev = queries.device
    q = queries.reshape(count, heads, group_size, dim).contiguous()
    mask = torch.empty(heads, summary.num_blocks, device=dev, dtype=torch.uint8)
    lib = _native.load()
    slab = lib.rkv_select_split_slab(heads, group_size, plan.max_blocks, count)
    if slab == 0:
        raise ValueError("selection geometry out of range")
    ranks = plan.seq_ranks
    with torch.cuda.device(dev):
        nbytes = lib.rkv_select_workspace_size(heads, group_size, summary.num_blocks, dim, count)
        scratch = _scratch(workspace, f"rkv_select_scratch_{count}", nbytes, dev)
        exchange = _scratch(workspace, f"rkv_select_exchange_{count}", ranks * slab, dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        args = (summary.abi(), q.data_ptr(), _query_code(q), count, group_size, config.eps,
                _native.GQA_CODES[config.gqa_reduction], mask.data_ptr(), 0, scratch.data_ptr(),
                scratch.numel(), ranks, plan.seq_rank, plan.max_blocks, exchange.data_ptr(),
                exchange.numel())
        _native.check(lib.rkv_select_split(*args, _native.SPLIT_STATS, stream))
        all_gather_slabs(exchange[:ranks * slab], slab, plan.seq_rank, group)
        _native.check(lib.rkv_select_split(*args, _native.SPLIT_FINAL, stream))
    return mask.view(torch.bool)


class SplitDecode:
    """One layer's decode step on a rank of a sequence group.

    Same call as :func:`refinekv_b200.sparse_attention`, run by every rank of
    the group with its own summary; the returned output (every rank gets the
    group's full output for its heads) lives in ``workspace`` and is reused by
    the next call.  ``selected`` covers this rank's blocks.  Only the rank
    with ``plan.holds_suffix`` passes suffix K/V (the others pass None).
    Without a sequence split (``plan.seq_ranks == 1``) this is exactly
    ``sparse_attention``.  All calls are stream-ordered and allocation-free
    after the first, so a step can be captured in a CUDA graph (NCCL
    collectives included).
    """

    def __init__(self, plan: ShardPlan, group):
        if plan.seq_ranks > 1 and group is None:
            raise ValueError("a sequence split needs the sequence group")
        self.plan = plan
        self.group = group

    @torch.no_grad()
    def __call__(self, query, summary: BlockSummary, key_suffix, value_suffix,
                 config: RefineKVConfig | None = None, *, anchor_mask=None, workspace=None,
                 return_selected=False, suffix_length=None) -> AttentionResult:
        plan = self.plan
        config = config or RefineKVConfig(block_size=summary.block_size)
        if plan.seq_ranks == 1:
            return sparse_attention(query, summary, key_suffix, value_suffix, config,
                                    anchor_mask=anchor_mask, workspace=workspace,
                                    return_selected=return_selected, suffix_length=suffix_length)
        if workspace is None:
            raise ValueError("a sequence-split decode needs a workspace dict")
        _validate(query, summary, config, anchor_mask)
        _check_backend(query, config)
        if summary.num_blocks != plan.blocks:
            raise ValueError("summary must cover this rank's blocks")
        has_suffix = key_suffix is not None and key_suffix.shape[1] > 0
        if has_suffix and not plan.holds_suffix:
            raise ValueError("only the last rank of a sequence group holds the suffix")
        heads, group_size, _, dim = query.shape
        dev = query.device
        q = query.reshape(heads, group_size, dim).contiguous()
        capacity = key_suffix.shape[1] if has_suffix else 0
        if has_suffix:
            if key_suffix.shape != value_suffix.shape or key_suffix.shape[0] != heads:
                raise ValueError("suffix K/V must have matching (kv_heads, tokens, head_dim) shapes")
            if key_suffix.dtype != torch.bfloat16 or value_suffix.dtype != torch.bfloat16:
                raise TypeError("the CUDA backend requires BF16 suffix K/V")
            if key_suffix.stride(-1) != 1:
                key_suffix = key_suffix.contiguous()
            if value_suffix.stride(-1) != 1:
                value_suffix = value_suffix.contiguous()
        if suffix_length is not None and (suffix_length.shape != () or suffix_length.dtype != torch.int32
                                          or suffix_length.device != dev):
            raise ValueError("suffix_length must be a scalar int32 tensor on the query device")
        anchor = None
        if anchor_mask is not None:
            anchor = anchor_mask if anchor_mask.is_contiguous() else anchor_mask.contiguous()
        output = _buffer(workspace, "output", (heads, group_size, dim), dev, query.dtype)
        selected = _buffer(workspace, "selected", (heads, summary.num_blocks), dev, torch.uint8)
        stats_slab, output_slab = exchange_slabs(heads, group_size, plan.max_blocks, dim)
        ranks = plan.seq_ranks
        lib = _native.load()
        with torch.cuda.device(dev):
            nbytes = lib.rkv_decode_workspace_size(heads, group_size, summary.num_blocks, dim,
                                                   summary.block_size)
            scratch = _scratch(workspace, "rkv_decode_scratch", nbytes, dev)
            exchange = _scratch(workspace, "rkv_split_exchange", ranks * (stats_slab + output_slab),
                                dev)
            stream = torch.cuda.current_stream(dev).cuda_stream
            args = (summary.abi(), q.data_ptr(), _query_code(q), group_size,
                    key_suffix.data_ptr() if capacity else None,
                    value_suffix.data_ptr() if capacity else None, capacity,
                    key_suffix.stride(0) if capacity else 0, key_suffix.stride(1) if capacity else 0,
                    value_suffix.stride(0) if capacity else 0,
                    value_suffix.stride(1) if capacity else 0,
                    suffix_length.data_ptr() if (suffix_length is not None and capacity) else None,
                    capacity, anchor.data_ptr() if anchor is not None else None, config.eps,
                    _native.GQA_CODES[config.gqa_reduction], output.data_ptr(),
                    selected.data_ptr(), scratch.data_ptr(), scratch.numel(), ranks,
                    plan.seq_rank, plan.max_blocks, exchange.data_ptr(), exchange.numel())
            _native.check(lib.rkv_decode_split(*args, _native.SPLIT_STATS, stream))
            all_gather_slabs(exchange[:ranks * stats_slab], stats_slab, plan.seq_rank, self.group)
            _native.check(lib.rkv_decode_split(*args, _native.SPLIT_ATTEND, stream))
            all_gather_slabs(exchange[ranks * stats_slab:ranks * (stats_slab + output_slab)],
                             output_slab, plan.seq_rank, self.group)
            _native.check(lib.rkv_decode_split(*args, _native.SPLIT_MERGE, stream))
        return AttentionResult(output.view(heads, group_size, 1, dim),
                               selected.view(torch.bool).clone() if return_selected else None)

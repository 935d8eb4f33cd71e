"""Batched decode: several prompts stacked on the head axis (needs a B200).

No reference counterpart (the reference decodes one sequence,
``transformers.py:448-449``); the bar is the reference algorithm applied to
each prompt alone: every sequence's rows of a batched summary equal its own
``build_summary`` bit for bit, and a batched decode gives each sequence the
oracle's mask (outside the eps margin) and output (the parity tolerances of
``test_gpu_parity``).  Pages past a shorter prompt are never selected.
"""

import pytest
import torch

from oracle import refinekv_oracle as ora
from refinekv_b200 import (RefineKVConfig, build_summary, build_summary_batch, sparse_attention,
                           synthetic)
from refinekv_b200.attention import device_status, select_blocks_union
from test_gpu_parity import check_mask, check_output

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _prompts(lengths, heads, dim, seed=5):
    return [synthetic.make_layer(seed, i, heads, n, dim, 32, device=DEV)
            for i, n in enumerate(lengths)]


def _queries(layers, group, scale, step=0, count=None):
    qs = [synthetic.make_queries(7, i, step, d.planted_mean, group, count or 1)
          for i, d in enumerate(layers)]
    q = torch.cat(qs, dim=1).float() * scale  # (count, sequences*heads, group, 1, dim)
    return q.to(torch.bfloat16) if count else q[0].to(torch.bfloat16)


@pytest.mark.parametrize("lengths,heads,dim", [
    ((1000, 4096, 2529), 2, 128),
    ((64, 33, 97, 2048), 4, 64),
    ((3000, 3000), 2, 256),
])
def test_batched_rows_equal_single_summaries(lengths, heads, dim):
    layers = _prompts(lengths, heads, dim)
    cfg = RefineKVConfig()
    batch = build_summary_batch([d.keys for d in layers], [d.values for d in layers], cfg)
    blocks = -(-max(lengths) // 32)
    assert batch.sequences == len(lengths) and batch.num_blocks == blocks
    assert batch.prompt_lengths.tolist() == list(lengths)
    for i, d in enumerate(layers):
        one = build_summary(d.keys, d.values, cfg)
        rows, nb = slice(i * heads, (i + 1) * heads), one.num_blocks
        assert torch.equal(batch.counts[i, :nb], one.counts)
        assert not batch.counts[i, nb:].any()
        for name in ("key_mean", "value_mean", "ellipsoid", "value_norm"):
            got = getattr(batch, name)[rows]
            assert torch.equal(got[:, :nb], getattr(one, name)), name
            assert not got[:, nb:].any(), name
        assert torch.equal(batch.max_value_norm[rows], one.max_value_norm)
        assert torch.equal(batch.keys[rows, :nb], one.keys.contiguous())
        assert torch.equal(batch.values[rows, :nb], one.values.contiguous())


@pytest.mark.parametrize("lengths,heads,group,dim,reduction,scale,anchors,partial", [
    ((1000, 4096, 2529), 2, 4, 128, "any", 8.0, 0, True),
    ((1000, 4096, 2529), 2, 4, 128, "mean", 2.0, 4, True),
    ((64, 33, 2048, 700), 4, 8, 64, "max", 4.0, 2, True),
    ((3000, 1500), 2, 16, 256, "any", 4.0, 3, False),  # 16 rows x "any": every page refined
])
def test_batched_decode_matches_each_sequence(lengths, heads, group, dim, reduction, scale,
                                              anchors, partial):
    layers = _prompts(lengths, heads, dim)
    cfg = RefineKVConfig(eps=0.05, gqa_reduction=reduction)
    batch = build_summary_batch([d.keys for d in layers], [d.values for d in layers], cfg)
    rows = len(lengths) * heads
    q = _queries(layers, group, scale)
    gen = torch.Generator(device=DEV).manual_seed(3)
    cap, visible = 48, 37
    ks = torch.randn(rows, cap, dim, device=DEV, generator=gen).to(torch.bfloat16)
    vs = torch.randn(rows, cap, dim, device=DEV, generator=gen).to(torch.bfloat16)
    length = torch.full((), visible, device=DEV, dtype=torch.int32)
    anchor = None
    if anchors:
        aq = _queries(layers, group, scale, step=-1, count=anchors)
        anchor = select_blocks_union(aq, batch, cfg)
    ws = {}
    res = sparse_attention(q, batch, ks, vs, cfg, anchor_mask=anchor, workspace=ws,
                           return_selected=True, suffix_length=length)
    assert device_status(ws) == 0
    refined = 0
    for i, d in enumerate(layers):
        r = slice(i * heads, (i + 1) * heads)
        one = ora.build_summary(d.keys.cpu(), d.values.cpu(), 32)
        nb = one.counts.numel()
        assert not res.selected[r, nb:].any()  # padding pages are never selected
        anchor_i = None
        if anchor is not None:
            assert not anchor[r, nb:].any()
            want_anchor = ora.anchor_union(aq[:, r].cpu(), one, cfg.eps, cfg.gqa_reduction)
            margin = ora.margin_blocks(aq[0, r].cpu(), one, cfg.eps, cfg.gqa_reduction)
            for a in range(1, anchors):
                margin |= ora.margin_blocks(aq[a, r].cpu(), one, cfg.eps, cfg.gqa_reduction)
            assert not ((anchor[r, :nb].cpu() != want_anchor) & ~margin).any()
            anchor_i = anchor[r, :nb]
        want, z, _ = check_mask(res.selected[r, :nb], q[r], one, cfg, anchor_i)
        refined += int(want.sum())
        check_output(res.output[r], q[r], one, ks[r, :visible], vs[r, :visible],
                     res.selected[r, :nb].cpu(), z)
    total = sum(-(-n // 32) for n in lengths) * heads
    assert 0 < refined <= total and (refined < total) == partial


def test_batched_and_single_decode_agree_on_equal_prompts():
    """Two copies of one prompt in a batch decode identically, and like the prompt alone."""
    (d,) = _prompts((2500,), 2, 128)
    cfg = RefineKVConfig(eps=0.05)
    one = build_summary(d.keys, d.values, cfg)
    batch = build_summary_batch([d.keys, d.keys], [d.values, d.values], cfg)
    q1 = (synthetic.make_queries(7, 0, 0, d.planted_mean, 4)[0].float() * 4).to(torch.bfloat16)
    q = torch.cat([q1, q1])
    ks = torch.zeros(4, 8, 128, device=DEV, dtype=torch.bfloat16)
    single = sparse_attention(q1, one, ks[:2, :0], ks[:2, :0], cfg, return_selected=True)
    both = sparse_attention(q, batch, ks[:, :0], ks[:, :0], cfg, return_selected=True)
    # Same per-row selector partitioning: the same decisions.  The attention
    # work list cuts the two copies' pages differently over the CTAs, so the
    # outputs agree to rounding.
    assert torch.equal(both.selected[:2], both.selected[2:])
    torch.testing.assert_close(both.output[:2].float(), both.output[2:].float(),
                               atol=2e-3, rtol=1e-2)
    margin = ora.margin_blocks(q1.cpu(), ora.as_cpu_summary(one), cfg.eps, cfg.gqa_reduction)
    assert not ((both.selected[:2].cpu() != single.selected.cpu()) & ~margin).any()
    torch.testing.assert_close(both.output[:2].float(), single.output.float(),
                               atol=4e-3, rtol=2e-2)

"""Decode from a vLLM-style K/V page pool through a page table (needs a B200).

No reference counterpart (the reference keeps one contiguous cache per
layer).  The pages a selection refines are the same bytes wherever they
live, so a decode from a pool with the prompt's pages scattered over it
(HND and NHD pools, garbage in every other page) must equal the decode from
the summary's own contiguous pages bit for bit; the same holds for a ragged
batch sharing one pool.
"""

import pytest
import torch

from refinekv_b200 import (RefineKVConfig, attach_page_pool, build_summary, build_summary_batch,
                           sparse_attention, synthetic)
from refinekv_b200.attention import device_status, select_blocks_union

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _pool(page_lists, heads, block, dim, spare, layout, seed=11):
    """A pool holding each sequence's (heads, pages, block, dim) pages at random slots."""
    gen = torch.Generator(device=DEV).manual_seed(seed)
    total = sum(p.shape[1] for p in page_lists) + spare
    shape = (total, heads, block, dim) if layout == "HND" else (total, block, heads, dim)
    pool = torch.randn(shape, device=DEV, generator=gen).to(torch.bfloat16)  # garbage elsewhere
    slots = torch.randperm(total, device=DEV, generator=gen)
    width = max(p.shape[1] for p in page_lists)
    table = torch.full((len(page_lists), width + 3), -1, device=DEV, dtype=torch.int32)
    at = 0
    for i, pages in enumerate(page_lists):
        n = pages.shape[1]
        phys = slots[at:at + n]
        at += n
        table[i, :n] = phys.to(torch.int32)
        if layout == "HND":
            pool[phys] = pages.permute(1, 0, 2, 3)
        else:
            pool[phys] = pages.permute(1, 2, 0, 3)
    return pool, table


def _decode(summary, q, ks, vs, cfg, anchor=None, length=None):
    ws = {}
    res = sparse_attention(q, summary, ks, vs, cfg, anchor_mask=anchor, workspace=ws,
                           return_selected=True, suffix_length=length)
    assert device_status(ws) == 0
    return res.output.view(torch.int16).clone(), res.selected.clone()


@pytest.mark.parametrize("layout", ["HND", "NHD"])
@pytest.mark.parametrize("tokens,heads,group,dim,scale", [
    (4096, 2, 4, 128, 8.0), (3000, 4, 8, 64, 4.0), (2113, 2, 16, 256, 16.0)])
def test_pool_decode_equals_contiguous_decode(layout, tokens, heads, group, dim, scale):
    d = synthetic.make_layer(2, 0, heads, tokens, dim, 32, device=DEV)
    cfg = RefineKVConfig(eps=0.05)
    summary = build_summary(d.keys, d.values, cfg)
    kpool, table = _pool([summary.keys.contiguous()], heads, 32, dim, 37, layout)
    vpool = torch.zeros_like(kpool)  # V pages at the K pages' slots
    phys = table[0, :summary.num_blocks].long()
    src = summary.values.contiguous()
    vpool[phys] = src.permute(1, 0, 2, 3) if layout == "HND" else src.permute(1, 2, 0, 3)
    paged = attach_page_pool(summary, kpool, vpool, table[0], layout)
    q = (synthetic.make_queries(2, 0, 0, d.planted_mean, group)[0].float() * scale).to(
        torch.bfloat16)
    gen = torch.Generator(device=DEV).manual_seed(4)
    ks = torch.randn(heads, 24, dim, device=DEV, generator=gen).to(torch.bfloat16)
    vs = torch.randn(heads, 24, dim, device=DEV, generator=gen).to(torch.bfloat16)
    length = torch.full((), 17, device=DEV, dtype=torch.int32)
    anchor = select_blocks_union(
        synthetic.make_queries(2, 0, -1, d.planted_mean, group, 3), summary, cfg)
    want = _decode(summary, q, ks, vs, cfg, anchor, length)
    got = _decode(paged, q, ks, vs, cfg, anchor, length)
    assert 0 < int(want[1].sum())
    assert torch.equal(got[1], want[1]) and torch.equal(got[0], want[0])


def test_ragged_batch_in_one_pool_equals_padded_batch():
    heads, dim, lengths = 2, 128, (1000, 4096, 2529)
    layers = [synthetic.make_layer(5, i, heads, n, dim, 32, device=DEV) for i, n in enumerate(lengths)]
    cfg = RefineKVConfig(eps=0.05)
    batch = build_summary_batch([d.keys for d in layers], [d.values for d in layers], cfg)
    pages_k = [batch.keys[i * heads:(i + 1) * heads, :-(-n // 32)] for i, n in enumerate(lengths)]
    pages_v = [batch.values[i * heads:(i + 1) * heads, :-(-n // 32)] for i, n in enumerate(lengths)]
    kpool, table = _pool(pages_k, heads, 32, dim, 11, "HND")
    vpool = torch.zeros_like(kpool)
    for i, pv in enumerate(pages_v):
        vpool[table[i, :pv.shape[1]].long()] = pv.permute(1, 0, 2, 3)
    paged = attach_page_pool(batch, kpool, vpool, table, "HND")
    q = torch.cat([(synthetic.make_queries(7, i, 0, d.planted_mean, 4)[0].float() * 8)
                   for i, d in enumerate(layers)]).to(torch.bfloat16)
    ks = torch.zeros(len(lengths) * heads, 8, dim, device=DEV, dtype=torch.bfloat16)
    want = _decode(batch, q, ks[:, :0], ks[:, :0], cfg)
    got = _decode(paged, q, ks[:, :0], ks[:, :0], cfg)
    assert torch.equal(got[1], want[1]) and torch.equal(got[0], want[0])


def test_out_of_range_page_sets_the_status_word():
    d = synthetic.make_layer(2, 0, 2, 1024, 128, 32, device=DEV)
    cfg = RefineKVConfig(eps=0.0)  # every page refined
    summary = build_summary(d.keys, d.values, cfg)
    pool = torch.zeros(40, 2, 32, 128, device=DEV, dtype=torch.bfloat16)
    table = torch.arange(32, device=DEV, dtype=torch.int32)
    table[5] = 40  # one past the pool
    paged = attach_page_pool(summary, pool, pool, table, "HND")
    q = synthetic.make_queries(2, 0, 0, d.planted_mean, 4)[0]
    none = torch.zeros(2, 0, 128, device=DEV, dtype=torch.bfloat16)
    ws = {}
    res = sparse_attention(q, paged, none, none, cfg, workspace=ws, return_selected=True)
    assert bool(res.selected[:, 5].all())  # the bad page was refined
    assert device_status(ws) & 2

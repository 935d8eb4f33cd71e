"""The one-kernel decode against the four-kernel decode and the oracle (needs a B200).

rkv_decode runs, by default, one kernel per layer and step: the selector's
two phases (a per-row barrier between them), every page the step needs, the
representatives and the combine (a second per-row barrier).
rkv_set_fused_selector(0) switches back to the stats, final, attention and
combine kernels.  Both paths must give the same masks outside the eps margin
and outputs within the parity tolerance (bf16: atol 4e-3 + rtol 2e-2, max-abs
2e-2; fp32 queries: 1e-4), and each must match the oracle.
"""

import contextlib

import pytest
import torch

from oracle import refinekv_oracle as ora
from refinekv_b200 import (RefineKVConfig, _native, attach_page_pool, build_summary,
                           sparse_attention, synthetic)
from refinekv_b200.attention import device_status, select_blocks_union

pytestmark = pytest.mark.gpu
DEV = "cuda"


@contextlib.contextmanager
def unfused():
    lib = _native.load()
    lib.rkv_set_fused_selector(0)
    try:
        yield
    finally:
        lib.rkv_set_fused_selector(1)


def _close(a, b, fp32):
    if fp32:
        torch.testing.assert_close(a.float(), b.float(), atol=1e-4, rtol=0)
    else:
        torch.testing.assert_close(a.float(), b.float(), atol=4e-3, rtol=2e-2)
        assert float((a.float() - b.float()).abs().max()) <= 2e-2


@pytest.mark.parametrize("heads,group,dim,block,tokens,scale,anchors,qdtype", [
    (8, 4, 128, 32, 65536, 1.0, 32, torch.bfloat16),   # every page anchored and refined
    (8, 4, 128, 32, 65536, 16.0, 8, torch.bfloat16),   # sharp queries: few pages, many reps
    (4, 7, 128, 64, 40000, 4.0, 16, torch.bfloat16),   # Qwen-like group, 64-token pages
    (2, 16, 256, 16, 9000, 2.0, 4, torch.float32),     # two n8 tiles, fp32 queries
    (1, 8, 64, 32, 131072, 8.0, 0, torch.bfloat16),    # one head: one tile per CTA, no anchors
    (3, 2, 96, 32, 777, 1.0, 2, torch.bfloat16),       # padded head dim, ragged tail
])
def test_fused_and_two_kernel_selectors_agree_and_match_the_oracle(
        heads, group, dim, block, tokens, scale, anchors, qdtype):
    data = synthetic.make_layer(11, 0, heads, tokens, dim, block, device=DEV)
    cfg = RefineKVConfig(block_size=block, eps=0.01, anchor_tokens=anchors)
    summary = build_summary(data.keys, data.values, cfg)
    lib = _native.load()
    assert lib.rkv_decode_kernel_count(heads, group, summary.num_blocks, dim, block) == 1
    anchor = None
    if anchors:
        aq = synthetic.make_queries(11, 0, -1, data.planted_mean, group, anchors)
        anchor = select_blocks_union(aq, summary, cfg)
    q = (synthetic.make_queries(11, 0, 0, data.planted_mean, group)[0].float() * scale).to(qdtype)
    gen = torch.Generator(device=DEV).manual_seed(5)
    ks = torch.randn(heads, 19, dim, device=DEV, generator=gen).to(torch.bfloat16)
    vs = torch.randn(heads, 19, dim, device=DEV, generator=gen).to(torch.bfloat16)
    ws = {}
    fused = sparse_attention(q, summary, ks, vs, cfg, anchor_mask=anchor, workspace=ws,
                             return_selected=True)
    fused_out, fused_sel = fused.output.clone(), fused.selected.clone()
    assert device_status(ws) == 0
    with unfused():
        assert lib.rkv_decode_kernel_count(heads, group, summary.num_blocks, dim, block) == 4
        ws2 = {}
        plain = sparse_attention(q, summary, ks, vs, cfg, anchor_mask=anchor, workspace=ws2,
                                 return_selected=True)
        assert device_status(ws2) == 0
    s_cpu = ora.as_cpu_summary(summary)
    margin = ora.margin_blocks(q.cpu(), s_cpu, cfg.eps, cfg.gqa_reduction)
    if anchor is not None:
        margin &= ~anchor.cpu()
    assert not ((fused_sel.cpu() != plain.selected.cpu()) & ~margin).any()
    _close(fused_out, plain.output, qdtype == torch.float32)
    want, z = ora.select_blocks(q.cpu(), s_cpu, cfg.eps, cfg.gqa_reduction)
    if anchor is not None:
        want |= anchor.cpu()
    assert not ((fused_sel.cpu() != want) & ~margin).any()
    ref = ora.mixed_attention(q.cpu(), s_cpu, ks.cpu(), vs.cpu(), fused_sel.cpu(), z)
    _close(fused_out.cpu(), ref if qdtype == torch.float32 else ref.to(torch.bfloat16),
           qdtype == torch.float32)


def test_fused_selector_with_a_batch_and_a_page_pool():
    """Ragged batch (padding pages never selected) decoding from an HND page pool."""
    from refinekv_b200 import build_summary_batch

    heads, group, dim, block = 4, 4, 128, 32
    lengths = [5000, 12345, 777]
    cfg = RefineKVConfig(eps=0.01, anchor_tokens=4)
    layers = [synthetic.make_layer(20 + i, 0, heads, n, dim, block, device=DEV)
              for i, n in enumerate(lengths)]
    summary = build_summary_batch([d.keys for d in layers], [d.values for d in layers], cfg)
    aq = torch.cat([synthetic.make_queries(20 + i, 0, -1, d.planted_mean, group, 4)
                    for i, d in enumerate(layers)], dim=1)
    anchor = select_blocks_union(aq, summary, cfg)
    q = torch.cat([synthetic.make_queries(20 + i, 0, 0, d.planted_mean, group)[0]
                   for i, d in enumerate(layers)])
    gen = torch.Generator(device=DEV).manual_seed(6)
    ks = torch.randn(len(lengths) * heads, 7, dim, device=DEV, generator=gen).to(torch.bfloat16)
    vs = torch.randn(len(lengths) * heads, 7, dim, device=DEV, generator=gen).to(torch.bfloat16)
    # the same pages scattered over a pool
    nb = summary.num_blocks
    pool_pages = len(lengths) * nb + 5
    perm = torch.randperm(pool_pages, generator=torch.Generator().manual_seed(1))[
        :len(lengths) * nb].view(len(lengths), nb).to(torch.int32)
    key_pool = torch.randn(pool_pages, heads, block, dim, device=DEV).to(torch.bfloat16)
    value_pool = torch.randn_like(key_pool)
    for i in range(len(lengths)):
        rows = slice(i * heads, (i + 1) * heads)
        key_pool[perm[i].long()] = summary.keys[rows].permute(1, 0, 2, 3)
        value_pool[perm[i].long()] = summary.values[rows].permute(1, 0, 2, 3)
    paged = attach_page_pool(summary, key_pool, value_pool, perm.to(DEV), "HND")
    outs = []
    for s in (summary, paged):
        for fused in (True, False):
            ctx = contextlib.nullcontext() if fused else unfused()
            with ctx:
                ws = {}
                res = sparse_attention(q, s, ks, vs, cfg, anchor_mask=anchor, workspace=ws,
                                       return_selected=True)
                assert device_status(ws) == 0
                outs.append((res.output.clone(), res.selected.clone()))
    ref_out, ref_sel = outs[0]
    counts = summary.counts.repeat_interleave(heads, 0)
    assert not (ref_sel & (counts == 0)).any()  # padding pages are never selected
    assert torch.equal(outs[2][0], ref_out) and torch.equal(outs[2][1], ref_sel)  # paged, fused
    for out, sel in outs[1::2]:
        torch.testing.assert_close(out.float(), ref_out.float(), atol=4e-3, rtol=2e-2)


def test_one_workspace_across_geometries():
    """A workspace reused for another geometry (larger, then smaller) stays consistent:
    the barrier words live in a fixed header that no other region writes."""
    ws = {}
    for heads, tokens, group in ((8, 65536, 4), (2, 4000, 8), (8, 32768, 4), (8, 65536, 4)):
        data = synthetic.make_layer(30 + heads, 0, heads, tokens, 128, 32, device=DEV)
        summary = build_summary(data.keys, data.values)
        q = synthetic.make_queries(30 + heads, 0, 0, data.planted_mean, group)[0]
        empty = torch.empty(heads, 0, 128, device=DEV, dtype=torch.bfloat16)
        res = sparse_attention(q, summary, empty, empty, workspace=ws, return_selected=True)
        assert device_status(ws) == 0
        fresh = sparse_attention(q, summary, empty, empty, return_selected=True)
        assert torch.equal(res.selected, fresh.selected)
        assert torch.equal(res.output, fresh.output)


def test_rows_anchored_throughout_skip_the_statistics():
    """A row whose every block is anchored skips the selector statistics in every
    part; next to it, rows with one block or every third block left to decide
    and a row without anchors.  Masks and outputs against the oracle and the
    four-kernel decode."""
    heads, group, dim, block, tokens = 4, 4, 128, 32, 40000
    data = synthetic.make_layer(41, 0, heads, tokens, dim, block, device=DEV)
    cfg = RefineKVConfig(block_size=block, eps=0.01)
    summary = build_summary(data.keys, data.values, cfg)
    nb = summary.num_blocks
    anchor = torch.zeros(heads, nb, dtype=torch.bool, device=DEV)
    anchor[0] = True                  # every block: no statistics for this row
    anchor[1] = True
    anchor[1, nb // 2] = False        # one block to decide
    anchor[2, ::3] = True             # every third block
    q = (synthetic.make_queries(41, 0, 0, data.planted_mean, group)[0].float() * 8.0).to(
        torch.bfloat16)
    gen = torch.Generator(device=DEV).manual_seed(9)
    ks = torch.randn(heads, 5, dim, device=DEV, generator=gen).to(torch.bfloat16)
    vs = torch.randn(heads, 5, dim, device=DEV, generator=gen).to(torch.bfloat16)
    ws = {}
    res = sparse_attention(q, summary, ks, vs, cfg, anchor_mask=anchor, workspace=ws,
                           return_selected=True)
    out, sel = res.output.clone(), res.selected.clone()
    assert device_status(ws) == 0
    assert bool(sel[0].all()) and bool(sel[1].sum() >= nb - 1)
    with unfused():
        plain = sparse_attention(q, summary, ks, vs, cfg, anchor_mask=anchor, return_selected=True)
    s_cpu = ora.as_cpu_summary(summary)
    margin = ora.margin_blocks(q.cpu(), s_cpu, cfg.eps, cfg.gqa_reduction) & ~anchor.cpu()
    want, z = ora.select_blocks(q.cpu(), s_cpu, cfg.eps, cfg.gqa_reduction)
    want |= anchor.cpu()
    assert not ((sel.cpu() != want) & ~margin).any()
    assert not ((sel.cpu() != plain.selected.cpu()) & ~margin).any()
    _close(out, plain.output, False)
    ref = ora.mixed_attention(q.cpu(), s_cpu, ks.cpu(), vs.cpu(), sel.cpu(), z)
    _close(out.cpu(), ref.to(torch.bfloat16), False)


def test_ragged_batch_anchored_throughout():
    """Rows of a ragged batch anchored on every real block skip the statistics;
    their padding pages stay unselected (mask 0) and unread, and the result
    matches the four-kernel decode and, per prompt, the oracle."""
    from refinekv_b200 import build_summary_batch

    heads, group, dim, block = 4, 4, 128, 32
    lengths = [9000, 40000, 1234]
    cfg = RefineKVConfig(eps=0.01)
    layers = [synthetic.make_layer(50 + i, 0, heads, n, dim, block, device=DEV)
              for i, n in enumerate(lengths)]
    summary = build_summary_batch([d.keys for d in layers], [d.values for d in layers], cfg)
    counts = summary.counts.repeat_interleave(heads, 0)
    anchor = counts > 0                       # every real block of every row
    anchor[heads + 1, 7] = False              # one row of the second prompt keeps a decision
    q = torch.cat([synthetic.make_queries(50 + i, 0, 0, d.planted_mean, group)[0]
                   for i, d in enumerate(layers)])
    gen = torch.Generator(device=DEV).manual_seed(8)
    ks = torch.randn(len(lengths) * heads, 3, dim, device=DEV, generator=gen).to(torch.bfloat16)
    vs = torch.randn(len(lengths) * heads, 3, dim, device=DEV, generator=gen).to(torch.bfloat16)
    ws = {}
    res = sparse_attention(q, summary, ks, vs, cfg, anchor_mask=anchor, workspace=ws,
                           return_selected=True)
    out, sel = res.output.clone(), res.selected.clone()
    assert device_status(ws) == 0
    assert not (sel & (counts == 0)).any()
    assert bool((sel | (counts == 0)).sum(1)[[r for r in range(sel.shape[0]) if r != heads + 1]]
                .eq(sel.shape[1]).all())
    with unfused():
        plain = sparse_attention(q, summary, ks, vs, cfg, anchor_mask=anchor, return_selected=True)
    assert torch.equal(sel[:heads], plain.selected[:heads])
    _close(out, plain.output, False)
    for i, d in enumerate(layers):
        rows = slice(i * heads, (i + 1) * heads)
        nb = -(-lengths[i] // block)
        s_cpu = ora.as_cpu_summary(build_summary(d.keys, d.values, cfg))
        qi, ai = q[rows].cpu(), anchor[rows, :nb].cpu()
        margin = ora.margin_blocks(qi, s_cpu, cfg.eps, cfg.gqa_reduction) & ~ai
        want, z = ora.select_blocks(qi, s_cpu, cfg.eps, cfg.gqa_reduction)
        want |= ai
        assert not ((sel[rows, :nb].cpu() != want) & ~margin).any()
        ref = ora.mixed_attention(qi, s_cpu, ks[rows].cpu(), vs[rows].cpu(), sel[rows, :nb].cpu(), z)
        _close(out[rows].cpu(), ref.to(torch.bfloat16), False)

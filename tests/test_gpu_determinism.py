"""Decode is deterministic and free of launch-order races (needs a B200).

The decode kernels (the fused selector or the two selector kernels, the
attention, the combine) are chained with programmatic dependent launch:
each may start while its predecessor drains, and the combine reads the
selector's partials before its own dependency wait.  Whatever the overlap,
the result must be the same bits as running the phases one call at a time
with the device synchronised in between, and repeated calls (same or fresh
workspace) must repeat those bits.
"""

import pytest
import torch

from refinekv_b200 import RefineKVConfig, _native, build_summary, sparse_attention, synthetic
from refinekv_b200.attention import device_status, select_blocks_union

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _phases(summary, group):
    """The launches of one decode, one call each: the fused selector is one launch."""
    lib = _native.load()
    if lib.rkv_decode_kernel_count(summary.num_heads, group, summary.num_blocks,
                                   summary.keys.shape[-1], summary.block_size) == 3:
        return (_native.PHASE_STATS | _native.PHASE_FINAL, _native.PHASE_ATTEND,
                _native.PHASE_COMBINE)
    return (_native.PHASE_STATS, _native.PHASE_FINAL, _native.PHASE_ATTEND,
            _native.PHASE_COMBINE)


def _layer(heads, tokens, dim, group, scale):
    data = synthetic.make_layer(3, 1, heads, tokens, dim, 32, device=DEV)
    cfg = RefineKVConfig(eps=0.01, anchor_tokens=32)
    summary = build_summary(data.keys, data.values, cfg)
    anchors = select_blocks_union(
        synthetic.make_queries(3, 1, -1, data.planted_mean, group, 32), summary, cfg)
    q = (synthetic.make_queries(3, 1, 0, data.planted_mean, group)[0].float() * scale)
    gen = torch.Generator(device=DEV).manual_seed(17)
    ks = torch.randn(heads, 40, dim, device=DEV, generator=gen).to(torch.bfloat16)
    vs = torch.randn(heads, 40, dim, device=DEV, generator=gen).to(torch.bfloat16)
    return summary, anchors, q.to(torch.bfloat16), ks, vs, cfg


def _run(layer, ws, length, phases=(_native.PHASE_ALL,), sync=False):
    summary, anchors, q, ks, vs, cfg = layer
    for ph in phases:
        res = sparse_attention(q, summary, ks, vs, cfg, anchor_mask=anchors, workspace=ws,
                               return_selected=True, suffix_length=length, _phases=ph)
        if sync:
            torch.cuda.synchronize()
    assert device_status(ws) == 0
    return res.output.clone(), res.selected.clone()


@pytest.mark.parametrize("heads,tokens,dim,group,scale", [
    (8, 65536, 128, 4, 1.0),    # every page refined: attention-dominated
    (8, 65536, 128, 4, 16.0),   # sharp queries: few pages, many representatives
    (2, 131072, 64, 8, 8.0),    # few heads: long work ranges per CTA
    (4, 40960, 256, 16, 4.0),
])
def test_chained_decode_equals_synchronised_phases(heads, tokens, dim, group, scale):
    layer = _layer(heads, tokens, dim, group, scale)
    length = torch.full((), 33, device=DEV, dtype=torch.int32)
    ws = {}
    ref_out, ref_sel = _run(layer, ws, length, _phases(layer[0], group), sync=True)
    assert 0 < int(ref_sel.sum()) <= ref_sel.numel()
    for _ in range(3):  # same workspace, back to back without a sync
        out, sel = _run(layer, ws, length)
        assert torch.equal(sel, ref_sel)
        assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16))
    out, sel = _run(layer, {}, length)  # fresh workspace
    assert torch.equal(sel, ref_sel)
    assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16))

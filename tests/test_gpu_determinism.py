"""Decode is deterministic and free of launch-order races (needs a B200).

A decode step is one kernel (the default one-kernel decode, whose CTAs wait
for one another at two bounded per-row barriers) or four kernels chained with
programmatic dependent launch (a phase subset, or with the one-kernel decode
switched off).  The four phases run one call at a time, with the device
synchronised in between, must give the same mask as the chained step and its
output within an output rounding; repeated chained calls (same or fresh
workspace) must repeat their own bits exactly.
"""

import pytest
import torch

from refinekv_b200 import RefineKVConfig, _native, build_summary, sparse_attention, synthetic
from refinekv_b200.attention import device_status, select_blocks_union

pytestmark = pytest.mark.gpu
DEV = "cuda"


PHASES = (_native.PHASE_STATS, _native.PHASE_FINAL, _native.PHASE_ATTEND,
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
    # The four kernels one call at a time (a phase subset runs the multi-kernel
    # path), then the whole step chained (the one-kernel decode by default).
    ref_out, ref_sel = _run(layer, ws, length, PHASES, sync=True)
    assert 0 < int(ref_sel.sum()) <= ref_sel.numel()
    first_out, first_sel = _run(layer, ws, length)
    # The one-kernel decode sums the softmax partials in another order: the same
    # mask, the output within an output rounding of the multi-kernel path.
    assert torch.equal(first_sel, ref_sel)
    torch.testing.assert_close(first_out.float(), ref_out.float(), atol=4e-3, rtol=2e-2)
    for _ in range(3):  # same workspace, back to back without a sync
        out, sel = _run(layer, ws, length)
        assert torch.equal(sel, first_sel)
        assert torch.equal(out.view(torch.int16), first_out.view(torch.int16))
    out, sel = _run(layer, {}, length)  # fresh workspace
    assert torch.equal(sel, first_sel)
    assert torch.equal(out.view(torch.int16), first_out.view(torch.int16))

"""Dense decode on the refinement kernel (rkv_decode_dense; needs a B200).

``dense_attention`` attends to every prompt page of a KV cache (a page view,
no copy) and the suffix rows after it up to a device length: the dense
decode of the adapter's ``full_attention_layers`` (reference
``integrations/transformers.py:510-520``).  Judged against a plain PyTorch
fp32 softmax over the visible rows (rounded to bf16 first, as the reference
rounds K/V), with the parity tolerances: bf16 queries atol 4e-3 + rtol 2e-2
and max-abs 2e-2, fp32 queries 1e-4.
"""

import pytest
import torch

from refinekv_b200 import RefineKVConfig, build_summary, dense_attention, page_view
from refinekv_b200 import sparse_attention

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _reference(q, keys, values, visible):
    qf = q[:, :, 0].to(torch.bfloat16).float()
    k = keys[:, :visible].to(torch.bfloat16).float()
    v = values[:, :visible].to(torch.bfloat16).float()
    p = (qf @ k.transpose(1, 2) * q.shape[-1] ** -0.5).softmax(-1)
    return (p @ v).unsqueeze(2)


@pytest.mark.parametrize("heads,group,dim,block,tokens,suffix", [
    (8, 4, 128, 32, 5000, 37),
    (4, 7, 128, 64, 4097, 1),
    (2, 16, 256, 16, 777, 65),
    (3, 8, 64, 32, 64, 0),
    (1, 2, 96, 32, 1000, 5),
])
@pytest.mark.parametrize("qdtype", [torch.bfloat16, torch.float32])
def test_dense_attention_matches_a_plain_softmax(heads, group, dim, block, tokens, suffix, qdtype):
    gen = torch.Generator(device=DEV).manual_seed(tokens + dim)
    capacity = -(-(tokens + suffix + 3) // 64) * 64
    cache_k = torch.randn(heads, capacity, dim, device=DEV, generator=gen).to(torch.bfloat16)
    cache_v = torch.randn(heads, capacity, dim, device=DEV, generator=gen).to(torch.bfloat16)
    q = torch.randn(heads, group, 1, dim, device=DEV, generator=gen).to(qdtype)
    pages = page_view(cache_k, cache_v, tokens, block)
    length = torch.tensor(suffix, device=DEV, dtype=torch.int32)
    ws = {}
    got = dense_attention(q, pages, cache_k[:, tokens:], cache_v[:, tokens:], workspace=ws,
                          suffix_length=length)
    want = _reference(q, cache_k, cache_v, tokens + suffix)
    if qdtype == torch.float32:
        torch.testing.assert_close(got.float(), want, atol=1e-4, rtol=0)
    else:
        torch.testing.assert_close(got.float(), want.to(torch.bfloat16).float(), atol=4e-3,
                                   rtol=2e-2)
        assert float((got.float() - want).abs().max()) <= 2e-2
    # the host length over a sliced suffix gives the same bits
    again = dense_attention(q, pages, cache_k[:, tokens:tokens + suffix],
                            cache_v[:, tokens:tokens + suffix]).clone()
    assert torch.equal(again, got)
    assert int(ws["rkv_dense_scratch"][:4].view(torch.int32).item()) == 0


def test_dense_equals_refinement_with_every_block_selected():
    """eps = 0 selects every block: sparse_attention is then the same dense softmax."""
    gen = torch.Generator(device=DEV).manual_seed(3)
    heads, group, dim, tokens = 8, 4, 128, 8192
    cache_k = torch.randn(heads, tokens + 64, dim, device=DEV, generator=gen).to(torch.bfloat16)
    cache_v = torch.randn(heads, tokens + 64, dim, device=DEV, generator=gen).to(torch.bfloat16)
    q = torch.randn(heads, group, 1, dim, device=DEV, generator=gen).to(torch.bfloat16)
    ks, vs = cache_k[:, tokens:tokens + 9], cache_v[:, tokens:tokens + 9]
    dense = dense_attention(q, page_view(cache_k, cache_v, tokens), ks, vs).float()
    summary = build_summary(cache_k[:, :tokens], cache_v[:, :tokens])
    res = sparse_attention(q, summary, ks, vs, RefineKVConfig(eps=0.0), return_selected=True)
    assert bool(res.selected.all())
    assert float((res.output.float() - dense).abs().max()) <= 8e-3


def test_dense_attention_replays_from_a_cuda_graph():
    gen = torch.Generator(device=DEV).manual_seed(4)
    heads, group, dim, tokens, cap = 8, 4, 128, 3000, 32
    cache_k = torch.randn(heads, tokens + cap + 8, dim, device=DEV, generator=gen).to(torch.bfloat16)
    cache_v = torch.randn(heads, tokens + cap + 8, dim, device=DEV, generator=gen).to(torch.bfloat16)
    q = torch.randn(heads, group, 1, dim, device=DEV, generator=gen).to(torch.bfloat16)
    pages = page_view(cache_k, cache_v, tokens)
    length = torch.zeros((), device=DEV, dtype=torch.int32)
    ws = {}
    ks, vs = cache_k[:, tokens:tokens + cap], cache_v[:, tokens:tokens + cap]
    length.fill_(5)
    eager = dense_attention(q, pages, ks, vs, workspace=ws, suffix_length=length).clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = dense_attention(q, pages, ks, vs, workspace=ws, suffix_length=length)
    for n in (5, 17, 32):
        length.fill_(n)
        graph.replay()
        torch.cuda.synchronize()
        want = dense_attention(q, pages, ks[:, :n], vs[:, :n])
        assert torch.equal(out, want), n
    length.fill_(5)
    graph.replay()
    assert torch.equal(out, eager)

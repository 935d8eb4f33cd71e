"""Host logic of batched and paged summaries (no GPU): views, strides, validation."""

import pytest
import torch

from refinekv_b200.summary import BlockSummary, _stacked, attach_page_pool


def _summary(sequences=1, heads=2, blocks=5, dim=64, block=32):
    rows = sequences * heads
    z = torch.zeros
    return BlockSummary(z(rows, blocks, block, dim, dtype=torch.bfloat16),
                        z(rows, blocks, block, dim, dtype=torch.bfloat16),
                        z(sequences, blocks, dtype=torch.int64) if sequences > 1
                        else z(blocks, dtype=torch.int64),
                        z(rows, blocks, dim, dtype=torch.bfloat16),
                        z(rows, blocks, dim, dtype=torch.bfloat16),
                        z(rows, blocks, dim, dtype=torch.bfloat16),
                        z(rows, blocks), z(rows), blocks * block - 3, block,
                        sequences=sequences,
                        prompt_lengths=(torch.full((sequences,), blocks * block - 3)
                                        if sequences > 1 else None))


def test_stacked_views_a_batched_cache_and_copies_otherwise():
    cache = torch.arange(2 * 3 * 4 * 8, dtype=torch.float32).reshape(2, 3, 4, 8)
    view = _stacked(list(cache))
    assert view.data_ptr() == cache.data_ptr() and view.shape == (6, 4, 8)
    assert torch.equal(view, cache.reshape(6, 4, 8))
    a, b = torch.randn(3, 4, 8), torch.randn(3, 4, 8)
    copy = _stacked([a, b])
    assert copy.data_ptr() not in (a.data_ptr(), b.data_ptr())
    assert torch.equal(copy, torch.cat([a, b]))
    assert _stacked([cache[1], cache[0]]).data_ptr() != cache.data_ptr()  # out of order: copy


@pytest.mark.parametrize("layout", ["HND", "NHD"])
def test_pool_views_and_abi_strides(layout):
    s = _summary(sequences=2)
    pages, heads, block, dim = 11, 2, 32, 64
    shape = (pages, heads, block, dim) if layout == "HND" else (pages, block, heads, dim)
    kpool = torch.zeros(shape, dtype=torch.bfloat16)
    vpool = torch.zeros(shape, dtype=torch.bfloat16)
    table = torch.zeros(2, 7, dtype=torch.int32)
    paged = attach_page_pool(s, kpool, vpool, table, layout)
    assert paged.keys.shape == (heads, pages, block, dim)
    assert paged.num_heads == 4 and paged.num_blocks == 5
    a = paged.abi()
    assert a.key_pages == kpool.data_ptr() and a.page_table == table.data_ptr()
    assert (a.heads, a.sequences, a.page_table_stride, a.pool_pages) == (4, 2, 7, pages)
    if layout == "HND":
        assert (a.key_page_stride, a.key_page_head_stride, a.key_token_stride) == (
            heads * block * dim, block * dim, dim)
    else:
        assert (a.key_page_stride, a.key_page_head_stride, a.key_token_stride) == (
            block * heads * dim, dim, heads * dim)
    # element (page p, head h, row t, channel c) of the pool is where the ABI says
    flat = kpool.view(-1)
    p_, h_, t_, c_ = 7, 1, 5, 3
    idx = p_ * a.key_page_stride + h_ * a.key_page_head_stride + t_ * a.key_token_stride + c_
    flat[idx] = 1.0
    assert float(paged.keys[h_, p_, t_, c_]) == 1.0


def test_unpaged_summary_abi_has_no_page_table():
    a = _summary().abi()
    assert not a.page_table and a.sequences == 1 and a.heads == 2


@pytest.mark.parametrize("bad", [
    dict(layout="XYZ"),
    dict(table=torch.zeros(1, 7, dtype=torch.int32)),        # one row for two sequences
    dict(table=torch.zeros(2, 4, dtype=torch.int32)),        # narrower than the blocks
    dict(table=torch.zeros(2, 7, dtype=torch.int64)),        # not int32
    dict(kpool=torch.zeros(11, 3, 32, 64, dtype=torch.bfloat16)),   # wrong head count
    dict(kpool=torch.zeros(11, 2, 16, 64, dtype=torch.bfloat16)),   # wrong block size
    dict(kpool=torch.zeros(11, 2, 32, 64)),                           # not bf16
])
def test_pool_validation(bad):
    s = _summary(sequences=2)
    kpool = bad.get("kpool", torch.zeros(11, 2, 32, 64, dtype=torch.bfloat16))
    vpool = torch.zeros(kpool.shape, dtype=kpool.dtype)
    table = bad.get("table", torch.zeros(2, 7, dtype=torch.int32))
    with pytest.raises((ValueError, TypeError)):
        attach_page_pool(s, kpool, vpool, table, bad.get("layout", "HND"))

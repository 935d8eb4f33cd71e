"""rkv_decode_static: decode for callers that cannot allocate device memory.

Some callers of this library cannot hand it a device workspace: a host that
reaches the library only through its C ABI and has no device allocator of its
own, or a serving stack that has partitioned all device memory before decoding
starts and may not allocate afterwards.  rkv_decode_static runs the same kernels as
rkv_decode but takes its scratch from one fixed array inside the library.

These tests call it through the C ABI and require the same results as the
workspace entry point (through refinekv_b200.sparse_attention) on two
consecutive calls, the second of which reuses the array after the first.  The
file is named so that pytest collects it last; it also passes on its own in a
fresh process, where the first call performs the one-time address lookup.
"""

import ctypes

import pytest
import torch

from refinekv_b200 import RefineKVConfig, _native, build_summary, sparse_attention, synthetic

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _static_status():
    """The device status word of the last rkv_decode_static call, read without allocating in C."""
    lib = _native.load()
    word = torch.full((1,), -1, device=DEV, dtype=torch.int32)
    _native.check(lib.rkv_decode_static_status(word.data_ptr(),
                                               torch.cuda.current_stream().cuda_stream))
    return int(word.item())


def _decode_static(q, summary, ks, vs, cfg, out, selected):
    lib = _native.load()
    heads, group, _, dim = q.shape
    rc = lib.rkv_decode_static(
        summary.abi(), q.data_ptr(),
        _native.DTYPE_F32 if q.dtype == torch.float32 else _native.DTYPE_BF16, group,
        ks.data_ptr(), vs.data_ptr(), ks.shape[1], ks.stride(0), ks.stride(1),
        vs.stride(0), vs.stride(1), None, ks.shape[1], None, cfg.eps,
        _native.GQA_CODES[cfg.gqa_reduction], out.data_ptr(), selected.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    _native.check(rc)


@pytest.mark.parametrize("qdtype", [torch.bfloat16, torch.float32])
def test_static_scratch_matches_workspace_entry_point_twice(qdtype):
    heads, group, dim, tokens = 8, 4, 128, 32768
    data = synthetic.make_layer(21, 0, heads, tokens, dim, 32, device=DEV)
    cfg = RefineKVConfig(eps=0.01)
    summary = build_summary(data.keys, data.values, cfg)
    ks = data.keys[:, :19].contiguous()
    vs = data.values[:, :19].contiguous()
    for step in range(2):  # the second call reuses the static array after the first
        q = synthetic.make_queries(21, 0, step, data.planted_mean, group, 1, qdtype)[0]
        want = sparse_attention(q, summary, ks, vs, cfg, return_selected=True)
        out = torch.full((heads, group, 1, dim), float("nan"), device=DEV, dtype=qdtype)
        selected = torch.full((heads, summary.num_blocks), 7, device=DEV, dtype=torch.uint8)
        _decode_static(q, summary, ks, vs, cfg, out, selected)
        torch.cuda.synchronize()
        assert _static_status() == 0  # no bounded wait ran out, no device input out of range
        assert torch.equal(selected.bool(), want.selected)
        tol = dict(atol=1e-4, rtol=0) if qdtype == torch.float32 else dict(atol=4e-3, rtol=2e-2)
        torch.testing.assert_close(out, want.output, **tol)


def test_static_scratch_rejects_geometry_larger_than_the_array():
    lib = _native.load()
    heads, group, blocks, dim, block = 64, 4, 1 << 16, 128, 32
    need = lib.rkv_decode_workspace_size(heads, group, blocks, dim, block)
    capacity = 32 << 20  # RKV_DECODE_STATIC_SCRATCH_BYTES
    assert need > capacity  # so the call below is rejected before anything is launched
    t = torch.zeros(16, device=DEV, dtype=torch.bfloat16)
    s = _native.Summary(key_pages=t.data_ptr(), value_pages=t.data_ptr(), key_page_head_stride=0,
                        value_page_head_stride=0, counts=t.data_ptr(), key_mean=t.data_ptr(),
                        value_mean=t.data_ptr(), ellipsoid=t.data_ptr(),
                        value_norm=t.data_ptr(), max_value_norm=t.data_ptr(), heads=heads,
                        blocks=blocks, block_size=block, head_dim=dim,
                        prompt_length=blocks * block)
    rc = lib.rkv_decode_static(ctypes.byref(s), t.data_ptr(), _native.DTYPE_BF16, group, None,
                               None, 0, 0, 0, 0, 0, None, 0, None, 0.01, 2, t.data_ptr(),
                               t.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == _native.RKV_ERR_WORKSPACE
    assert b"static array" in lib.rkv_last_error()
    rc = lib.rkv_decode_static(None, t.data_ptr(), _native.DTYPE_BF16, group, None, None, 0, 0, 0,
                               0, 0, None, 0, None, 0.01, 2, t.data_ptr(), t.data_ptr(),
                               torch.cuda.current_stream().cuda_stream)
    assert rc == _native.RKV_ERR_INVALID_ARGUMENT
    assert lib.rkv_last_error() == b"summary is null"

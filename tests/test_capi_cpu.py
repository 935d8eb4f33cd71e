"""The C-ABI library loads, exports every declared symbol and validates arguments (no GPU)."""

import ctypes
import pathlib
import re

import pytest
import torch

from refinekv_b200 import RefineKVConfig, _native

REPO = pathlib.Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def lib():
    from conftest import native_build_module

    native_build_module().build()
    return _native.load()


def _declared_symbols():
    names = set()
    for header in (REPO / "include").glob("*.h"):
        text = header.read_text()
        names.update(re.findall(r"RKV_API\s+[\w\s\*]+?\b(rkv_\w+)\s*\(", text))
    return names


def test_header_declares_the_binding_surface():
    assert _declared_symbols() == set(_native.EXPORTS)


def test_library_exports_every_declared_symbol(lib):
    for name in _declared_symbols():
        assert hasattr(lib, name), name
    assert lib.rkv_abi_version() == _native.ABI_VERSION


def test_library_exports_nothing_else(lib):
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", str(_native.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    public = {name for name in exported if not name.startswith("_")}
    assert public == set(_native.EXPORTS)


def test_status_strings(lib):
    assert lib.rkv_status_string(0) == b"ok"
    assert lib.rkv_status_string(_native.RKV_ERR_ALIGNMENT) == b"misaligned pointer or stride"
    assert lib.rkv_decode_launch_count(_native.PHASE_ALL) == 4
    assert lib.rkv_decode_launch_count(_native.PHASE_ATTEND) == 1


def test_summarize_rejects_bad_arguments_before_touching_a_device(lib):
    args = [ctypes.c_void_p(16), ctypes.c_void_p(16), 2, 64, 80, 0, 80, 0, 80, 32,
            None, None, ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16),
            ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), None]
    assert lib.rkv_summarize(*args) == _native.RKV_ERR_UNSUPPORTED  # head_dim 80
    assert b"head_dim" in lib.rkv_last_error()
    args[4] = 288
    assert lib.rkv_summarize(*args) == _native.RKV_ERR_UNSUPPORTED  # above 256
    args[4], args[9] = 128, 24
    assert lib.rkv_summarize(*args) == _native.RKV_ERR_UNSUPPORTED  # block 24
    args[9] = 32
    args[0] = ctypes.c_void_p(18)
    assert lib.rkv_summarize(*args) == _native.RKV_ERR_ALIGNMENT
    args[0] = None
    assert lib.rkv_summarize(*args) == _native.RKV_ERR_INVALID_ARGUMENT


def test_fp32_summarize_requires_bf16_page_copies_before_touching_a_device(lib):
    args = [ctypes.c_void_p(16), ctypes.c_void_p(16), 2, 64, 128, 64 * 128, 128, 64 * 128, 128,
            32, None, None, ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16),
            ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), None]
    assert lib.rkv_summarize_f32(*args) == _native.RKV_ERR_INVALID_ARGUMENT
    assert b"page copies" in lib.rkv_last_error()
    args[10], args[11] = ctypes.c_void_p(16), ctypes.c_void_p(16)
    args[7] = 64 * 128 + 2  # fp32 head stride of 8 bytes past a 16-byte multiple
    assert lib.rkv_summarize_f32(*args) == _native.RKV_ERR_ALIGNMENT


def test_static_status_rejects_a_null_destination(lib):
    assert lib.rkv_decode_static_status(None, None) == _native.RKV_ERR_INVALID_ARGUMENT
    assert lib.rkv_last_error() == b"out is null"


def test_decode_rejects_bad_arguments_before_touching_a_device(lib):
    s = _native.Summary(key_pages=16, value_pages=16, counts=16, key_mean=16, value_mean=16,
                        ellipsoid=16, value_norm=16, max_value_norm=16, heads=2, blocks=3,
                        block_size=32, head_dim=128, prompt_length=71)

    def call(summary, group=4, eps=0.01, reduction=2):
        return lib.rkv_decode(ctypes.byref(summary), 16, 0, group, None, None, 0, 0, 0, 0, 0,
                              None, 0, None, eps, reduction, 16, 16, None, 0, 15, None)

    assert call(s, group=17) == _native.RKV_ERR_UNSUPPORTED
    assert call(s, eps=-1.0) == _native.RKV_ERR_INVALID_ARGUMENT
    assert call(s, eps=float("nan")) == _native.RKV_ERR_INVALID_ARGUMENT
    assert call(s, reduction=5) == _native.RKV_ERR_INVALID_ARGUMENT
    bad = _native.Summary.from_buffer_copy(s)
    bad.blocks = 4  # ceil(71 / 32) == 3
    assert call(bad) == _native.RKV_ERR_INVALID_ARGUMENT
    bad = _native.Summary.from_buffer_copy(s)
    bad.block_size = 8
    assert call(bad) == _native.RKV_ERR_UNSUPPORTED


def test_batch_geometry_is_checked_before_touching_a_device(lib):
    def summary(**kw):
        base = dict(key_pages=16, value_pages=16, counts=16, key_mean=16, value_mean=16,
                    ellipsoid=16, value_norm=16, max_value_norm=16, heads=4, blocks=3,
                    block_size=32, head_dim=128, prompt_length=71, sequences=2,
                    prompt_lengths=16)
        base.update(kw)
        return _native.Summary(**base)

    def decode(s):
        return lib.rkv_decode(ctypes.byref(s), 16, 0, 4, None, None, 0, 0, 0, 0, 0,
                              None, 0, None, 0.01, 2, 16, 16, None, 0, 15, None)

    assert decode(summary(sequences=3)) == _native.RKV_ERR_INVALID_ARGUMENT  # 3 does not divide 4
    assert decode(summary(prompt_lengths=None)) == _native.RKV_ERR_INVALID_ARGUMENT
    assert decode(summary(sequences=-1)) == _native.RKV_ERR_INVALID_ARGUMENT
    assert b"sequences" in lib.rkv_last_error()
    # a sequence split takes one prompt
    rc = lib.rkv_select_split(ctypes.byref(summary()), 16, 0, 1, 4, 0.01, 2, 16, 0, 16, 1 << 20,
                              2, 0, 3, 16, 1 << 20, 1, None)
    assert rc == _native.RKV_ERR_UNSUPPORTED and b"batch" in lib.rkv_last_error()
    rc = lib.rkv_decode_split(ctypes.byref(summary()), 16, 0, 4, None, None, 0, 0, 0, 0, 0, None,
                              0, None, 0.01, 2, 16, 16, 16, 1 << 20, 2, 0, 3, 16, 1 << 20, 1,
                              None)
    assert rc == _native.RKV_ERR_UNSUPPORTED and b"batch" in lib.rkv_last_error()


def test_page_table_geometry_is_checked_before_touching_a_device(lib):
    def summary(**kw):
        base = dict(key_pages=16, value_pages=16, counts=16, key_mean=16, value_mean=16,
                    ellipsoid=16, value_norm=16, max_value_norm=16, heads=2, blocks=3,
                    block_size=32, head_dim=128, prompt_length=71, page_table=16,
                    page_table_stride=3, pool_pages=8, key_page_stride=8192,
                    value_page_stride=8192, key_token_stride=128, value_token_stride=128)
        base.update(kw)
        return _native.Summary(**base)

    def decode(s):
        return lib.rkv_decode(ctypes.byref(s), 16, 0, 4, None, None, 0, 0, 0, 0, 0,
                              None, 0, None, 0.01, 2, 16, 16, None, 0, 15, None)

    for bad in ({"pool_pages": 0}, {"page_table_stride": 2}, {"key_token_stride": 0},
                {"value_page_stride": -8192}):
        assert decode(summary(**bad)) == _native.RKV_ERR_INVALID_ARGUMENT, bad
        assert b"page table" in lib.rkv_last_error()
    rc = lib.rkv_decode_split(ctypes.byref(summary()), 16, 0, 4, None, None, 0, 0, 0, 0, 0, None,
                              0, None, 0.01, 2, 16, 16, 16, 1 << 20, 2, 0, 3, 16, 1 << 20, 1,
                              None)
    assert rc == _native.RKV_ERR_UNSUPPORTED and b"page pool" in lib.rkv_last_error()


def test_workspace_size_needs_a_device(lib):
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    assert lib.rkv_decode_workspace_size(8, 4, 4096, 128, 32) == 0


@pytest.mark.parametrize(
    "kwargs", [{"eps": float("nan")}, {"eps": -1}, {"block_size": 10}, {"anchor_tokens": -1},
               {"gqa_reduction": "sum"}, {"backend": "jax"}, {"summary_chunk_blocks": 0}])
def test_invalid_config_is_rejected(kwargs):
    with pytest.raises(ValueError):
        RefineKVConfig(**kwargs)


def test_config_defaults_match_reference():
    c = RefineKVConfig()
    assert (c.block_size, c.eps, c.gqa_reduction, c.anchor_tokens, c.full_attention_layers,
            c.backend, c.summary_chunk_blocks, c.collect_stats) == (
        32, 0.01, "any", 0, 0, "auto", 512, False)


def test_cpu_tensors_fail_loudly():
    from refinekv_b200 import build_summary, select_blocks

    keys = torch.zeros(2, 64, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        build_summary(keys, keys)
    with pytest.raises(ValueError, match="same nonempty"):
        build_summary(keys, keys[:, :3])
    with pytest.raises(TypeError, match="floating point"):
        build_summary(keys.to(torch.int32), keys.to(torch.int32))

    class _Summary:  # enough of a summary for argument validation
        keys = torch.zeros(2, 2, 32, 128)
        block_size = 32
        num_blocks = 2
        num_heads = 2

    q = torch.zeros(2, 4, 1, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        select_blocks(q, _Summary())
    with pytest.raises(ValueError, match="torch"):
        select_blocks(q, _Summary(), RefineKVConfig(backend="torch"))
    with pytest.raises(ValueError, match="query must have shape"):
        select_blocks(q[:, :, 0], _Summary())


def test_reference_backend_stub_matches_the_abi():
    """The ctypes module a maintainer copies into the reference declares rkv_summary as the
    library does and builds the view with every field."""
    import importlib.util
    import inspect
    import os

    os.environ["RKV_LIBRARY"] = str(_native.LIB_PATH)
    path = REPO / "refinekv-release_b200" / "integration" / "reference_backend_stub.py"
    spec = importlib.util.spec_from_file_location("reference_backend_stub", path)
    stub = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(stub)
    assert [n for n, _ in stub._Summary._fields_] == [n for n, _ in _native.Summary._fields_]
    assert [t for _, t in stub._Summary._fields_] == [t for _, t in _native.Summary._fields_]
    fake = type("S", (), {})()
    t = torch.zeros(2, 3, 4, 128)
    fake.keys = fake.values = fake.key_mean = fake.value_mean = fake.ellipsoid = t
    fake.counts = torch.zeros(3, dtype=torch.int64)
    fake.value_norm, fake.max_value_norm = torch.zeros(2, 3), torch.zeros(2)
    fake.block_size, fake.prompt_length = 4, 12
    view = stub._view(fake)
    assert (view.heads, view.blocks, view.block_size, view.head_dim, view.prompt_length,
            view.sequences) == (2, 3, 4, 128, 12, 1)
    ref_args = inspect.signature(stub.sparse_attention_b200).parameters
    assert list(ref_args) == ["query", "summary", "key_suffix", "value_suffix", "config",
                              "anchor_mask", "workspace", "return_selected", "suffix_length"]


def test_page_view_and_dense_attention_validate_before_touching_a_device():
    from refinekv_b200 import dense_attention, page_view

    cache = torch.zeros(2, 100, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="whole pages"):
        page_view(cache, cache, 90, 64)  # 2 pages of 64 rows need 128
    with pytest.raises(ValueError, match="bf16"):
        page_view(cache.float(), cache.float(), 10)
    pages = page_view(cache, cache, 90, 32)
    assert pages.keys.shape == (2, 3, 32, 128) and pages.keys.data_ptr() == cache.data_ptr()
    q = torch.zeros(2, 4, 1, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        dense_attention(q, pages, cache[:, 90:], cache[:, 90:])
    with pytest.raises(ValueError, match="query heads"):
        dense_attention(q[:1], pages, cache[:, 90:], cache[:, 90:])

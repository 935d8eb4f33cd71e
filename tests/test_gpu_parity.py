"""CUDA path vs. the CPU oracle and the reference's golden outputs (needs a B200).

Tolerances (stated by the north star and the reference tests):
* summaries: counts, page copies and bf16 means exact (the K/V sums follow
  the reference's FP32 order); the ellipsoid within 1-2 bf16 ulp (its
  channel sum is vectorised in another order by torch's CPU kernels);
* masks: identical except blocks whose decisive risk lies within 1e-3
  (relative) of eps, which are counted and reported separately;
* outputs: atol 4e-3 + rtol 2e-2 (reference test_attention.py:183) and a
  max-abs error <= 2e-2 for bf16 queries; 1e-4 for FP32 queries.
"""

import pytest
import torch
import torch.nn.functional as F

from helpers import bf16_ulp_diff, checksum, reference_inputs, sha256
from oracle import refinekv_oracle as ora
from refinekv_b200 import (RefineKVConfig, build_summary, build_summary_into, select_blocks,
                           sparse_attention, synthetic)
from refinekv_b200.attention import device_status, select_blocks_union

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _gpu(t):
    return t.to(DEV) if t is not None else None


def assert_summary_close(gpu, want, *, max_ulp=2):
    """Means bit-exact (the summarizer adds in the reference's FP32 order); the
    ellipsoid within `max_ulp` bf16 ulp on under 2 % of elements."""
    assert torch.equal(gpu.counts.cpu(), want["counts"] if isinstance(want, dict) else want.counts)
    get = (lambda n: want[n]) if isinstance(want, dict) else (lambda n: getattr(want, n))
    for name in ("key_mean", "value_mean"):
        assert torch.equal(getattr(gpu, name).cpu(), get(name)), name
    ulp = bf16_ulp_diff(gpu.ellipsoid.cpu(), get("ellipsoid"))
    assert int(ulp.max()) <= max_ulp, ("ellipsoid", int(ulp.max()))
    assert float((ulp > 0).float().mean()) < 0.02, "ellipsoid"
    torch.testing.assert_close(gpu.value_norm.cpu(), get("value_norm"), rtol=2e-6, atol=1e-6)
    torch.testing.assert_close(gpu.max_value_norm.cpu(), get("max_value_norm"), rtol=2e-6,
                               atol=1e-6)


def check_mask(gpu_mask, q, summary_cpu, cfg, anchor=None):
    """GPU mask equals the oracle's outside the eps margin; returns (oracle mask, z, #margin)."""
    want, z = ora.select_blocks(q.cpu(), summary_cpu, cfg.eps, cfg.gqa_reduction)
    margin = ora.margin_blocks(q.cpu(), summary_cpu, cfg.eps, cfg.gqa_reduction)
    if anchor is not None:
        want = want | anchor.cpu()
        margin = margin & ~anchor.cpu()
    diff = (gpu_mask.cpu() != want) & ~margin
    assert not diff.any(), f"{int(diff.sum())} blocks differ outside the eps margin"
    return want, z, int(margin.sum())


def check_output(out, q, summary_cpu, ks, vs, selected, z, *, fp32=False):
    want = ora.mixed_attention(q.cpu(), summary_cpu, ks.cpu(), vs.cpu(), selected.cpu(), z)
    got = out.float().cpu()
    if fp32:
        torch.testing.assert_close(got, want, atol=1e-4, rtol=0)
    else:
        torch.testing.assert_close(got, want.to(torch.bfloat16).float(), atol=4e-3, rtol=2e-2)
        assert float((got - want).abs().max()) <= 2e-2


# --------------------------------------------------------------------------
# summarizer
# --------------------------------------------------------------------------

def test_summaries_match_reference_golden(golden):
    """bf16 and fp32 caches; an fp32 cache's pages come back rounded to bf16."""
    dtypes = set()
    for case in golden["summary_cases"]:
        cfg = RefineKVConfig(block_size=case["block"])
        s = build_summary(_gpu(case["keys"]), _gpu(case["values"]), cfg)
        assert_summary_close(s, case["out"])
        assert s.keys.dtype == torch.bfloat16
        assert torch.equal(s.keys.cpu(), case["key_pages"].to(torch.bfloat16))
        assert torch.equal(s.values.cpu(), case["value_pages"].to(torch.bfloat16))
        dtypes.add(case["dtype"])
    assert dtypes == {"torch.bfloat16", "torch.float32"}


def test_summary_aliases_aligned_cache_and_keeps_inputs():
    gen = torch.Generator(device=DEV).manual_seed(17)
    cache_k = torch.randn(2, 96, 128, device=DEV, generator=gen).to(torch.bfloat16)
    cache_v = torch.randn(2, 96, 128, device=DEV, generator=gen).to(torch.bfloat16)
    ck, cv = cache_k.clone(), cache_v.clone()
    s = build_summary(cache_k[:, :64], cache_v[:, :64], RefineKVConfig())
    assert s.keys.data_ptr() == cache_k.data_ptr()  # page view aliases the cache
    assert s.keys.stride() == (96 * 128, 32 * 128, 128, 1)
    s2 = build_summary(cache_k[:, :67], cache_v[:, :67], RefineKVConfig())
    assert s2.keys.data_ptr() != cache_k.data_ptr()  # partial page -> padded copy
    assert torch.equal(s2.keys.reshape(2, -1, 128)[:, :67], cache_k[:, :67])
    assert not s2.keys.reshape(2, -1, 128)[:, 67:].any()
    assert torch.equal(cache_k, ck) and torch.equal(cache_v, cv)
    assert_summary_close(s2, ora.build_summary(cache_k[:, :67].cpu(), cache_v[:, :67].cpu(), 32))


@pytest.mark.parametrize("tokens", [64, 67, 1000])
def test_summary_into_cache_equals_build_summary(tokens):
    """The prefill's cache write fused with the summary: the same summaries, the prompt in the cache."""
    gen = torch.Generator(device=DEV).manual_seed(23)
    big_k = torch.randn(2, tokens + 5, 128, device=DEV, generator=gen).to(torch.bfloat16)
    big_v = torch.randn(2, tokens + 5, 128, device=DEV, generator=gen).to(torch.bfloat16)
    keys, values = big_k[:, 2:2 + tokens], big_v[:, 2:2 + tokens]  # strided prompt
    padded = -(-tokens // 32) * 32
    cache_k = torch.randn(2, padded + 40, 128, device=DEV, generator=gen).to(torch.bfloat16)
    cache_v = torch.randn(2, padded + 40, 128, device=DEV, generator=gen).to(torch.bfloat16)
    before_k, before_v = cache_k.clone(), cache_v.clone()
    fused = build_summary_into(keys, values, cache_k, cache_v)
    plain = build_summary(keys, values)
    for name in ("counts", "key_mean", "value_mean", "ellipsoid", "value_norm", "max_value_norm"):
        assert torch.equal(getattr(fused, name), getattr(plain, name)), name
    for cache, src, before in ((cache_k, keys, before_k), (cache_v, values, before_v)):
        assert torch.equal(cache[:, :tokens], src)
        assert not cache[:, tokens:padded].any()
        assert torch.equal(cache[:, padded:], before[:, padded:])
    assert fused.keys.data_ptr() == cache_k.data_ptr()
    assert torch.equal(fused.keys, plain.keys.contiguous())
    q = torch.randn(2, 4, 1, 128, device=DEV, generator=gen).to(torch.bfloat16)
    suffix = torch.randn(2, 3, 128, device=DEV, generator=gen).to(torch.bfloat16)
    a = sparse_attention(q, fused, suffix, suffix, return_selected=True)
    b = sparse_attention(q, plain, suffix, suffix, return_selected=True)
    assert torch.equal(a.selected, b.selected)


@pytest.mark.parametrize("tokens", [1020, 67])
def test_fused_summary_decodes_after_generated_tokens_fill_the_last_page(tokens):
    """A decoder appends its tokens to the cache the fused summary aliases: the rows
    after the prompt in its last page stop being zero, and decode must not notice."""
    gen = torch.Generator(device=DEV).manual_seed(29)
    heads, dim, steps = 4, 128, 12
    keys = torch.randn(heads, tokens, dim, device=DEV, generator=gen).to(torch.bfloat16)
    values = torch.randn(heads, tokens, dim, device=DEV, generator=gen).to(torch.bfloat16)
    new_k = torch.randn(heads, steps, dim, device=DEV, generator=gen).to(torch.bfloat16)
    new_v = torch.randn(heads, steps, dim, device=DEV, generator=gen).to(torch.bfloat16)
    assert tokens % 32  # the prompt ends inside a page; 1020 + 12 also crosses into the next
    cache_k = torch.zeros(heads, tokens + steps + 64, dim, device=DEV, dtype=torch.bfloat16)
    cache_v = torch.zeros_like(cache_k)
    cfg = RefineKVConfig(eps=0.02)
    fused = build_summary_into(keys, values, cache_k, cache_v, cfg)
    plain = build_summary(keys, values, cfg)
    ws_fused, ws_plain = {}, {}
    for step in range(steps):
        cache_k[:, tokens + step] = new_k[:, step]  # the decoder's cache write
        cache_v[:, tokens + step] = new_v[:, step]
        q = torch.randn(heads, 4, 1, dim, device=DEV, generator=gen).to(torch.bfloat16)
        ks, vs = cache_k[:, tokens:tokens + step + 1], cache_v[:, tokens:tokens + step + 1]
        a = sparse_attention(q, fused, ks, vs, cfg, workspace=ws_fused, return_selected=True)
        b = sparse_attention(q, plain, new_k[:, :step + 1], new_v[:, :step + 1], cfg,
                             workspace=ws_plain, return_selected=True)
        assert torch.equal(a.selected, b.selected), step
        assert torch.equal(a.output, b.output), step
    assert device_status(ws_fused) == 0 and device_status(ws_plain) == 0
    assert torch.equal(a.output.view(torch.int16), b.output.view(torch.int16))


def test_summary_takes_bf16_and_fp32_caches_only():
    k = torch.zeros(2, 64, 128, device=DEV, dtype=torch.float16)
    with pytest.raises(TypeError, match="BF16 or FP32"):
        build_summary(k, k)
    s = build_summary(k.float(), k.float())
    assert s.keys.dtype == torch.bfloat16 and not s.keys.any()


def test_ellipsoid_bounds_sampled_queries():
    """|q.(k - kbar)| <= sqrt(q^2 . W2) for every real row (reference test_attention.py:59-71)."""
    q, keys, values = reference_inputs(65, 128, device=DEV)
    keys[..., :3] = torch.tensor([96, 48, -80], dtype=torch.bfloat16, device=DEV)
    s = build_summary(keys, values, RefineKVConfig())
    assert torch.isfinite(s.ellipsoid).all()
    centered = s.keys.float() - s.key_mean.float().unsqueeze(2)
    exact = torch.einsum("hgd,hbtd->hgbt", q[:, :, 0].float(), centered).abs()
    valid = torch.arange(s.block_size, device=DEV)[None] < s.counts[:, None]
    exact = exact.masked_fill(~valid[None, None], 0).amax(-1)
    bound = torch.einsum("hgd,hbd->hgb", q[:, :, 0].float().square(), s.ellipsoid.float()).sqrt()
    assert (exact <= bound + 1e-5).all()


# --------------------------------------------------------------------------
# selector + attention on the reference's agreement shapes
# --------------------------------------------------------------------------

def _agreement_inputs(case):
    if case["keys"] is not None:
        return case["q"], case["keys"], case["values"]
    q, k, v = reference_inputs(case["length"], case["dim"], case["seed"])
    assert [checksum(q), checksum(k), checksum(v)] == case["input_checksum"]
    return q, k, v


@pytest.mark.parametrize("index", range(4))
def test_agreement_cases(golden, index):
    case = golden["agreement_cases"][index]
    q, keys, values = (_gpu(t) for t in _agreement_inputs(case))
    cfg = RefineKVConfig(block_size=case["block"], eps=case["eps"],
                         gqa_reduction=case["reduction"])
    s = build_summary(keys, values, cfg)
    if isinstance(case["summary"]["key_mean"], torch.Tensor):
        assert_summary_close(s, case["summary"])
    s_cpu = ora.as_cpu_summary(s)
    workspace = {}
    sel = select_blocks(q, s, cfg, workspace=workspace)
    check_mask(sel, q, s_cpu, cfg)
    # and against the reference's own mask on its own summary, outside the margin
    ref_margin = ora.margin_blocks(q.cpu(), ora.build_summary(keys.cpu(), values.cpu(),
                                                              case["block"]), cfg.eps,
                                   cfg.gqa_reduction)
    assert not ((sel.cpu() != case["mask"]) & ~ref_margin).any()
    anchor = _gpu(case["anchor"])
    for n, rec in case["attention"].items():
        res = sparse_attention(q, s, keys[:, :n], values[:, :n], cfg, anchor_mask=anchor,
                               workspace=workspace, return_selected=True)
        want_mask, z, _ = check_mask(res.selected, q, s_cpu, cfg, anchor)
        check_output(res.output, q, s_cpu, keys[:, :n], values[:, :n], res.selected, z)
        if torch.equal(res.selected.cpu(), rec["selected"]):
            torch.testing.assert_close(res.output.float().cpu(), rec["output"].float(),
                                       atol=4e-3, rtol=2e-2)
    assert device_status(workspace) == 0


def test_device_suffix_length_masks_fixed_capacity():
    """Reference test_attention.py:186-204: device length == sliced suffix, bitwise."""
    q, keys, values = reference_inputs(71, 128, device=DEV)
    cfg = RefineKVConfig(gqa_reduction="mean")
    s = build_summary(keys, values, cfg)
    suffix_k, suffix_v = reference_inputs(16, 128, device=DEV)[1:]
    visible = torch.zeros((), device=DEV, dtype=torch.int32)
    for count in (0, 1, 5, 16):
        visible.fill_(count)
        got = sparse_attention(q, s, suffix_k, suffix_v, cfg, suffix_length=visible).output.clone()
        want = sparse_attention(q, s, suffix_k[:, :count], suffix_v[:, :count], cfg).output.clone()
        assert torch.equal(got, want), count


def test_representative_multiplicity_known_answer(golden):
    case = golden["special_cases"]["known_answer"]
    cfg = RefineKVConfig(eps=1e6, block_size=16)
    keys, values = _gpu(case["keys"]), _gpu(case["values"])
    s = build_summary(keys, values, cfg)
    q = torch.zeros(1, 2, 1, 64, device=DEV)
    res = sparse_attention(q, s, keys[:, :0], values[:, :0], cfg, return_selected=True)
    assert not res.selected.any()
    torch.testing.assert_close(res.output.cpu(), torch.full((1, 2, 1, 64), (16 + 9) / 19))


def test_anchor_union_expands_only_requested_pages():
    q, keys, values = reference_inputs(71, 64, device=DEV)
    cfg = RefineKVConfig(eps=1e6)
    s = build_summary(keys, values, cfg)
    anchor = torch.zeros(2, s.num_blocks, dtype=torch.bool, device=DEV)
    anchor[:, -1] = True
    res = sparse_attention(q, s, keys[:, :0], values[:, :0], cfg, anchor_mask=anchor,
                           return_selected=True)
    assert torch.equal(res.selected, anchor)
    assert torch.isfinite(res.output).all()
    s_cpu = ora.as_cpu_summary(s)
    _, z = ora.select_blocks(q.cpu(), s_cpu, cfg.eps, cfg.gqa_reduction)
    check_output(res.output, q, s_cpu, keys[:, :0], values[:, :0], res.selected, z)


def test_large_finite_delta_stays_finite(golden):
    case = golden["special_cases"]["large_query"]
    q, keys, values = _gpu(case["q"]), _gpu(case["keys"]), _gpu(case["values"])
    cfg = RefineKVConfig()
    s = build_summary(keys, values, cfg)
    sel = select_blocks(q, s, cfg)
    check_mask(sel, q, ora.as_cpu_summary(s), cfg)
    res = sparse_attention(q, s, keys[:, :0], values[:, :0], cfg)
    assert torch.isfinite(res.output).all()


@pytest.mark.parametrize("suffix_length", [0, 5])
def test_full_expansion_matches_dense_attention(suffix_length):
    """eps = 0 selects every block and equals dense SDPA (reference test_attention.py:74-90)."""
    q, keys, values = reference_inputs(71, 64, device=DEV)
    cfg = RefineKVConfig(eps=0)
    s = build_summary(keys, values, cfg)
    res = sparse_attention(q, s, keys[:, :suffix_length], values[:, :suffix_length], cfg,
                           return_selected=True)
    assert res.selected.all()
    ek = torch.cat([keys, keys[:, :suffix_length]], 1).repeat_interleave(4, 0)
    ev = torch.cat([values, values[:, :suffix_length]], 1).repeat_interleave(4, 0)
    want = F.scaled_dot_product_attention(q.reshape(8, 1, 64).float(), ek.float(), ev.float())
    torch.testing.assert_close(res.output.float().reshape(8, 1, 64), want, atol=0.004, rtol=0.02)


def test_batched_anchor_union_equals_or_of_single_queries():
    data = synthetic.make_layer(3, 0, 8, 4096, 128, 32, device=DEV)
    s = build_summary(data.keys, data.values, RefineKVConfig())
    cfg = RefineKVConfig(eps=0.05)
    anchors = synthetic.make_queries(3, 0, -1, data.planted_mean, 4, 8)
    union = select_blocks_union(anchors, s, cfg)
    single = None
    for a in anchors:
        m = select_blocks(a, s, cfg)
        single = m if single is None else single | m
    assert torch.equal(union, single)
    check = ora.anchor_union(anchors.cpu(), ora.as_cpu_summary(s), cfg.eps, cfg.gqa_reduction)
    margin = torch.zeros_like(check)
    for a in anchors:
        margin |= ora.margin_blocks(a.cpu(), ora.as_cpu_summary(s), cfg.eps, cfg.gqa_reduction)
    assert not ((union.cpu() != check) & ~margin).any()


@pytest.mark.parametrize("index", range(2))
def test_synthetic_workload_vs_reference(golden, index):
    """Scaled-down config-0 workload: anchors, three decode steps, fp32 and bf16 caches.

    The cache stays in its own dtype on the GPU (an fp32 cache is summarised
    from its fp32 values), and the summary is judged against the reference's
    own summary of that cache (the golden record); masks and outputs against
    the oracle deciding from the reference's summary, outputs also against
    the reference's own outputs where the masks agree.
    """
    case = golden["synthetic_cases"][index]
    fp32 = case["dtype"] == "torch.float32"
    dtype = torch.float32 if fp32 else torch.bfloat16
    data = synthetic.make_layer(case["seed"], case["layer"], case["heads"], case["tokens"],
                                case["dim"], case["block"], dtype=dtype)
    assert [checksum(data.keys), checksum(data.values)] == case["input_checksum"]
    cfg = RefineKVConfig(block_size=case["block"], eps=case["eps"],
                         gqa_reduction=case["reduction"])
    s = build_summary(data.keys.to(DEV), data.values.to(DEV), cfg)
    # The oracle's summary of the same cache reproduces the reference's (its digests are
    # the golden record, checked in test_oracle_golden).
    ref = ora.build_summary(data.keys, data.values, case["block"])
    assert sha256(ref.key_mean) == case["summary"]["key_mean"]["sha256"]
    assert_summary_close(s, ref)
    qdtype = torch.float32 if fp32 else torch.bfloat16
    anchor_q = synthetic.make_queries(case["seed"], case["layer"], -1, data.planted_mean,
                                      case["group"], case["anchors"], qdtype)
    anchor = select_blocks_union(anchor_q.to(DEV), s, cfg)
    margin = torch.zeros_like(case["anchor_mask"])
    for a in anchor_q:
        margin |= ora.margin_blocks(a, ref, cfg.eps, cfg.gqa_reduction)
    assert not ((anchor.cpu() != case["anchor_mask"]) & ~margin).any()
    workspace = {}
    ks, vs = [], []
    for step, rec in enumerate(case["per_step"]):
        k, v = synthetic.make_decode_token(case["seed"], case["layer"], step, case["heads"],
                                           case["dim"], case["tokens"] + step, dtype=dtype)
        ks.append(k)
        vs.append(v)
        q = rec["q"].to(DEV)
        kk, vv = torch.cat(ks, 1).to(DEV), torch.cat(vs, 1).to(DEV)
        res = sparse_attention(q, s, kk, vv, cfg, anchor_mask=anchor, workspace=workspace,
                               return_selected=True)
        _, z, _ = check_mask(res.selected, q, ref, cfg, anchor)
        check_output(res.output, q, ref, kk, vv, res.selected, z, fp32=fp32)
        if torch.equal(res.selected.cpu(), rec["selected"]):
            got, want = res.output.float().cpu(), rec["output"].float()
            if fp32:
                torch.testing.assert_close(got, want, atol=1e-4, rtol=0)
            else:
                assert float((got - want).abs().max()) <= 2e-2
    assert device_status(workspace) == 0


# --------------------------------------------------------------------------
# shapes and edge cases
# --------------------------------------------------------------------------

SHAPES = [
    # heads, group, dim, block, tokens, suffix, reduction, eps
    (8, 4, 128, 32, 4096, 3, "any", 0.01),
    (4, 7, 128, 64, 5000, 9, "max", 0.005),
    (2, 1, 64, 16, 100, 0, "mean", 0.02),
    (2, 16, 256, 32, 1000, 40, "any", 0.02),
    (3, 8, 192, 64, 777, 65, "mean", 0.01),
    (1, 2, 128, 32, 17, 1, "any", 0.0),
    (2, 12, 64, 16, 300, 17, "max", 0.1),
    # head dims that are not multiples of 64 (TMA zero-fills the padding columns)
    (2, 4, 32, 32, 1000, 5, "any", 0.01),
    (4, 7, 96, 64, 2000, 9, "max", 0.005),
    (2, 8, 160, 16, 700, 3, "mean", 0.02),
    (1, 16, 224, 32, 900, 33, "any", 0.02),
]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("qdtype", [torch.bfloat16, torch.float32])
def test_shapes_match_oracle(shape, qdtype):
    heads, group, dim, block, tokens, suffix, reduction, eps = shape
    data = synthetic.make_layer(11, heads * 7 + group, heads, tokens, dim, block, device=DEV)
    cfg = RefineKVConfig(block_size=block, eps=eps, gqa_reduction=reduction)
    s = build_summary(data.keys, data.values, cfg)
    s_cpu = ora.as_cpu_summary(s)
    assert_summary_close(s, ora.build_summary(data.keys.cpu(), data.values.cpu(), block))
    q = synthetic.make_queries(11, 0, 0, data.planted_mean, group, 1, qdtype)[0]
    gen = torch.Generator(device=DEV).manual_seed(5)
    ks = torch.randn(heads, suffix, dim, device=DEV, generator=gen).to(torch.bfloat16)
    vs = torch.randn(heads, suffix, dim, device=DEV, generator=gen).to(torch.bfloat16)
    workspace = {}
    for _ in range(2):  # a reused workspace must give the same answer
        res = sparse_attention(q, s, ks, vs, cfg, workspace=workspace, return_selected=True)
        _, z, _ = check_mask(res.selected, q, s_cpu, cfg)
        check_output(res.output, q, s_cpu, ks, vs, res.selected, z,
                     fp32=qdtype == torch.float32)
    assert res.output.dtype == qdtype
    assert device_status(workspace) == 0


def test_repeated_calls_are_bitwise_deterministic():
    data = synthetic.make_layer(5, 1, 8, 20000, 128, 32, device=DEV)
    cfg = RefineKVConfig(eps=0.02)
    s = build_summary(data.keys, data.values, cfg)
    q = synthetic.make_queries(5, 1, 0, data.planted_mean, 4)[0]
    ks = data.keys[:, :50].contiguous()
    outs = [sparse_attention(q, s, ks, ks, cfg).output.clone() for _ in range(3)]
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])


def test_strided_suffix_from_cache_view():
    """The suffix may be a strided slice of a larger cache (as the adapter passes it)."""
    data = synthetic.make_layer(6, 0, 4, 1000, 128, 32, device=DEV)
    cache = torch.randn(1, 4, 1100, 128, device=DEV).to(torch.bfloat16)
    cache[0, :, :1000] = data.keys
    cfg = RefineKVConfig(eps=0.01)
    s = build_summary(cache[0, :, :1000], cache[0, :, :1000], cfg)
    q = synthetic.make_queries(6, 0, 0, data.planted_mean, 4)[0]
    sk = cache[0, :, 1000:1037]
    res = sparse_attention(q, s, sk, sk, cfg, return_selected=True)
    s_cpu = ora.as_cpu_summary(s)
    _, z, _ = check_mask(res.selected, q, s_cpu, cfg)
    check_output(res.output, q, s_cpu, sk, sk, res.selected, z)


def test_128k_context_properties():
    """Full-size geometry: eps=0 equals dense attention; a huge eps uses representatives only."""
    heads, group, dim, tokens = 8, 4, 128, 131072
    data = synthetic.make_layer(0, 0, heads, tokens, dim, 32, device=DEV)
    s = build_summary(data.keys, data.values, RefineKVConfig())
    q = synthetic.make_queries(0, 0, 0, data.planted_mean, group)[0]
    ks, vs = data.keys[:, :64].contiguous(), data.values[:, :64].contiguous()
    dense = sparse_attention(q, s, ks, vs, RefineKVConfig(eps=0), return_selected=True)
    assert dense.selected.all()
    ek = torch.cat([data.keys, ks], 1).repeat_interleave(group, 0).float()
    ev = torch.cat([data.values, vs], 1).repeat_interleave(group, 0).float()
    want = F.scaled_dot_product_attention(q.reshape(heads * group, 1, dim).float(), ek, ev)
    torch.testing.assert_close(dense.output.float().reshape(-1, 1, dim), want, atol=2e-3,
                               rtol=2e-2)
    sparse = sparse_attention(q, s, ks, vs, RefineKVConfig(eps=1e9), return_selected=True)
    assert not sparse.selected.any()
    s_cpu = ora.as_cpu_summary(s)
    _, z = ora.select_blocks(q.cpu(), s_cpu, 1e9, "any")
    check_output(sparse.output, q, s_cpu, ks, vs, sparse.selected, z)
    lit = sparse_attention(q, s, ks, vs, RefineKVConfig(eps=0.01), return_selected=True)
    check_mask(lit.selected, q, s_cpu, RefineKVConfig(eps=0.01))


def test_cuda_graph_replay_matches_eager():
    data = synthetic.make_layer(8, 0, 8, 8192, 128, 32, device=DEV)
    cfg = RefineKVConfig(eps=0.01)
    s = build_summary(data.keys, data.values, cfg)
    q = synthetic.make_queries(8, 0, 0, data.planted_mean, 4)[0].clone()
    cap = 16
    sk = torch.randn(8, cap, 128, device=DEV).to(torch.bfloat16)
    sv = torch.randn(8, cap, 128, device=DEV).to(torch.bfloat16)
    length = torch.zeros((), device=DEV, dtype=torch.int32)
    workspace = {}
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        sparse_attention(q, s, sk, sv, cfg, workspace=workspace, suffix_length=length)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = sparse_attention(q, s, sk, sv, cfg, workspace=workspace, suffix_length=length).output
    for n in (3, 9, 16):
        length.fill_(n)
        graph.replay()
        torch.cuda.synchronize()
        want = sparse_attention(q, s, sk[:, :n], sv[:, :n], cfg).output
        assert torch.equal(out, want), n

"""Host logic of the Transformers adapter on the CPU (the scenarios of the reference's adapter tests).

The adapter's three kernel entry points (``build_summary``,
``select_blocks_union``, ``sparse_attention``) are replaced here by
oracle-backed stand-ins so that the session logic -- registration, hooks,
request reset, anchors, dense layers, static caches, stats, restore on exit
-- runs on tiny random-init Llama/Qwen2 models without a GPU.  The same
scenarios run on the real kernels in ``test_gpu_adapter.py``.  Model shapes
and seeds follow the reference's ``tests/test_transformers.py:10-30``.
"""

from __future__ import annotations

import pytest
import torch

transformers = pytest.importorskip("transformers")

from oracle import refinekv_oracle as ora  # noqa: E402
from refinekv_b200 import RefineKV, RefineKVConfig  # noqa: E402
from refinekv_b200.attention import AttentionResult  # noqa: E402
from refinekv_b200.integrations import transformers as adapter  # noqa: E402


@pytest.fixture
def oracle_backend(monkeypatch):
    calls = {"summaries": 0, "anchor_unions": 0, "decodes": 0}

    def build_summary(keys, values, config):
        calls["summaries"] += 1
        return ora.build_summary(keys.float(), values.float(), block_size=config.block_size)

    def select_blocks_union(queries, summary, config, *, workspace=None):
        calls["anchor_unions"] += 1
        return ora.anchor_union(queries.float(), summary, config.eps, config.gqa_reduction)

    def sparse_attention(query, summary, key_suffix, value_suffix, config, *, anchor_mask=None,
                         workspace=None, return_selected=False, suffix_length=None):
        calls["decodes"] += 1
        out, selected = ora.sparse_attention(query.float(), summary, key_suffix.float(),
                                             value_suffix.float(), config.eps,
                                             config.gqa_reduction, anchor_mask=anchor_mask)
        return AttentionResult(out.to(query.dtype), selected if return_selected else None)

    monkeypatch.setattr(adapter, "build_summary", build_summary)
    monkeypatch.setattr(adapter, "select_blocks_union", select_blocks_union)
    monkeypatch.setattr(adapter, "sparse_attention", sparse_attention)
    return calls


def _model(family="llama"):
    torch.manual_seed(9)
    config_type, model_type = (
        (transformers.LlamaConfig, transformers.LlamaForCausalLM) if family == "llama"
        else (transformers.Qwen2Config, transformers.Qwen2ForCausalLM))
    config = config_type(vocab_size=64, hidden_size=128, intermediate_size=256,
                         num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                         pad_token_id=0, eos_token_id=None)
    return model_type(config).eval()


def _generate(model, length=39, static=False):
    ids = torch.arange(length, device=model.device)[None] % 61 + 3
    options = {"cache_implementation": "static"} if static else {}
    return model.generate(input_ids=ids, attention_mask=torch.ones_like(ids), max_new_tokens=4,
                          do_sample=False, **options)


@pytest.mark.parametrize("family", ["llama", "qwen2"])
@pytest.mark.parametrize("static", [False, True])
def test_generation_with_anchors_stats_and_request_reset(oracle_backend, family, static):
    model = _model(family)
    original = model.config._attn_implementation
    hooks = len(model._forward_pre_hooks), len(model._forward_hooks)
    config = RefineKVConfig(anchor_tokens=3, eps=1e6, collect_stats=True)
    with RefineKV(model, config) as session:
        output = _generate(model, static=static)
        assert output.shape == (1, 43)
        if static:
            assert isinstance(session._cache.layers[0], adapter._VisibleStaticLayer)
        assert 0 < session.stats["equivalent_access_ratio"] <= 1
        assert session.stats["decode_attention_calls"] == 6  # 3 decode steps x 2 layers
        assert all(state.anchor_mask is not None for state in session._layers.values())
        assert oracle_backend["anchor_unions"] == 2  # one batched union per layer
        shorter = _generate(model, length=17, static=static)  # a new request resets the state
        assert shorter.shape == (1, 21)
        assert session.stats["decode_attention_calls"] == 6
        assert all(state.prompt_length == 17 for state in session._layers.values())
    assert model.config._attn_implementation == original
    assert hooks == (len(model._forward_pre_hooks), len(model._forward_hooks))
    assert not session._layers
    assert not hasattr(model, "_refinekv_session")
    assert all(not hasattr(layer.self_attn, "_refinekv_session") for layer in model.model.layers)


def test_huge_eps_decodes_from_representatives_and_anchors_only(oracle_backend):
    model = _model()
    with RefineKV(model, RefineKVConfig(anchor_tokens=2, eps=1e6, collect_stats=True)) as session:
        _generate(model, length=64)
        stats = session.stats
    # eps=1e6 expands no page beyond the anchors: access well below dense
    assert stats["equivalent_access_ratio"] < 0.9


def test_generation_config_static_uses_visible_cache(oracle_backend):
    model = _model()
    model.generation_config.cache_implementation = "static"
    with RefineKV(model) as session:
        assert _generate(model).shape == (1, 43)
        assert isinstance(session._cache.layers[0], adapter._VisibleStaticLayer)


def test_visible_static_cache_masks_and_lengths():
    model = _model()
    cache = adapter.make_visible_static_cache(model, 10)
    layer = cache.layers[0]
    k = torch.randn(1, 2, 4, 32)
    keys, values = layer.update(k, k.clone())
    assert keys.shape[2] == 4 and layer.get_seq_length() == 4
    assert layer.get_mask_sizes(1) == (5, 0)
    keys, _ = layer.update(k[:, :, :1], k[:, :, :1])
    assert keys.shape[2] == 5 and torch.equal(keys[:, :, :4], k)
    with pytest.raises(ValueError, match="capacity"):
        layer.update(torch.randn(1, 2, 6, 32), torch.randn(1, 2, 6, 32))
    with pytest.raises(ValueError):
        adapter.make_visible_static_cache(model, 0)


def test_stock_static_cache_is_rejected(oracle_backend):
    model = _model()
    ids = torch.arange(39)[None] % 61 + 3
    cache = transformers.StaticCache(config=model.config, max_cache_len=43)
    with RefineKV(model):
        with pytest.raises(ValueError, match="stock StaticCache is unsupported"):
            model.generate(input_ids=ids, max_new_tokens=4, past_key_values=cache)


def test_full_layers_match_native_generation_and_other_models_are_untouched(oracle_backend):
    model = _model()
    other = _model()
    with torch.inference_mode():
        expected = _generate(model)
    other_implementation = other.config._attn_implementation
    config = RefineKVConfig(full_attention_layers=2, collect_stats=True)
    with RefineKV(model, config) as session:
        actual = _generate(model)
        assert other.config._attn_implementation == other_implementation
    assert torch.equal(actual, expected)
    assert session.stats["equivalent_access_ratio"] == 1
    assert oracle_backend["summaries"] == 0 and oracle_backend["decodes"] == 0


def test_exception_and_nested_context_restore_model(oracle_backend):
    model = _model()
    original = model.config._attn_implementation
    with pytest.raises(ValueError, match="unpadded"):
        with RefineKV(model):
            with pytest.raises(RuntimeError, match="active"):
                with RefineKV(model):
                    pass
            model.generate(input_ids=torch.tensor([[0, 3, 4]]),
                           attention_mask=torch.tensor([[0, 1, 1]]), max_new_tokens=2)
    assert model.config._attn_implementation == original
    assert not hasattr(model, "_refinekv_session")


def test_context_rejects_training_mode_and_other_families():
    model = _model()
    model.train()
    with pytest.raises(ValueError, match="inference-only"):
        with RefineKV(model):
            pass
    model.eval()
    model.config.model_type = "mistral"
    with pytest.raises(ValueError, match="model_type"):
        with RefineKV(model):
            pass


@pytest.mark.parametrize("family", ["llama", "qwen2"])
def test_anchors_use_tail_projection(oracle_backend, family, monkeypatch):
    """A zero query has zero risk and selects no page; only the full-prompt GEMM is perturbed."""
    model = _model(family)
    for layer in model.model.layers:
        projection = layer.self_attn.q_proj
        with torch.no_grad():
            projection.weight.zero_()
            if projection.bias is not None:
                projection.bias.zero_()
        original = projection.forward

        def perturbed(hidden, original=original):
            result = original(hidden)
            return result + 1 if hidden.shape[1] > 2 else result

        monkeypatch.setattr(projection, "forward", perturbed)
    with RefineKV(model, RefineKVConfig(eps=0, anchor_tokens=2)) as session:
        _generate(model)
        assert all(not state.anchor_mask.any() for state in session._layers.values())


def test_cuda_graph_arguments_are_validated_before_any_work():
    model = _model()
    ids = torch.tensor([[3, 4, 5]])
    with RefineKV(model, cuda_graph=True):
        with pytest.raises(ValueError, match="fixed output"):
            model.generate(input_ids=ids, max_new_tokens=4, min_new_tokens=2, eos_token_id=None)
        with pytest.raises(ValueError, match="max_new_tokens"):
            model.generate(input_ids=ids, max_new_tokens=3, min_new_tokens=3, eos_token_id=None)
        with pytest.raises(ValueError, match="does not support"):
            model.generate(input_ids=ids, max_new_tokens=4, min_new_tokens=4, eos_token_id=None,
                           temperature=0.5)
        with pytest.raises(ValueError, match="CUDA BF16"):  # a CPU model is refused
            model.generate(input_ids=ids, max_new_tokens=4, min_new_tokens=4, eos_token_id=None)


class _OracleBatch:
    """Stand-in batched summary: one oracle summary per prompt (rows stacked per prompt)."""

    def __init__(self, parts):
        self.parts = parts


@pytest.fixture
def oracle_batch_backend(monkeypatch, oracle_backend):
    single_union, single_decode = adapter.select_blocks_union, adapter.sparse_attention
    calls = {"summaries": 0, "anchor_unions": 0, "decodes": 0}

    def build_summary_batch(keys, values, config):
        calls["summaries"] += 1
        return _OracleBatch([ora.build_summary(k.float(), v.float(), block_size=config.block_size)
                             for k, v in zip(keys, values)])

    def select_blocks_union(queries, summary, config, *, workspace=None):
        if not isinstance(summary, _OracleBatch):
            return single_union(queries, summary, config, workspace=workspace)
        calls["anchor_unions"] += 1
        h = queries.shape[1] // len(summary.parts)
        return [ora.anchor_union(queries[:, i * h:(i + 1) * h].float(), s, config.eps,
                                 config.gqa_reduction) for i, s in enumerate(summary.parts)]

    def sparse_attention(query, summary, key_suffix, value_suffix, config, *, anchor_mask=None,
                         workspace=None, return_selected=False, suffix_length=None):
        if not isinstance(summary, _OracleBatch):
            return single_decode(query, summary, key_suffix, value_suffix, config,
                                 anchor_mask=anchor_mask, return_selected=return_selected)
        calls["decodes"] += 1
        h = query.shape[0] // len(summary.parts)
        outs = []
        for i, s in enumerate(summary.parts):
            r = slice(i * h, (i + 1) * h)
            out, _ = ora.sparse_attention(query[r].float(), s, key_suffix[r].float(),
                                          value_suffix[r].float(), config.eps,
                                          config.gqa_reduction,
                                          anchor_mask=None if anchor_mask is None else anchor_mask[i])
            outs.append(out)
        return AttentionResult(torch.cat(outs).to(query.dtype), None)

    monkeypatch.setattr(adapter, "build_summary_batch", build_summary_batch)
    monkeypatch.setattr(adapter, "select_blocks_union", select_blocks_union)
    monkeypatch.setattr(adapter, "sparse_attention", sparse_attention)
    return calls


def _prefill_and_step(model, ids, mask, token):
    """Dense prefill then one decode step, positions from the padding as generate sets them."""
    cache = transformers.DynamicCache(config=model.config)
    positions = (mask.cumsum(1) - 1).clamp(min=0)
    first = model(input_ids=ids, attention_mask=mask, position_ids=positions,
                  past_key_values=cache, use_cache=True).logits[:, -1]
    mask = torch.cat([mask, torch.ones_like(mask[:, :1])], 1)
    step = model(input_ids=token, attention_mask=mask, position_ids=positions[:, -1:] + 1,
                 past_key_values=cache, use_cache=True).logits[:, -1]
    return first, step


@pytest.mark.parametrize("family", ["llama", "qwen2"])
def test_left_padded_batch_decodes_like_each_prompt_alone(family, oracle_batch_backend):
    """Beyond the reference (batch 1): a left-padded batch, one summary per row's own prompt."""
    model = _model(family)
    config = RefineKVConfig(eps=0.05, anchor_tokens=16, full_attention_layers=1)
    lengths = (9, 40, 23)  # the 9-token prompt is shorter than the 16 anchors
    width = max(lengths)
    ids = torch.zeros(len(lengths), width, dtype=torch.long)
    mask = torch.zeros_like(ids)
    prompts = [torch.arange(n) % 61 + 3 + i for i, n in enumerate(lengths)]
    for i, p in enumerate(prompts):
        ids[i, width - len(p):] = p
        mask[i, width - len(p):] = 1
    token = torch.tensor([[5], [7], [11]])
    with RefineKV(model, config):
        first, step = _prefill_and_step(model, ids, mask, token)
    # layer 0 dense, layer 1 through the batched summary, anchors and decode
    assert oracle_batch_backend == {"summaries": 1, "anchor_unions": 1, "decodes": 1}
    for i, p in enumerate(prompts):
        with RefineKV(model, config):
            first_i, step_i = _prefill_and_step(model, p[None], torch.ones_like(p[None]),
                                                token[i:i + 1])
        torch.testing.assert_close(first[i], first_i[0], atol=1e-4, rtol=1e-4)
        torch.testing.assert_close(step[i], step_i[0], atol=1e-4, rtol=1e-4)


def test_batch_rejects_right_padding_and_beams(oracle_batch_backend):
    model = _model()
    ids = torch.full((2, 6), 4, dtype=torch.long)
    right = torch.tensor([[1, 1, 1, 1, 1, 1], [1, 1, 1, 1, 0, 0]])
    with RefineKV(model, RefineKVConfig()):
        with pytest.raises(ValueError, match="left-padded"):
            model(input_ids=ids, attention_mask=right,
                  past_key_values=transformers.DynamicCache(config=model.config), use_cache=True)
        with pytest.raises(ValueError, match="num_beams"):
            model.generate(input_ids=ids, attention_mask=torch.ones_like(ids), num_beams=2,
                           max_new_tokens=2, do_sample=False)

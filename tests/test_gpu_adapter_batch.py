"""Transformers adapter with a left-padded batch of prompts, on the B200 kernels.

Beyond the reference adapter, which decodes one sequence
(``transformers.py:448-449``).  Each row of a batch keeps a summary of its
own prompt (the padding excluded), so one batched decode step must give every
row the logits of that prompt decoded alone, to bf16 rounding (the padded
prefill and the stacked kernels round differently in the last bits); a
captured decode step gives the eager batch's tokens exactly.
"""

from __future__ import annotations

import pytest
import torch

transformers = pytest.importorskip("transformers")

from refinekv_b200 import RefineKV, RefineKVConfig  # noqa: E402
from test_gpu_adapter import _model  # noqa: E402

pytestmark = pytest.mark.gpu
LENGTHS = (39, 300, 120)


def _batch(lengths, vocab=64):
    width = max(lengths)
    ids = torch.zeros(len(lengths), width, dtype=torch.long, device="cuda")
    mask = torch.zeros_like(ids)
    prompts = [(torch.arange(n, device="cuda") * (i + 3)) % (vocab - 3) + 3
               for i, n in enumerate(lengths)]
    for i, p in enumerate(prompts):
        ids[i, width - len(p):] = p
        mask[i, width - len(p):] = 1
    return ids, mask, prompts


def _prefill_and_step(model, ids, mask, token):
    cache = transformers.DynamicCache(config=model.config)
    positions = (mask.cumsum(1) - 1).clamp(min=0)
    first = model(input_ids=ids, attention_mask=mask, position_ids=positions,
                  past_key_values=cache, use_cache=True).logits[:, -1].float()
    mask = torch.cat([mask, torch.ones_like(mask[:, :1])], 1)
    step = model(input_ids=token, attention_mask=mask, position_ids=positions[:, -1:] + 1,
                 past_key_values=cache, use_cache=True).logits[:, -1].float()
    return first, step


@pytest.mark.parametrize("family", ["llama", "qwen2"])
@pytest.mark.parametrize("reduction,anchors", [("any", 4), ("mean", 0)])
def test_batch_step_matches_each_prompt_alone(family, reduction, anchors):
    model = _model(family)
    config = RefineKVConfig(eps=0.01, gqa_reduction=reduction, anchor_tokens=anchors)
    ids, mask, prompts = _batch(LENGTHS)
    token = torch.tensor([[5], [7], [11]], device="cuda")
    with torch.inference_mode(), RefineKV(model, config):
        first, step = _prefill_and_step(model, ids, mask, token)
    for i, p in enumerate(prompts):
        with torch.inference_mode(), RefineKV(model, config):
            first_i, step_i = _prefill_and_step(model, p[None], torch.ones_like(p[None]),
                                                token[i:i + 1])
        for got, want in ((first[i], first_i[0]), (step[i], step_i[0])):
            scale = float(want.abs().max())
            assert float((got - want).abs().max()) <= 0.02 * scale


@pytest.mark.parametrize("family", ["llama", "qwen2"])
def test_batch_generate_dynamic_and_static_caches_agree(family):
    model = _model(family, layers=3)
    config = RefineKVConfig(eps=0.01, anchor_tokens=4, full_attention_layers=1,
                            collect_stats=True)
    ids, mask, _ = _batch(LENGTHS)
    opts = dict(input_ids=ids, attention_mask=mask, max_new_tokens=6, min_new_tokens=6,
                do_sample=False, eos_token_id=None, pad_token_id=0)
    with RefineKV(model, config) as session:
        dynamic = model.generate(**opts)
        assert 0 < session.stats["equivalent_access_ratio"] <= 1
        assert session.stats["decode_attention_calls"] == 3 * 5
    with RefineKV(model, config):
        static = model.generate(**opts, cache_implementation="static")
    assert dynamic.shape == (len(LENGTHS), max(LENGTHS) + 6)
    assert torch.equal(dynamic, static)


@pytest.mark.parametrize("family", ["llama", "qwen2"])
@pytest.mark.parametrize("dense_layers", [0, 1])
def test_batch_cuda_graph_decode_matches_eager(family, dense_layers):
    """One captured step for a left-padded batch gives the eager batch's tokens."""
    model = _model(family, layers=3)
    if family == "qwen2":
        model.generation_config.repetition_penalty = 1.05
    config = RefineKVConfig(eps=0.01, anchor_tokens=4, full_attention_layers=dense_layers)
    ids, mask, _ = _batch(LENGTHS)
    opts = dict(input_ids=ids, attention_mask=mask, max_new_tokens=8, min_new_tokens=8,
                do_sample=False, eos_token_id=None, pad_token_id=0)
    with RefineKV(model, config):
        eager = model.generate(**opts)
    with RefineKV(model, config, cuda_graph=True):
        graph = model.generate(**opts)
    assert torch.equal(graph, eager)


def test_cuda_graph_refuses_right_padding():
    model = _model()
    ids = torch.full((2, 8), 4, dtype=torch.long, device="cuda")
    right = torch.ones_like(ids)
    right[1, -2:] = 0
    with RefineKV(model, cuda_graph=True):
        with pytest.raises(ValueError, match="left-padded"):
            model.generate(input_ids=ids, attention_mask=right, max_new_tokens=4,
                           min_new_tokens=4, eos_token_id=None)

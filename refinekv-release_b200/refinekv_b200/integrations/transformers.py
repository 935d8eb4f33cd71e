"""Transformers adapter: dense prefill, then RefineKV decode on the B200 kernels.

Public surface of the reference adapter (``src/refinekv/integrations/transformers.py``):
``RefineKV(model, config, *, cuda_graph=False)`` as a context manager with a
``stats`` property, and ``make_visible_static_cache(model, max_cache_len)``.
The session registers a named attention implementation with Transformers'
attention interface (the reference does the same, ``:126-129``), never
replacing the library's own functions, and restores the model on exit.

Per layer, the first call of a request is the dense prompt prefill (SDPA,
exactly the native path); the adapter then builds the block summaries
(``rkv_summarize``) and, with ``anchor_tokens``, ORs the masks of the
prompt's last queries in one batched selector launch pair instead of one
selector chain per anchor (``:539-552`` of the reference).  Every later call
is a single-token decode through ``rkv_decode``; the first
``full_attention_layers`` layers stay dense.

Changes from the reference, all for transformers 5.5 (the version installed
here) or from the B200 design:

* cache layers take the 5.5 signatures (``update(k, v, *args)``,
  ``get_mask_sizes(query_length: int)``); the reference's visible cache breaks
  on the latter;
* CUDA-graph decode no longer needs ``cache_position`` (5.5 dropped it from
  the model forward): the graph cache writes at a device-side cursor;
* ``full_attention_layers`` works under CUDA graphs (the reference refuses):
  a dense layer of one sequence decodes with ``dense_attention`` (the
  refinement kernel over all of the prompt's pages and the suffix up to the
  device length, no mask); a left-padded batch's dense layers attend over the
  fixed-capacity cache with a device-side mask;
* beyond the reference (batch 1 only, ``:448-449``), decode also takes a
  left-padded batch of prompts, eagerly or from one captured CUDA graph:
  each row's summary covers its own prompt (the padding excluded) and all
  rows decode in one batched launch set (``build_summary_batch``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from functools import wraps

import torch

try:
    from transformers import AttentionInterface, AttentionMaskInterface
    from transformers.cache_utils import Cache, StaticCache, StaticLayer
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
except ImportError as error:  # pragma: no cover - exercised only without transformers
    raise ImportError("the Transformers adapter needs the `transformers` package") from error

from ..attention import dense_attention, select_blocks_union, sparse_attention
from ..config import RefineKVConfig
from ..summary import (BlockSummary, PageView, build_summary, build_summary_batch,
                       build_summary_into, page_view)

ATTN_IMPLEMENTATION = "refinekv_b200"
_MISSING = object()


# ---------------------------------------------------------------------------
# caches
# ---------------------------------------------------------------------------

def _write_prompt(layer, key_states, value_states, end):
    """A static layer's prefill write, fused with the layer's summary when asked for.

    The session sets ``summary_config`` on the layers it summarises; for one
    sequence on the GPU whose padded last page fits the capacity, the prompt
    reaches the cache through ``build_summary_into``, which summarises it in
    the same pass (``fused_summary``, picked up by the session's prefill).
    """
    config = getattr(layer, "summary_config", None)
    if (config is not None and key_states.shape[0] == 1 and key_states.is_cuda
            and key_states.dtype == torch.bfloat16
            and -(-end // config.block_size) * config.block_size <= layer.max_cache_len):
        layer.fused_summary = build_summary_into(key_states[0], value_states[0], layer.keys[0],
                                                 layer.values[0], config)
        return
    layer.keys[:, :, :end].copy_(key_states)
    layer.values[:, :, :end].copy_(value_states)

def decode_access_counts(selected, counts, groups, query_heads, suffix_tokens):
    """K/V rows one decode step of a layer reads, the reference's access counter.

    ``integrations/transformers.py:590-594``: every row of a selected block and
    one representative of every other block, for each of the ``groups`` query
    rows of a KV head, plus the visible suffix for every one of the
    ``query_heads``.  ``counts`` (tokens per block) broadcasts against the
    (kv_heads, blocks) mask ``selected``; a batch's padding blocks (count 0)
    cost nothing.  Returns a 0-d device tensor (no host sync).
    """
    real = counts > 0
    accessed = ((selected * counts).sum() + (~selected & real).sum()) * groups
    return accessed + query_heads * suffix_tokens


class _VisibleStaticLayer(StaticLayer):
    """Preallocated KV that exposes only the tokens written so far (``:25-62`` of the reference)."""

    is_compileable = False

    def __init__(self, max_cache_len: int):
        super().__init__(max_cache_len)
        self.visible = 0

    def lazy_initialization(self, key_states, value_states):
        self.dtype, self.device = key_states.dtype, key_states.device
        self.max_batch_size, self.num_heads = key_states.shape[:2]
        self.k_head_dim, self.v_head_dim = key_states.shape[-1], value_states.shape[-1]
        shape = (self.max_batch_size, self.num_heads, self.max_cache_len)
        self.keys = torch.empty(*shape, self.k_head_dim, dtype=self.dtype, device=self.device)
        self.values = torch.empty(*shape, self.v_head_dim, dtype=self.dtype, device=self.device)
        self.is_initialized = True

    def update(self, key_states, value_states, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        end = self.visible + key_states.shape[-2]
        if end > self.max_cache_len:
            raise ValueError("visible KV cache capacity exceeded")
        if self.visible == 0:  # the prompt
            _write_prompt(self, key_states, value_states, end)
        else:
            self.keys[:, :, self.visible:end].copy_(key_states)
            self.values[:, :, self.visible:end].copy_(value_states)
        self.visible = end
        return self.keys[:, :, :end], self.values[:, :, :end]

    def get_mask_sizes(self, query_length, *args):
        return self.visible + int(query_length), 0

    def get_seq_length(self):
        return self.visible


def make_visible_static_cache(model, max_cache_len):
    """A preallocated cache whose visible prefix grows with each write (mask-free prefill)."""
    if not isinstance(max_cache_len, int) or isinstance(max_cache_len, bool) or max_cache_len <= 0:
        raise ValueError("max_cache_len must be a positive integer")
    return Cache(layers=[_VisibleStaticLayer(max_cache_len) for _ in model.model.layers])


class _GraphCursor:
    """Device-side decode position shared by every layer of a graph cache."""

    def __init__(self, device):
        self.position = torch.zeros(1, device=device, dtype=torch.long)


class _GraphStaticLayer(StaticLayer):
    """Fixed KV addresses: one prompt prefill, then writes at the device cursor."""

    is_compileable = False

    def __init__(self, max_cache_len: int, cursor: _GraphCursor):
        super().__init__(max_cache_len)
        self.cursor = cursor
        self.visible = 0
        self.graph_decode = False

    def lazy_initialization(self, key_states, value_states):
        _VisibleStaticLayer.lazy_initialization(self, key_states, value_states)

    def update(self, key_states, value_states, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        if not self.graph_decode:
            end = key_states.shape[-2]
            if self.visible or end > self.max_cache_len:
                raise ValueError("the graph cache takes one complete prompt prefill")
            _write_prompt(self, key_states, value_states, end)
            self.visible = end
            return self.keys[:, :, :end], self.values[:, :, :end]
        self.keys.index_copy_(2, self.cursor.position, key_states)
        self.values.index_copy_(2, self.cursor.position, value_states)
        return self.keys, self.values

    def get_mask_sizes(self, query_length, *args):
        return (self.max_cache_len if self.graph_decode else int(query_length)), 0

    def get_seq_length(self):
        return self.visible


# ---------------------------------------------------------------------------
# session
# ---------------------------------------------------------------------------

@dataclass
class _LayerState:
    prompt_length: int
    visible_length: int
    summary: BlockSummary | None = None
    anchor_mask: torch.Tensor | None = None
    workspace: dict = field(default_factory=dict)
    pages: PageView | None = None  # a dense layer's page view of the graph cache
    pads: list | None = None  # left padding per row of a batch
    pad_rows: torch.Tensor | None = None  # the same, (rows, 1, 1, 1) on the device


def _attention_forward(module, query, key, value, attention_mask, dropout=0.0, scaling=None,
                       **kwargs):
    session = getattr(module, "_refinekv_session", None)
    if session is None:
        raise RuntimeError("the refinekv_b200 attention runs only inside a RefineKV context")
    return session._attention(module, query, key, value, attention_mask, scaling, kwargs)


def _register():
    # A named implementation next to Transformers' own; its masks are SDPA's.
    AttentionInterface.register(ATTN_IMPLEMENTATION, _attention_forward)
    AttentionMaskInterface.register(ATTN_IMPLEMENTATION, AttentionMaskInterface()["sdpa"])


def _rotary(model_type):
    if model_type == "qwen2":
        from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb
    else:
        from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
    return apply_rotary_pos_emb


class RefineKV:
    """Dense prefill followed by RefineKV single-sequence decode, scoped to one model.

    Example::

        with RefineKV(model, RefineKVConfig(anchor_tokens=32)):
            output = model.generate(**inputs, max_new_tokens=128, do_sample=False)

    Same contract as the reference (``transformers.py:132-146``): the model is
    in evaluation mode, of the Llama or Qwen2/Qwen2.5 family, on a B200 in
    bf16 for the sparse layers; every generation starts from an empty cache
    with one unpadded prompt; DynamicCache, ``cache_implementation="static"``
    and :func:`make_visible_static_cache` are supported.  ``cuda_graph=True``
    runs fixed-length greedy decode from one captured CUDA graph per request.
    Beyond the reference, generation (eager or CUDA graph) also takes a batch
    of prompts, left-padded as Transformers pads decoder-only batches
    (``num_beams=1``).
    """

    def __init__(self, model, config: RefineKVConfig | None = None, *, cuda_graph=False):
        self.model = model
        self.config = config or RefineKVConfig()
        self.cuda_graph = cuda_graph
        self._graph_mode = False
        self._graph_suffix_length = None
        self._graph_capacity = 0
        self._layers: dict[int, _LayerState] = {}
        self._anchor_queries: dict[int, torch.Tensor] = {}
        self._handles = []
        self._cache = None
        self._pads = None
        self._active = False
        self._totals = dict(accessed=0, dense=0, decode_attention_calls=0)

    # ---- statistics --------------------------------------------------------
    @property
    def stats(self):
        """Decode-only equivalent KV access (reference ``transformers.py:162-175``).

        An unexpanded page counts as one representative.  Reading this
        synchronises with the device when the counters are device tensors.
        """
        totals = {k: (v.item() if torch.is_tensor(v) else v) for k, v in self._totals.items()}
        totals["equivalent_access_ratio"] = (
            totals["accessed"] / totals["dense"] if totals["dense"] else None)
        return totals

    def _record(self, accessed, dense):
        self._totals["accessed"] = self._totals["accessed"] + accessed
        self._totals["dense"] += dense
        self._totals["decode_attention_calls"] += 1

    def _reset_request(self, cache):
        self._layers.clear()
        self._anchor_queries.clear()
        self._totals = dict(accessed=0, dense=0, decode_attention_calls=0)
        self._cache = cache
        self._pads = None

    # ---- context -----------------------------------------------------------
    def __enter__(self):
        if self._active or hasattr(self.model, "_refinekv_session"):
            raise RuntimeError("this model already has an active RefineKV context")
        if self.model.training:
            raise ValueError("RefineKV is inference-only; call model.eval() first")
        if self.model.config.model_type not in ("llama", "qwen2"):
            raise ValueError("the Transformers adapter supports model_type='llama' or 'qwen2'")
        if getattr(self.model.config, "use_sliding_window", False):
            raise ValueError("sliding-window attention is not supported")
        if getattr(self.model.config, "output_attentions", False):
            raise ValueError("RefineKV does not return attention weights")
        self._modules = list(self.model.model.layers)
        if any(getattr(layer.self_attn, "sliding_window", None) is not None
               for layer in self._modules):
            raise ValueError("sliding-window attention is not supported")
        _register()
        self._original_implementation = self.model.config._attn_implementation
        self._original_layer_implementations = [
            layer.self_attn.config._attn_implementation for layer in self._modules]
        self._inference = torch.inference_mode()
        self._inference.__enter__()
        try:
            self.model.set_attn_implementation(ATTN_IMPLEMENTATION)
            self.model._refinekv_session = self
            self._module_indices = {}
            for index, layer in enumerate(self._modules):
                layer.self_attn._refinekv_session = self
                self._module_indices[id(layer.self_attn)] = index
                if self.config.anchor_tokens and index >= self.config.full_attention_layers:
                    self._handles.append(layer.self_attn.register_forward_pre_hook(
                        self._capture_anchor_queries, with_kwargs=True))
            self._original_generate_attribute = self.model.__dict__.get("generate", _MISSING)
            self.model.generate = self._wrap_generate(self.model.generate)
            self._handles.append(
                self.model.register_forward_pre_hook(self._before_forward, with_kwargs=True))
            self._handles.append(
                self.model.register_forward_hook(self._after_forward, with_kwargs=True))
            self._active = True
            return self
        except BaseException:
            self._restore()
            self._inference.__exit__(None, None, None)
            raise

    def _wrap_generate(self, original_generate):
        @wraps(original_generate)
        def generate(*args, **kwargs):
            self._reset_request(None)
            if self.cuda_graph:
                return self._generate_cuda_graph(*args, **kwargs)
            if isinstance(kwargs.get("past_key_values"), StaticCache):
                raise ValueError("stock StaticCache is unsupported; use "
                                 "cache_implementation='static' or make_visible_static_cache")
            generation = kwargs.get("generation_config") or self.model.generation_config
            if (kwargs.get("num_beams", generation.num_beams) or 1) != 1:
                # Beam search reorders the cache; the summaries cannot follow.
                raise ValueError("RefineKV requires num_beams=1")
            implementation = kwargs.get("cache_implementation", generation.cache_implementation)
            if implementation == "static":
                if kwargs.get("past_key_values") is not None:
                    raise ValueError("pass either a static cache request or past_key_values")
                inputs = kwargs.get("input_ids")
                if inputs is None and args:
                    inputs = args[0]
                if not isinstance(inputs, torch.Tensor) or inputs.ndim != 2:
                    raise ValueError(
                        "static cache generation requires input_ids of shape (batch, tokens)")
                prompt = inputs.shape[1]
                new_tokens = kwargs.get("max_new_tokens", generation.max_new_tokens)
                capacity = (prompt + int(new_tokens) if new_tokens is not None
                            else int(kwargs.get("max_length", generation.max_length)))
                if capacity <= prompt:
                    raise ValueError("static cache capacity must exceed prompt length")
                kwargs["past_key_values"] = make_visible_static_cache(self.model, capacity)
                kwargs["cache_implementation"] = None
            kwargs["disable_compile"] = True  # summaries are built outside compiled forwards
            return original_generate(*args, **kwargs)

        return generate

    def _restore(self):
        for handle in self._handles:
            handle.remove()
        self._handles.clear()
        for layer, original in zip(getattr(self, "_modules", []),
                                   getattr(self, "_original_layer_implementations", [])):
            if getattr(layer.self_attn, "_refinekv_session", None) is self:
                del layer.self_attn._refinekv_session
            layer.self_attn.config._attn_implementation = original
        if getattr(self.model, "_refinekv_session", None) is self:
            del self.model._refinekv_session
        if hasattr(self, "_original_generate_attribute"):
            if self._original_generate_attribute is _MISSING:
                self.model.__dict__.pop("generate", None)
            else:
                self.model.generate = self._original_generate_attribute
        if hasattr(self, "_original_implementation"):
            self.model.config._attn_implementation = self._original_implementation
        self._layers.clear()
        self._anchor_queries.clear()
        self._cache = None
        self._graph_mode = False
        self._graph_suffix_length = None
        self._active = False

    def __exit__(self, exc_type, exc_value, traceback):
        try:
            self._restore()
        finally:
            self._inference.__exit__(exc_type, exc_value, traceback)
        return False

    # ---- CUDA-graph generation ---------------------------------------------
    _GRAPH_KWARGS = {
        "input_ids", "attention_mask", "max_new_tokens", "min_new_tokens", "do_sample",
        "num_beams", "use_cache", "eos_token_id", "forced_eos_token_id", "pad_token_id",
        "cache_implementation", "disable_compile", "repetition_penalty",
    }
    _UNSUPPORTED_PROCESSORS = {
        "encoder_repetition_penalty": (None, 1.0), "no_repeat_ngram_size": (None, 0),
        "bad_words_ids": (None, []), "suppress_tokens": (None, []),
        "begin_suppress_tokens": (None, []), "forced_bos_token_id": (None,),
        "sequence_bias": (None, {}), "force_words_ids": (None, []), "constraints": (None, []),
        "watermarking_config": (None,),
    }

    def _graph_arguments(self, args, kwargs):
        """Restates the reference's graph-generation contract (``transformers.py:304-382``):
        the same whitelist, checks and messages, so callers see the same errors.
        Returns (input_ids, max_new_tokens, penalty, mask)."""
        unsupported = set(kwargs) - self._GRAPH_KWARGS
        if unsupported:
            raise ValueError(f"CUDA Graph generation does not support {sorted(unsupported)}")
        if args:
            if len(args) != 1 or "input_ids" in kwargs:
                raise ValueError("pass one input_ids tensor to CUDA Graph generation")
            input_ids = args[0]
        else:
            input_ids = kwargs.get("input_ids")
        if (not isinstance(input_ids, torch.Tensor) or input_ids.ndim != 2
                or input_ids.dtype != torch.long):
            raise ValueError("CUDA Graph generation requires an input_ids tensor (batch, tokens)")
        max_new_tokens = kwargs.get("max_new_tokens")
        if not isinstance(max_new_tokens, int) or max_new_tokens < 4:
            raise ValueError("CUDA Graph generation requires max_new_tokens >= 4")
        if (kwargs.get("min_new_tokens") != max_new_tokens
                or "eos_token_id" not in kwargs or kwargs["eos_token_id"] is not None):
            raise ValueError("CUDA Graph generation requires fixed output: "
                             "min_new_tokens=max_new_tokens and eos_token_id=None")
        generation = self.model.generation_config
        if (kwargs.get("do_sample", generation.do_sample)
                or (kwargs.get("num_beams", generation.num_beams) or 1) != 1
                or kwargs.get("use_cache", generation.use_cache) not in (None, True)
                or kwargs.get("forced_eos_token_id", generation.forced_eos_token_id) is not None
                or kwargs.get("cache_implementation", generation.cache_implementation)
                not in (None, "static")
                or (generation.num_return_sequences or 1) != 1):
            raise ValueError(
                "CUDA Graph generation supports greedy, single-beam, static-cache decode only")
        penalty = kwargs.get("repetition_penalty", getattr(generation, "repetition_penalty", 1.0))
        penalty = 1.0 if penalty is None else float(penalty)
        if not math.isfinite(penalty) or penalty <= 0:
            raise ValueError("repetition_penalty must be finite and positive")
        active = [name for name, defaults in self._UNSUPPORTED_PROCESSORS.items()
                  if getattr(generation, name, None) not in defaults]
        if active:
            raise ValueError(f"CUDA Graph generation does not support logits processors {active}")
        if (not input_ids.is_cuda or input_ids.device != self.model.device
                or self.model.dtype != torch.bfloat16 or self.config.backend == "torch"
                or self.config.collect_stats):
            raise ValueError("CUDA Graph requires a CUDA BF16 model, the CUDA backend and no stats")
        mask = kwargs.get("attention_mask")
        if mask is not None:
            if (not isinstance(mask, torch.Tensor) or mask.shape != input_ids.shape
                    or mask.device != input_ids.device):
                raise ValueError("attention_mask must match input_ids")
            rows = mask.bool()
            left_padded = bool(rows[:, -1].all()) and bool((rows[:, 1:] >= rows[:, :-1]).all())
            if not (bool(rows.all()) or (input_ids.shape[0] > 1 and left_padded)):
                raise ValueError("CUDA Graph generation requires an unpadded prompt "
                                 "(a batch may be left-padded)")
        return input_ids, max_new_tokens, penalty, mask

    def _generate_cuda_graph(self, *args, **kwargs):
        """Prefill eagerly, capture one greedy decode step, replay it: restates the
        reference's warm-up, capture and replay protocol (``transformers.py:302-440``)."""
        input_ids, max_new_tokens, penalty, mask = self._graph_arguments(args, kwargs)
        device = input_ids.device
        rows, prompt_length = input_ids.shape
        cursor = _GraphCursor(device)
        # Whole 64-token pages: a dense layer's page view of the cache (any
        # block size) must stay inside the allocation.
        capacity = -(-(prompt_length + max_new_tokens) // 64) * 64
        cache = Cache(layers=[_GraphStaticLayer(capacity, cursor) for _ in self.model.model.layers])
        # Left padding (a batch): each row's positions count its real tokens only.
        pads = torch.zeros(rows, 1, device=device, dtype=torch.long)
        positions = None
        if mask is not None and not bool(mask.all()):
            pads = (mask == 0).sum(1, keepdim=True)
            positions = (mask.long().cumsum(1) - 1).clamp(min=0)
        prefill = self.model(input_ids=input_ids, attention_mask=mask, position_ids=positions,
                             past_key_values=cache, use_cache=True, logits_to_keep=1)
        seen = None
        if penalty != 1.0:
            seen = torch.zeros_like(prefill.logits[:, -1], dtype=torch.bool)
            seen.scatter_(1, input_ids, True)

        def greedy(scores):
            scores = scores.float()
            if seen is not None:
                adjusted = torch.where(scores < 0, scores * penalty, scores / penalty)
                scores = torch.where(seen, adjusted, scores)
            return scores.argmax(-1, keepdim=True)

        token = greedy(prefill.logits[:, -1]).clone()  # (rows, 1)
        output_tokens = torch.empty(max_new_tokens, rows, device=device, dtype=input_ids.dtype)
        output_tokens[:1].copy_(token.reshape(1, rows))
        del prefill
        for layer in cache.layers:
            layer.graph_decode = True
        cursor.position.fill_(prompt_length)
        output_index = torch.ones(1, device=device, dtype=torch.long)
        self._graph_suffix_length = torch.zeros((), device=device, dtype=torch.int32)
        self._graph_capacity = capacity
        self._graph_mode = True

        def step():
            self._graph_suffix_length.add_(1)
            if seen is not None:
                seen.scatter_(1, token, True)
            result = self.model(input_ids=token, attention_mask=None, past_key_values=cache,
                                position_ids=cursor.position.view(1, 1) - pads, use_cache=True,
                                logits_to_keep=1)
            following = greedy(result.logits[:, -1])
            output_tokens.index_copy_(0, output_index, following.reshape(1, rows))
            token.copy_(following)
            cursor.position.add_(1)
            output_index.add_(1)

        graph = None
        try:
            warmup_steps = min(2, max_new_tokens - 2)
            stream = torch.cuda.Stream(device=device)
            stream.wait_stream(torch.cuda.current_stream(device))
            with torch.cuda.stream(stream):
                for _ in range(warmup_steps):
                    step()
            torch.cuda.current_stream(device).wait_stream(stream)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step()
            # Capture only records; the replays produce the remaining tokens.
            for _ in range(max_new_tokens - 1 - warmup_steps):
                graph.replay()
            torch.cuda.synchronize(device)
            return torch.cat((input_ids, output_tokens.t()), dim=1)
        finally:
            del graph
            self._graph_mode = False
            self._graph_suffix_length = None

    # ---- hooks -------------------------------------------------------------
    def _before_forward(self, module, args, kwargs):
        inputs = kwargs.get("input_ids")
        if inputs is None:
            inputs = kwargs.get("inputs_embeds")
        if inputs is None and args:
            inputs = args[0]
        batch = inputs.shape[0] if inputs is not None else 1
        if not kwargs.get("use_cache", self.model.config.use_cache):
            raise ValueError("RefineKV requires use_cache=True")
        if kwargs.get("output_attentions", False):
            raise ValueError("RefineKV does not return attention weights")
        cache = kwargs.get("past_key_values")
        if cache is None or cache is not self._cache:
            if cache is not None and cache.get_seq_length() != 0:
                raise ValueError("start each RefineKV generation with an empty KV cache")
            mask = kwargs.get("attention_mask")
            if isinstance(mask, dict):
                mask = mask.get("full_attention")
            pads = None
            if mask is not None:
                if mask.ndim == 2 and batch > 1:
                    # A batch may be left-padded: every row 0...0 1...1.
                    rows = mask.bool()
                    valid = bool(rows[:, -1].all()) and bool((rows[:, 1:] >= rows[:, :-1]).all())
                    pads = (~rows).sum(1).tolist()
                elif mask.ndim == 2:
                    valid = bool(mask.all())
                elif mask.ndim == 4 and inputs is not None and batch == 1:
                    last = mask[0, 0, -1, :inputs.shape[1]]
                    valid = bool(last.all()) if mask.dtype == torch.bool else bool((last == 0).all())
                else:
                    valid = False
                if not valid:
                    raise ValueError("RefineKV requires an unpadded prompt (a batch may be "
                                     "left-padded, with a 2-D attention_mask)")
            self._reset_request(cache)
            self._pads = pads
            for i, layer in enumerate(getattr(cache, "layers", None) or []):
                if isinstance(layer, (_VisibleStaticLayer, _GraphStaticLayer)):
                    layer.summary_config = (self.config if i >= self.config.full_attention_layers
                                            else None)
                    layer.fused_summary = None

    def _after_forward(self, module, args, kwargs, output):
        cache = getattr(output, "past_key_values", None)
        if cache is not None:
            self._cache = cache

    def _capture_anchor_queries(self, module, args, kwargs):
        """Project the prompt's last ``anchor_tokens`` hidden states to RoPE'd queries.

        The tail is projected on its own, as in the reference
        (``transformers.py:485-508``): a full-prompt GEMM can round differently
        in bf16 and move blocks across the eps threshold.
        """
        index = self._module_indices[id(module)]
        if index in self._layers:
            return
        hidden = kwargs.get("hidden_states")
        if hidden is None and args:
            hidden = args[0]
        positions = kwargs.get("position_embeddings")
        if positions is None and len(args) > 1:
            positions = args[1]
        if hidden is None or positions is None:
            raise RuntimeError("prompt anchors require hidden states and RoPE embeddings")
        count = min(self.config.anchor_tokens, hidden.shape[1])
        tail = hidden[:, -count:]
        query = module.q_proj(tail).view(*tail.shape[:-1], -1, module.head_dim).transpose(1, 2)
        cos, sin = positions
        query, _ = _rotary(self.model.config.model_type)(
            query, query, cos[..., -count:, :], sin[..., -count:, :])
        self._anchor_queries[index] = query.detach()  # (batch, query heads, count, dim)

    # ---- attention ---------------------------------------------------------
    def _prefill(self, module, index, query, key, value, mask, scaling, kwargs):
        output = sdpa_attention_forward(module, query, key, value, mask, dropout=0,
                                        scaling=scaling, **kwargs)
        prompt = query.shape[2]
        state = _LayerState(prompt, prompt)
        if index >= self.config.full_attention_layers:
            layers = getattr(self._cache, "layers", None) or []
            fused = getattr(layers[index], "fused_summary", None) if index < len(layers) else None
            if fused is not None:  # summarised while the prompt was written to the cache
                layers[index].fused_summary = None
                state.summary = fused
            else:
                state.summary = build_summary(key[0, :, :prompt], value[0, :, :prompt],
                                              self.config)
            count = min(self.config.anchor_tokens, prompt)
            anchors = self._anchor_queries.pop(index, None)
            if count and anchors is None:
                raise RuntimeError(f"missing prompt anchor queries in layer {index}")
            if count:
                heads, dim = key.shape[1], query.shape[-1]
                groups = query.shape[1] // heads
                # (query heads, anchors, dim) -> (anchors, kv heads, group, 1, dim)
                grouped = anchors[0, :, -count:].transpose(0, 1).reshape(
                    count, heads, groups, 1, dim)
                state.anchor_mask = select_blocks_union(grouped, state.summary, self.config,
                                                        workspace=state.workspace)
        self._layers[index] = state
        return output

    def _dense_decode(self, module, query, key, value, mask, scaling, kwargs, visible_length):
        # The reference's explicit-mask SDPA (``transformers.py:510-520``),
        # including KV-head repetition: the mask-free GQA path can round
        # differently in bf16.
        if mask is None:
            mask = query.new_full((1, 1, 1, key.shape[2]), torch.finfo(query.dtype).min)
            mask[..., :visible_length] = 0
        elif mask.dtype == torch.bool:
            mask = query.new_zeros(mask.shape).masked_fill(~mask, torch.finfo(query.dtype).min)
        return sdpa_attention_forward(module, query, key, value, mask, dropout=0, scaling=scaling,
                                      **kwargs)

    def _dense_graph_decode(self, module, query, key, value, scaling, kwargs, state):
        """Dense layer under CUDA graphs.

        One sequence: ``dense_attention`` over the prompt's pages of the cache
        and the suffix up to the device length (the refinement kernel with no
        selector: no mask over the fixed capacity, no KV-head repetition).
        A left-padded batch: SDPA over the whole fixed-capacity cache with a
        device-side mask that also hides each row's padding.
        """
        if query.shape[0] == 1 and state.pad_rows is None:
            heads, dim = key.shape[1], query.shape[-1]
            groups = query.shape[1] // heads
            if state.pages is None:
                state.pages = page_view(key[0], value[0], state.prompt_length,
                                        self.config.block_size)
            out = dense_attention(query[0].reshape(heads, groups, 1, dim), state.pages,
                                  key[0, :, state.prompt_length:],
                                  value[0, :, state.prompt_length:], workspace=state.workspace,
                                  suffix_length=self._graph_suffix_length)
            return out.reshape(query.shape[1], 1, dim).transpose(0, 1).unsqueeze(0), None
        visible = state.prompt_length + self._graph_suffix_length
        columns = torch.arange(key.shape[2], device=key.device)
        live = (columns < visible).view(1, 1, 1, -1)
        if state.pad_rows is not None:  # a left-padded batch: skip each row's padding
            live = live & (columns.view(1, 1, 1, -1) >= state.pad_rows)
        mask = query.new_zeros((live.shape[0], 1, 1, key.shape[2])).masked_fill(
            ~live, torch.finfo(query.dtype).min)
        return sdpa_attention_forward(module, query, key, value, mask, dropout=0, scaling=scaling,
                                      **kwargs)

    def _attention(self, module, query, key, value, mask, scaling, kwargs):
        if query.shape[0] != 1:
            return self._attention_batch(module, query, key, value, mask, scaling, kwargs)
        index = self._module_indices[id(module)]
        state = self._layers.get(index)
        if state is None:
            return self._prefill(module, index, query, key, value, mask, scaling, kwargs)
        if query.shape[2] != 1:
            raise ValueError("RefineKV supports one full prefill followed by single-token decode")
        heads, dim = key.shape[1], query.shape[-1]
        groups = query.shape[1] // heads
        if self._graph_mode:
            if state.summary is None:
                return self._dense_graph_decode(module, query, key, value, scaling, kwargs, state)
            result = sparse_attention(
                query[0].reshape(heads, groups, 1, dim), state.summary,
                key[0, :, state.prompt_length:], value[0, :, state.prompt_length:], self.config,
                anchor_mask=state.anchor_mask, workspace=state.workspace,
                suffix_length=self._graph_suffix_length)
            return result.output.reshape(query.shape[1], 1, dim).transpose(0, 1).unsqueeze(0), None
        state.visible_length += 1
        if key.shape[2] < state.visible_length:
            raise ValueError("the KV cache no longer contains the full visible prefix")
        if state.summary is None:
            if self.config.collect_stats:
                dense = query.shape[1] * state.visible_length
                self._record(dense, dense)
            return self._dense_decode(module, query, key, value, mask, scaling, kwargs,
                                      state.visible_length)
        result = sparse_attention(
            query[0].reshape(heads, groups, 1, dim), state.summary,
            key[0, :, state.prompt_length:state.visible_length],
            value[0, :, state.prompt_length:state.visible_length], self.config,
            anchor_mask=state.anchor_mask, workspace=state.workspace,
            return_selected=self.config.collect_stats)
        if self.config.collect_stats:
            accessed = decode_access_counts(result.selected, state.summary.counts, groups,
                                            query.shape[1],
                                            state.visible_length - state.prompt_length)
            self._record(accessed, query.shape[1] * state.visible_length)
        return result.output.reshape(query.shape[1], 1, dim).transpose(0, 1).unsqueeze(0), None

    # ---- batches (beyond the reference) ------------------------------------
    def _attention_batch(self, module, query, key, value, mask, scaling, kwargs):
        """A left-padded batch: prompts stacked on the KV-head axis of one summary.

        Row i's prompt is its last ``prompt - pads[i]`` positions; the
        generated tokens follow the padded prompt in every row, so all rows
        decode in lockstep with one suffix length, the layout of
        :func:`~refinekv_b200.build_summary_batch`.
        """
        index = self._module_indices[id(module)]
        state = self._layers.get(index)
        rows, heads, dim = query.shape[0], key.shape[1], query.shape[-1]
        groups = query.shape[1] // heads
        if state is None:
            return self._prefill_batch(module, index, query, key, value, mask, scaling, kwargs)
        if query.shape[2] != 1:
            raise ValueError("RefineKV supports one full prefill followed by single-token decode")
        if self._graph_mode:
            if state.summary is None:
                return self._dense_graph_decode(module, query, key, value, scaling, kwargs, state)
            result = sparse_attention(
                query.reshape(rows * heads, groups, 1, dim), state.summary,
                key[:, :, state.prompt_length:].flatten(0, 1),
                value[:, :, state.prompt_length:].flatten(0, 1), self.config,
                anchor_mask=state.anchor_mask, workspace=state.workspace,
                suffix_length=self._graph_suffix_length)
            return result.output.reshape(rows, query.shape[1], 1, dim).transpose(1, 2), None
        state.visible_length += 1
        if key.shape[2] < state.visible_length:
            raise ValueError("the KV cache no longer contains the full visible prefix")
        dense = query.shape[1] * sum(state.visible_length - pad for pad in state.pads)
        if state.summary is None:
            if self.config.collect_stats:
                self._record(dense, dense)
            return self._dense_decode(module, query, key, value, mask, scaling, kwargs,
                                      state.visible_length)
        result = sparse_attention(
            query.reshape(rows * heads, groups, 1, dim), state.summary,
            key[:, :, state.prompt_length:state.visible_length].flatten(0, 1),
            value[:, :, state.prompt_length:state.visible_length].flatten(0, 1), self.config,
            anchor_mask=state.anchor_mask, workspace=state.workspace,
            return_selected=self.config.collect_stats)
        if self.config.collect_stats:
            counts = state.summary.counts.repeat_interleave(heads, 0)  # per row, 0 past a prompt
            accessed = decode_access_counts(result.selected, counts, groups,
                                            query.shape[1] * rows,
                                            state.visible_length - state.prompt_length)
            self._record(accessed, dense)
        return result.output.reshape(rows, query.shape[1], 1, dim).transpose(1, 2), None

    def _prefill_batch(self, module, index, query, key, value, mask, scaling, kwargs):
        output = sdpa_attention_forward(module, query, key, value, mask, dropout=0,
                                        scaling=scaling, **kwargs)
        rows, prompt = query.shape[0], query.shape[2]
        pads = self._pads if self._pads is not None else [0] * rows
        if len(pads) != rows:
            raise RuntimeError("the batch's padding does not match its rows")
        state = _LayerState(prompt, prompt, pads=list(pads))
        if any(pads):
            state.pad_rows = torch.tensor(pads, device=key.device).view(-1, 1, 1, 1)
        if index >= self.config.full_attention_layers:
            state.summary = build_summary_batch(
                [key[i, :, pad:prompt] for i, pad in enumerate(pads)],
                [value[i, :, pad:prompt] for i, pad in enumerate(pads)], self.config)
            count = min(self.config.anchor_tokens, prompt)
            anchors = self._anchor_queries.pop(index, None)
            if count and anchors is None:
                raise RuntimeError(f"missing prompt anchor queries in layer {index}")
            if count:
                heads, dim = key.shape[1], query.shape[-1]
                groups = query.shape[1] // heads
                tail = anchors[:, :, -count:].clone()  # (rows, query heads, count, dim)
                for i, pad in enumerate(pads):
                    real = min(count, prompt - pad)
                    if real < count:  # a short prompt: repeat a real anchor, the union is unchanged
                        tail[i, :, :count - real] = tail[i, :, count - 1:count]
                grouped = tail.permute(2, 0, 1, 3).reshape(count, rows * heads, groups, 1, dim)
                state.anchor_mask = select_blocks_union(grouped, state.summary, self.config,
                                                        workspace=state.workspace)
        self._layers[index] = state
        return output

"""Prompt block summaries computed by the CUDA summarizer.

Mirrors ``src/refinekv/summary.py`` of the reference: the same ``BlockSummary``
fields, shapes and dtypes, and the same ``build_summary`` signature and
validation errors.  The computation is one call of ``rkv_summarize``.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import _native
from .config import RefineKVConfig

#: Head dims of the CUDA path: multiples of 32 up to 256, as the reference's GPU backend
#: (``attention.py:29-39``).
SUPPORTED_HEAD_DIMS = tuple(range(32, 257, 32))


@dataclass
class BlockSummary:
    """Per-KV-head page summaries; the original K/V stay available for refinement.

    Same fields as the reference ``BlockSummary`` (``summary.py:10-32``):
    ``keys``/``values`` are (kv_heads, pages, block_size, head_dim) page views
    that alias the cache when the prompt is page-aligned and page-contiguous
    (head stride free) and are a zero-padded copy otherwise; ``counts`` is
    int64 (pages,); ``key_mean``, ``value_mean`` and ``ellipsoid`` are bf16
    (kv_heads, pages, head_dim); ``value_norm`` is FP32 (kv_heads, pages) and
    ``max_value_norm`` FP32 (kv_heads,).  A summary belongs to one immutable
    prompt prefix.

    A batch of prompts (``build_summary_batch``; beyond the reference, which
    decodes one sequence) stacks them on the head axis, sequence-major
    (``sequences * kv_heads`` rows), padded to the longest prompt's page
    count: ``counts`` is then (sequences, pages) with 0 past each prompt,
    ``prompt_lengths`` the (sequences,) int64 device lengths and
    ``prompt_length`` their maximum.
    """

    keys: torch.Tensor
    values: torch.Tensor
    counts: torch.Tensor
    key_mean: torch.Tensor
    value_mean: torch.Tensor
    ellipsoid: torch.Tensor
    value_norm: torch.Tensor
    max_value_norm: torch.Tensor
    prompt_length: int
    block_size: int
    sequences: int = 1
    prompt_lengths: torch.Tensor | None = None
    page_table: torch.Tensor | None = None
    _abi: object = field(default=None, repr=False, compare=False)

    def __setattr__(self, name, value):
        # The C view holds raw pointers and sizes of the fields: any change to
        # a field drops it, and the next abi() call rebuilds it.
        if name != "_abi":
            object.__setattr__(self, "_abi", None)
        object.__setattr__(self, name, value)

    @property
    def num_blocks(self) -> int:
        return self.counts.shape[-1]

    @property
    def num_heads(self) -> int:
        """KV-head rows of the decode (sequences x KV heads for a paged batch)."""
        if self.page_table is not None:
            return self.sequences * self.keys.shape[0]
        return self.keys.shape[0]

    def abi(self) -> _native.Summary:
        """The ``rkv_summary`` view handed to the C ABI (built once per set of fields).

        Reassigning any field drops the cached view.  Changing a tensor in
        place (``summary.counts.copy_(...)``) keeps it valid, since the view
        holds the same storage; swapping the storage (``.set_()``) does not.
        """
        if self._abi is None:
            self._abi = _native.Summary(
                key_pages=self.keys.data_ptr(),
                value_pages=self.values.data_ptr(),
                key_page_head_stride=self.keys.stride(0),
                value_page_head_stride=self.values.stride(0),
                counts=self.counts.data_ptr(),
                key_mean=self.key_mean.data_ptr(),
                value_mean=self.value_mean.data_ptr(),
                ellipsoid=self.ellipsoid.data_ptr(),
                value_norm=self.value_norm.data_ptr(),
                max_value_norm=self.max_value_norm.data_ptr(),
                heads=self.num_heads,
                blocks=self.num_blocks,
                block_size=self.block_size,
                head_dim=self.keys.shape[-1],
                prompt_length=self.prompt_length,
                sequences=self.sequences,
                prompt_lengths=(self.prompt_lengths.data_ptr()
                                if self.prompt_lengths is not None else None),
            )
            if self.page_table is not None:
                a = self._abi
                a.page_table = self.page_table.data_ptr()
                a.page_table_stride = self.page_table.stride(0)
                a.pool_pages = self.keys.shape[1]
                a.key_page_stride, a.value_page_stride = self.keys.stride(1), self.values.stride(1)
                a.key_token_stride = self.keys.stride(2)
                a.value_token_stride = self.values.stride(2)
        return self._abi


@dataclass(frozen=True)
class PageView:
    """A prompt's K/V pages with no summaries, for dense decode (``dense_attention``).

    ``keys``/``values``: (kv_heads, pages, block_size, head_dim) bf16 page
    views (``page_view`` makes them from a KV cache without copying); rows of
    the last page past ``prompt_length`` are never read as prompt rows.
    """

    keys: torch.Tensor
    values: torch.Tensor
    prompt_length: int
    block_size: int

    @property
    def num_blocks(self) -> int:
        return self.keys.shape[1]

    @property
    def num_heads(self) -> int:
        return self.keys.shape[0]

    def abi(self) -> _native.Summary:
        return _native.Summary(
            key_pages=self.keys.data_ptr(), value_pages=self.values.data_ptr(),
            key_page_head_stride=self.keys.stride(0), value_page_head_stride=self.values.stride(0),
            heads=self.num_heads, blocks=self.num_blocks, block_size=self.block_size,
            head_dim=self.keys.shape[-1], prompt_length=self.prompt_length, sequences=1)


def page_view(key_cache: torch.Tensor, value_cache: torch.Tensor, prompt_length: int,
              block_size: int = 32) -> PageView:
    """Pages of the first ``prompt_length`` rows of a (kv_heads, capacity, head_dim) cache.

    No copy: the cache's rows must be contiguous and its capacity must hold
    the prompt rounded up to whole pages (the rows after the prompt may hold
    anything, e.g. the generated tokens).
    """
    heads, capacity, dim = key_cache.shape
    blocks = -(-int(prompt_length) // block_size)
    for cache in (key_cache, value_cache):
        if cache.shape != key_cache.shape or cache.dtype != torch.bfloat16:
            raise ValueError("caches must be bf16 with the same (kv_heads, capacity, head_dim)")
        if cache.stride(2) != 1 or cache.stride(1) != dim:
            raise ValueError("cache rows must be contiguous")
        if cache.data_ptr() % 16 or (cache.stride(0) * 2) % 16:
            raise ValueError("cache heads must start on 16-byte boundaries")
    if prompt_length <= 0 or blocks * block_size > capacity:
        raise ValueError("cache capacity must hold the prompt rounded up to whole pages")
    pages = lambda cache: cache.as_strided((heads, blocks, block_size, dim),  # noqa: E731
                                           (cache.stride(0), block_size * dim, dim, 1))
    return PageView(pages(key_cache), pages(value_cache), int(prompt_length), block_size)


def require_cuda_tensor(tensor: torch.Tensor, what: str) -> None:
    if not tensor.is_cuda:
        raise RuntimeError(
            f"{what} must be a CUDA tensor: refinekv_b200 runs on B200 GPUs only "
            "and has no CPU implementation")


def _page_alias(tensor: torch.Tensor, block: int):
    """(heads, tokens, dim) -> page view without copying, or None if a copy is needed."""
    heads, tokens, dim = tensor.shape
    if tokens % block or tensor.stride(2) != 1 or tensor.stride(1) != dim:
        return None
    if tensor.data_ptr() % 16 or (tensor.stride(0) * 2) % 16:
        return None
    return tensor.as_strided((heads, tokens // block, block, dim),
                             (tensor.stride(0), block * dim, dim, 1))


def _checked_prompt(keys: torch.Tensor, values: torch.Tensor):
    """The reference's argument checks (``summary.py:46-60``) plus the CUDA path's own."""
    if keys.ndim != 3 or keys.shape != values.shape or min(keys.shape) <= 0:
        raise ValueError(
            "keys and values must have the same nonempty (kv_heads, tokens, dim) shape")
    if keys.device != values.device or keys.dtype != values.dtype:
        raise ValueError("keys and values must have the same device and dtype")
    if not keys.is_floating_point():
        raise TypeError("keys and values must be floating point")
    require_cuda_tensor(keys, "keys")
    if keys.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("the CUDA summarizer requires BF16 or FP32 keys and values")
    if keys.shape[-1] not in SUPPORTED_HEAD_DIMS:
        raise ValueError(f"head_dim must be one of {SUPPORTED_HEAD_DIMS}")
    keys, values = keys.detach(), values.detach()
    w = keys.element_size()
    if keys.stride(2) != 1 or keys.data_ptr() % 16 or (keys.stride(1) * w) % 16 or (
            keys.stride(0) * w) % 16:
        keys = keys.contiguous()
    if values.stride(2) != 1 or values.data_ptr() % 16 or (values.stride(1) * w) % 16 or (
            values.stride(0) * w) % 16:
        values = values.contiguous()
    return keys, values


@torch.no_grad()
def build_summary(keys: torch.Tensor, values: torch.Tensor,
                  config: RefineKVConfig | None = None) -> BlockSummary:
    """Build BF16 block summaries in one pass over the prompt K/V.

    ``keys``/``values``: (kv_heads, tokens, head_dim) bf16 or fp32 CUDA
    tensors (any head/token strides, innermost stride 1).  Raises the
    reference's ``ValueError``/``TypeError`` for bad shapes, devices and
    dtypes (``summary.py:46-60``), ``TypeError`` for caches other than bf16
    and fp32, ``ValueError`` for unsupported head dimensions and
    ``RuntimeError`` for CPU tensors.

    An fp32 cache is summarised from its fp32 values, like the reference's
    ``build_summary``; its page views (``keys``/``values`` of the result)
    are a bf16 copy, not fp32 views of the cache as in the reference:
    the reference's attention rounds the pages to bf16 before using them
    (``reference.py:57``, ``:63-66``), so the decode reads the same values.
    """
    config = config or RefineKVConfig()
    keys, values = _checked_prompt(keys, values)
    heads, tokens, dim = keys.shape
    block = config.block_size
    blocks = -(-tokens // block)
    dev = keys.device
    f32 = keys.dtype == torch.float32
    key_pages = value_pages = None
    if not f32:
        key_pages, value_pages = _page_alias(keys, block), _page_alias(values, block)
    copy_pages = key_pages is None or value_pages is None
    if copy_pages:
        key_pages = torch.empty(heads, blocks, block, dim, device=dev, dtype=torch.bfloat16)
        value_pages = torch.empty_like(key_pages)
    key_mean = torch.empty(heads, blocks, dim, device=dev, dtype=torch.bfloat16)
    value_mean = torch.empty_like(key_mean)
    ellipsoid = torch.empty_like(key_mean)
    value_norm = torch.empty(heads, blocks, device=dev, dtype=torch.float32)
    max_value_norm = torch.empty(heads, device=dev, dtype=torch.float32)
    counts = torch.empty(blocks, device=dev, dtype=torch.int64)
    lib = _native.load()
    summarize = lib.rkv_summarize_f32 if f32 else lib.rkv_summarize
    with torch.cuda.device(dev):
        _native.check(summarize(
            keys.data_ptr(), values.data_ptr(), heads, tokens, dim,
            keys.stride(0), keys.stride(1), values.stride(0), values.stride(1), block,
            key_pages.data_ptr() if copy_pages else None,
            value_pages.data_ptr() if copy_pages else None,
            key_mean.data_ptr(), value_mean.data_ptr(), ellipsoid.data_ptr(),
            value_norm.data_ptr(), max_value_norm.data_ptr(), counts.data_ptr(),
            torch.cuda.current_stream(dev).cuda_stream))
    return BlockSummary(key_pages, value_pages, counts, key_mean, value_mean, ellipsoid,
                        value_norm, max_value_norm, tokens, block)


def _stacked(prompts: list[torch.Tensor]) -> torch.Tensor:
    """(sequences * heads, tokens, dim): a view when the prompts are consecutive
    equal slices of one buffer (a batched cache), else a stacked copy."""
    first = prompts[0]
    step = first.shape[0] * first.stride(0) * first.element_size()
    if all(p.stride() == first.stride() and p.data_ptr() == first.data_ptr() + i * step
           for i, p in enumerate(prompts)):
        return first.as_strided((len(prompts) * first.shape[0],) + tuple(first.shape[1:]),
                                first.stride())
    return torch.cat(prompts)


@torch.no_grad()
def build_summary_batch(keys: list[torch.Tensor], values: list[torch.Tensor],
                        config: RefineKVConfig | None = None) -> BlockSummary:
    """Summaries of several prompts that decode together, in one batched summary.

    ``keys[i]``/``values[i]``: (kv_heads, tokens_i, head_dim) bf16 CUDA
    tensors, the same heads, dim and device for every prompt.  The result
    stacks the prompts on the head axis (row ``i * kv_heads + h``) padded to
    the longest prompt's page count; every page, mean, ellipsoid and norm
    past a prompt is zero and its count is 0, so the decode kernels neither
    select, represent nor read it.  Each prompt's rows hold exactly what
    ``build_summary`` computes for it alone (the same kernel over the same
    pages).  No reference counterpart: the reference is batch 1
    (``transformers.py:448-449``).
    """
    config = config or RefineKVConfig()
    if len(keys) == 0 or len(keys) != len(values):
        raise ValueError("need the same nonzero number of key and value tensors")
    checked = [_checked_prompt(k, v) for k, v in zip(keys, values)]
    heads, _, dim = checked[0][0].shape
    dev, dtype = checked[0][0].device, checked[0][0].dtype
    for k, _ in checked:
        if k.shape[0] != heads or k.shape[2] != dim or k.device != dev:
            raise ValueError("every prompt needs the same kv_heads, head_dim and device")
    block = config.block_size
    lengths = [k.shape[1] for k, _ in checked]
    seqs, longest = len(checked), max(lengths)
    if len(set(lengths)) == 1:
        # Equal prompts: the batch is the summary of the stacked heads (one
        # launch; pages alias a batched cache the prompts are slices of).
        stacked_k = _stacked([k for k, _ in checked])
        stacked_v = _stacked([v for _, v in checked])
        one = build_summary(stacked_k, stacked_v, config)
        one.counts = one.counts.expand(seqs, -1).contiguous()
        one.sequences = seqs
        one.prompt_lengths = torch.tensor(lengths, device=dev, dtype=torch.int64)
        return one
    blocks = -(-longest // block)
    rows = seqs * heads
    key_pages = torch.zeros(rows, blocks, block, dim, device=dev, dtype=torch.bfloat16)
    value_pages = torch.zeros_like(key_pages)
    key_mean = torch.zeros(rows, blocks, dim, device=dev, dtype=torch.bfloat16)
    value_mean = torch.zeros_like(key_mean)
    ellipsoid = torch.zeros_like(key_mean)
    value_norm = torch.zeros(rows, blocks, device=dev, dtype=torch.float32)
    max_value_norm = torch.zeros(rows, device=dev, dtype=torch.float32)
    counts = torch.zeros(seqs, blocks, device=dev, dtype=torch.int64)
    lib = _native.load()
    summarize = lib.rkv_summarize_f32 if dtype == torch.float32 else lib.rkv_summarize
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        for i, (k, v) in enumerate(checked):
            tokens = k.shape[1]
            # A prompt of the full page count writes all its heads in one call;
            # a shorter one head by head (its rows are `blocks` pages apart).
            groups = [range(heads)] if -(-tokens // block) == blocks else [[h] for h in range(heads)]
            for hs in groups:
                h0, n = hs[0], len(hs)
                r0 = i * heads + h0
                _native.check(summarize(
                    k[h0].data_ptr(), v[h0].data_ptr(), n, tokens, dim,
                    k.stride(0), k.stride(1), v.stride(0), v.stride(1), block,
                    key_pages[r0].data_ptr(), value_pages[r0].data_ptr(),
                    key_mean[r0].data_ptr(), value_mean[r0].data_ptr(), ellipsoid[r0].data_ptr(),
                    value_norm[r0].data_ptr(), max_value_norm[r0:].data_ptr(),
                    counts[i].data_ptr(), stream))
    prompt_lengths = torch.tensor(lengths, device=dev, dtype=torch.int64)
    return BlockSummary(key_pages, value_pages, counts, key_mean, value_mean, ellipsoid,
                        value_norm, max_value_norm, longest, block, sequences=seqs,
                        prompt_lengths=prompt_lengths)


def attach_page_pool(summary: BlockSummary, key_pool: torch.Tensor, value_pool: torch.Tensor,
                     page_table: torch.Tensor, layout: str = "HND") -> BlockSummary:
    """The summary decoding from a vLLM-style K/V page pool instead of its own pages.

    ``key_pool``/``value_pool``: bf16 ``(pages, kv_heads, block, dim)``
    (``layout="HND"``) or ``(pages, block, kv_heads, dim)`` (``"NHD"``) on the
    summary's device; ``page_table``: int32 ``(sequences, >= blocks)`` with the
    physical page of each logical block of each sequence (a 1-D table for one
    sequence).  The pool must hold, at those pages, the same K/V rows the
    summary was built from (the prompt's pages, rows past a prompt's end
    zero); the summary's means, ellipsoid, norms and counts are used as they
    are.  No copy is made.  No reference counterpart (the reference keeps one
    contiguous cache per layer).
    """
    if layout not in ("HND", "NHD"):
        raise ValueError("layout must be 'HND' or 'NHD'")
    if key_pool.shape != value_pool.shape or key_pool.ndim != 4:
        raise ValueError("key and value pools must have the same 4-D shape")
    if key_pool.dtype != torch.bfloat16 or value_pool.dtype != torch.bfloat16:
        raise TypeError("page pools must be bf16")
    if key_pool.device != summary.key_mean.device or value_pool.device != key_pool.device:
        raise ValueError("page pools must be on the summary's device")
    keys = key_pool.permute(1, 0, 2, 3) if layout == "HND" else key_pool.permute(2, 0, 1, 3)
    values = value_pool.permute(1, 0, 2, 3) if layout == "HND" else value_pool.permute(2, 0, 1, 3)
    heads = summary.num_heads // summary.sequences
    if (keys.shape[0], keys.shape[2], keys.shape[3]) != (heads, summary.block_size,
                                                         summary.key_mean.shape[-1]):
        raise ValueError("pool pages must be (kv_heads, block_size, head_dim) per page")
    if keys.stride(3) != 1 or values.stride(3) != 1:
        raise ValueError("pool rows must be contiguous in head_dim")
    table = page_table.reshape(1, -1) if page_table.ndim == 1 else page_table
    if (table.dtype != torch.int32 or table.device != key_pool.device
            or table.shape[0] != summary.sequences or table.shape[1] < summary.num_blocks
            or table.stride(1) != 1):
        raise ValueError("page_table must be int32 (sequences, >= blocks) on the pool's device")
    return BlockSummary(keys, values, summary.counts, summary.key_mean, summary.value_mean,
                        summary.ellipsoid, summary.value_norm, summary.max_value_norm,
                        summary.prompt_length, summary.block_size, sequences=summary.sequences,
                        prompt_lengths=summary.prompt_lengths, page_table=table)


@torch.no_grad()
def build_summary_into(keys: torch.Tensor, values: torch.Tensor, key_cache: torch.Tensor,
                       value_cache: torch.Tensor,
                       config: RefineKVConfig | None = None) -> BlockSummary:
    """Write a prompt into its KV cache and summarise it in the same pass.

    ``keys``/``values``: the prompt's (kv_heads, tokens, head_dim) bf16 K/V
    (the attention layer's fresh projections); ``key_cache``/``value_cache``:
    the (kv_heads, capacity, head_dim) bf16 cache of the same device, rows
    contiguous, with capacity at least the prompt rounded up to whole
    pages.  Rows [0, tokens) of the caches receive the prompt, the rest of
    its last page zeros, and the returned summary's page views alias the
    caches.  The same summaries as ``build_summary(keys, values)``; the
    prompt is read once instead of once for the cache write and once more
    for the summary (the reference's prefill, ``transformers.py:529-536``).

    The zeroed rows after the prompt are ordinary cache rows: a decoder that
    appends generated tokens to the same cache writes them there, so the
    summary's last page may later hold those tokens past the prompt.  The
    decode kernels take each page's valid rows from ``counts`` and never
    read those rows as prompt rows; do not rely on them staying zero.
    """
    config = config or RefineKVConfig()
    keys, values = _checked_prompt(keys, values)
    if keys.dtype != torch.bfloat16:
        raise TypeError("build_summary_into writes a bf16 cache from bf16 keys and values")
    heads, tokens, dim = keys.shape
    block = config.block_size
    blocks = -(-tokens // block)
    for cache in (key_cache, value_cache):
        if (cache.ndim != 3 or cache.shape[0] != heads or cache.shape[2] != dim
                or cache.dtype != torch.bfloat16 or cache.device != keys.device):
            raise ValueError("caches must be bf16 (kv_heads, capacity, head_dim) on the keys' device")
        if cache.shape[1] < blocks * block:
            raise ValueError("cache capacity must hold the prompt rounded up to whole pages")
        if cache.stride(2) != 1 or cache.stride(1) != dim:
            raise ValueError("cache rows must be contiguous")
    dev = keys.device
    key_mean = torch.empty(heads, blocks, dim, device=dev, dtype=torch.bfloat16)
    value_mean = torch.empty_like(key_mean)
    ellipsoid = torch.empty_like(key_mean)
    value_norm = torch.empty(heads, blocks, device=dev, dtype=torch.float32)
    max_value_norm = torch.empty(heads, device=dev, dtype=torch.float32)
    counts = torch.empty(blocks, device=dev, dtype=torch.int64)
    lib = _native.load()
    with torch.cuda.device(dev):
        _native.check(lib.rkv_summarize_into(
            keys.data_ptr(), values.data_ptr(), heads, tokens, dim,
            keys.stride(0), keys.stride(1), values.stride(0), values.stride(1), block,
            key_cache.data_ptr(), key_cache.stride(0), value_cache.data_ptr(),
            value_cache.stride(0), key_mean.data_ptr(), value_mean.data_ptr(),
            ellipsoid.data_ptr(), value_norm.data_ptr(), max_value_norm.data_ptr(),
            counts.data_ptr(), torch.cuda.current_stream(dev).cuda_stream))
    pages = lambda cache: cache.as_strided((heads, blocks, block, dim),  # noqa: E731
                                           (cache.stride(0), block * dim, dim, 1))
    return BlockSummary(pages(key_cache), pages(value_cache), counts, key_mean, value_mean,
                        ellipsoid, value_norm, max_value_norm, tokens, block)

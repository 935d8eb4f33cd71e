"""RefineKV decode hot path on B200 (sm_100a): summarizer, selector, split decode attention.

Public names mirror the reference package ``refinekv`` v0.1.2
(``src/refinekv/__init__.py``): ``RefineKVConfig``, ``BlockSummary``,
``build_summary``, ``select_blocks``, ``sparse_attention``,
``AttentionResult``, and the Transformers adapter ``RefineKV`` /
``make_visible_static_cache`` (imported lazily, like the reference).
Beyond the reference: ``build_summary_batch`` (several prompts decoding in
lockstep, stacked on the head axis), ``build_summary_into`` (the prefill's
cache write and the summary in one pass), ``attach_page_pool`` (decode from a
vLLM-style K/V page pool through a page table), ``page_view`` and
``dense_attention`` (dense decode of the full-attention layers on the same
kernel) and ``refinekv_b200.parallel`` (KV-head sharding and sequence split
over GPUs).

All compute runs in the CUDA library ``librefinekv_b200.so`` built from
``csrc/``; it is loaded on first use and a missing or unloadable library is
an error, never a silent fallback.
"""

from .config import RefineKVConfig

__version__ = "0.1.2+b200"
__all__ = [
    "AttentionResult",
    "BlockSummary",
    "RefineKVConfig",
    "build_summary",
    "build_summary_batch",
    "build_summary_into",
    "attach_page_pool",
    "page_view",
    "PageView",
    "dense_attention",
    "select_blocks",
    "sparse_attention",
    "RefineKV",
    "make_visible_static_cache",
]


def __getattr__(name):
    if name in ("AttentionResult", "select_blocks", "sparse_attention", "dense_attention"):
        from . import attention

        return getattr(attention, name)
    if name in ("BlockSummary", "build_summary", "build_summary_batch", "build_summary_into",
                "attach_page_pool", "page_view", "PageView"):
        from . import summary

        return getattr(summary, name)
    if name in ("RefineKV", "make_visible_static_cache"):
        from .integrations import transformers as adapter

        return getattr(adapter, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")

"""Algorithm settings, field-for-field compatible with the reference ``RefineKVConfig``."""

from dataclasses import dataclass
import math

#: Accepted ``backend`` values.  ``"auto"``, ``"cuda"`` and ``"triton"`` all
#: select this package's CUDA kernels; ``"torch"`` is accepted so existing
#: configurations still construct, but the tensor API refuses it at call time
#: because this package has no CPU implementation.
BACKENDS = ("auto", "cuda", "triton", "torch")
GQA_REDUCTIONS = ("mean", "max", "any")


@dataclass(frozen=True)
class RefineKVConfig:
    """Settings for diagonal-ellipsoid selection and sparse decode.

    Mirrors ``src/refinekv/config.py:7-38`` of the reference: same fields,
    defaults and validation errors (``ValueError``).

    ``eps`` is the block-risk threshold (not a token budget).
    ``gqa_reduction`` combines the risks of the query rows that share a KV
    head: ``any`` expands a block if any row exceeds ``eps``, ``max`` compares
    the largest risk, ``mean`` the average.  ``anchor_tokens`` prompt queries
    are selected once after prefill and their masks stay expanded.
    ``full_attention_layers`` keeps the first layers dense.
    ``summary_chunk_blocks`` only bounds temporaries in the reference's
    chunked summary build; the CUDA summarizer streams one page at a time and
    accepts it for compatibility.
    """

    block_size: int = 32
    eps: float = 0.01
    gqa_reduction: str = "any"
    anchor_tokens: int = 0
    full_attention_layers: int = 0
    backend: str = "auto"
    summary_chunk_blocks: int = 512
    collect_stats: bool = False

    def __post_init__(self):
        if self.block_size not in (16, 32, 64):
            raise ValueError("block_size must be 16, 32, or 64")
        if not isinstance(self.eps, (int, float)) or not math.isfinite(self.eps) or self.eps < 0:
            raise ValueError("eps must be finite and nonnegative")
        if self.gqa_reduction not in GQA_REDUCTIONS:
            raise ValueError("gqa_reduction must be 'mean', 'max', or 'any'")
        if self.backend not in BACKENDS:
            raise ValueError("backend must be 'auto', 'cuda', 'triton', or 'torch'")
        for name in ("anchor_tokens", "full_attention_layers"):
            value = getattr(self, name)
            if not isinstance(value, int) or isinstance(value, bool) or value < 0:
                raise ValueError(f"{name} must be a nonnegative integer")
        chunk = self.summary_chunk_blocks
        if not isinstance(chunk, int) or isinstance(chunk, bool) or chunk <= 0:
            raise ValueError("summary_chunk_blocks must be a positive integer")

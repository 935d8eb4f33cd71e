"""Single-token decode entry points over the CUDA selector and split attention.

Mirrors ``src/refinekv/attention.py`` of the reference: ``select_blocks`` and
``sparse_attention`` keep their signatures, argument meaning, validation
errors and workspace semantics (outputs backed by ``workspace`` are reused by
the next call).  The reference's backend dispatch (``_backend``) is replaced
by one CUDA path through ``rkv_select`` / ``rkv_decode``.
"""

from __future__ import annotations

from typing import NamedTuple

import torch

from . import _native
from .config import RefineKVConfig
from .summary import SUPPORTED_HEAD_DIMS, BlockSummary, PageView, require_cuda_tensor

MAX_GROUP = 16


class AttentionResult(NamedTuple):
    output: torch.Tensor
    selected: torch.Tensor | None


def _check_backend(query: torch.Tensor, config: RefineKVConfig) -> None:
    """Errors of the reference ``_backend`` (``attention.py:17-40``) for the CUDA-only path."""
    if config.backend == "torch":
        raise ValueError(
            "backend='torch' is the reference's CPU path; refinekv_b200 implements only the "
            "CUDA backend (use 'auto', 'cuda' or 'triton')")
    require_cuda_tensor(query, "query")
    if query.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("the CUDA backend requires BF16 or FP32 queries")
    dim, group = query.shape[-1], query.shape[1]
    if dim not in SUPPORTED_HEAD_DIMS or group > MAX_GROUP:
        raise ValueError(
            f"the CUDA backend requires head_dim in {SUPPORTED_HEAD_DIMS} and GQA group <= 16")
    if torch.cuda.get_device_capability(query.device)[0] != 10:
        raise RuntimeError("librefinekv_b200 is built for sm_100a (B200) only")


def _validate(query, summary, config, anchor_mask=None):
    """Shape/device checks of the reference ``_validate`` (``attention.py:43-59``)."""
    if query.ndim != 4 or query.shape[2] != 1 or min(query.shape) <= 0:
        raise ValueError("query must have shape (kv_heads, group_size, 1, head_dim)")
    if query.shape[0] != summary.num_heads or query.shape[-1] != summary.keys.shape[-1]:
        raise ValueError("query heads and dimension must match the summary")
    if query.device != summary.keys.device:
        raise ValueError("query and summary must be on the same device")
    if config.block_size != summary.block_size:
        raise ValueError("config.block_size must match the summary")
    if anchor_mask is not None:
        if anchor_mask.dtype != torch.bool or tuple(anchor_mask.shape) != (
                query.shape[0], summary.num_blocks):
            raise ValueError("anchor_mask must be boolean with shape (kv_heads, blocks)")
        if anchor_mask.device != query.device:
            raise ValueError("anchor_mask must be on the query device")


def _buffer(workspace, name, shape, device, dtype, zero=False):
    """Reuse a workspace tensor keyed by name/shape/dtype/device, like ``runtime.py:26-37``."""
    tensor = workspace.get(name) if workspace is not None else None
    if (tensor is None or tuple(tensor.shape) != tuple(shape) or tensor.device != device
            or tensor.dtype != dtype):
        tensor = (torch.zeros if zero else torch.empty)(shape, device=device, dtype=dtype)
        if workspace is not None:
            workspace[name] = tensor
    return tensor


def _scratch(workspace, name, nbytes, device):
    """Zero-filled device scratch of at least ``nbytes`` (the C ABI's workspace)."""
    if nbytes == 0:
        raise RuntimeError("librefinekv_b200 rejected the workspace geometry")
    tensor = workspace.get(name) if workspace is not None else None
    if tensor is None or tensor.device != device or tensor.numel() < nbytes:
        tensor = torch.zeros(nbytes, device=device, dtype=torch.uint8)
        if workspace is not None:
            workspace[name] = tensor
    return tensor


def device_status(workspace: dict) -> int:
    """Sticky device status word of the decode workspace (synchronises); 0 means healthy."""
    scratch = workspace.get("rkv_decode_scratch") if workspace else None
    if scratch is None:
        return 0
    return int(scratch[:4].view(torch.int32).item())


def _query_code(query):
    return _native.DTYPE_F32 if query.dtype == torch.float32 else _native.DTYPE_BF16


@torch.no_grad()
def select_blocks(query, summary: BlockSummary, config=None, *, workspace=None):
    """Return a boolean ``(kv_heads, blocks)`` mask for one query (owned tensor)."""
    config = config or RefineKVConfig(block_size=summary.block_size)
    _validate(query, summary, config)
    _check_backend(query, config)
    return select_blocks_union(query.unsqueeze(0), summary, config, workspace=workspace)


@torch.no_grad()
def select_blocks_union(queries, summary: BlockSummary, config=None, *, workspace=None):
    """OR of the masks of ``queries`` (anchors, kv_heads, group, 1, head_dim) in one launch pair.

    Equals OR-ing ``select_blocks`` over the anchors one by one, as the
    reference adapter does at prefill (``integrations/transformers.py:543-552``).
    """
    config = config or RefineKVConfig(block_size=summary.block_size)
    if queries.ndim != 5 or queries.shape[3] != 1:
        raise ValueError("queries must have shape (anchors, kv_heads, group_size, 1, head_dim)")
    _validate(queries[0], summary, config)
    _check_backend(queries[0], config)
    count, heads, group, _, dim = queries.shape
    dev = queries.device
    q = queries.reshape(count, heads, group, dim).contiguous()
    mask = torch.empty(heads, summary.num_blocks, device=dev, dtype=torch.uint8)
    lib = _native.load()
    with torch.cuda.device(dev):
        nbytes = lib.rkv_select_workspace_size(heads, group, summary.num_blocks, dim, count)
        scratch = _scratch(workspace, f"rkv_select_scratch_{count}", nbytes, dev)
        _native.check(lib.rkv_select(
            summary.abi(), q.data_ptr(), _query_code(q), count, group, config.eps,
            _native.GQA_CODES[config.gqa_reduction], mask.data_ptr(), 0, scratch.data_ptr(),
            scratch.numel(), torch.cuda.current_stream(dev).cuda_stream))
    return mask.view(torch.bool)


@torch.no_grad()
def sparse_attention(
    query: torch.Tensor,
    summary: BlockSummary,
    key_suffix: torch.Tensor,
    value_suffix: torch.Tensor,
    config: RefineKVConfig | None = None,
    *,
    anchor_mask: torch.Tensor | None = None,
    workspace: dict | None = None,
    return_selected: bool = False,
    suffix_length: torch.Tensor | None = None,
    _phases: int = _native.PHASE_ALL,
) -> AttentionResult:
    """Attend to representatives, selected prompt pages and the exact suffix.

    ``query`` is (kv_heads, group_size, 1, head_dim); suffix K/V are
    (kv_heads, suffix_tokens, head_dim) and must hold only visible tokens,
    or a fixed-capacity buffer whose valid prefix is the device int32 scalar
    ``suffix_length`` (CUDA-graph replay).  Outputs backed by ``workspace``
    are reused on the next call; clone them to keep them.  Same contract as
    the reference ``sparse_attention`` (``attention.py:76-134``).
    """
    config = config or RefineKVConfig(block_size=summary.block_size)
    _validate(query, summary, config, anchor_mask)
    expected = (query.shape[0], query.shape[-1])
    if key_suffix.ndim != 3 or key_suffix.shape != value_suffix.shape:
        raise ValueError("suffix K/V must have matching (kv_heads, tokens, head_dim) shapes")
    if (key_suffix.shape[0], key_suffix.shape[-1]) != expected:
        raise ValueError("suffix heads and dimension must match the query")
    if key_suffix.device != query.device or value_suffix.device != query.device:
        raise ValueError("suffix K/V must be on the query device")
    _check_backend(query, config)
    if suffix_length is not None:
        if (suffix_length.shape != () or suffix_length.device != query.device
                or suffix_length.dtype != torch.int32):
            raise ValueError("suffix_length must be a scalar int32 tensor on the query device")
    if key_suffix.shape[1] and (key_suffix.dtype not in (torch.bfloat16, torch.float32)
                                or value_suffix.dtype != key_suffix.dtype):
        raise TypeError("the CUDA backend requires BF16 or FP32 suffix K/V")
    if key_suffix.dtype == torch.float32 and key_suffix.shape[1]:
        # The reference rounds the suffix to bf16 before use (reference.py:63-66);
        # the kernels read bf16 rows, so an fp32 suffix is rounded once here,
        # into workspace buffers reused while the shape stays the same.
        key_suffix = _buffer(workspace, "suffix_k_bf16", key_suffix.shape, key_suffix.device,
                             torch.bfloat16).copy_(key_suffix)
        value_suffix = _buffer(workspace, "suffix_v_bf16", value_suffix.shape,
                               value_suffix.device, torch.bfloat16).copy_(value_suffix)

    heads, group, _, dim = query.shape
    dev = query.device
    q = query.reshape(heads, group, dim)
    if not q.is_contiguous():
        q = q.contiguous()
    if key_suffix.stride(-1) != 1:
        key_suffix = key_suffix.contiguous()
    if value_suffix.stride(-1) != 1:
        value_suffix = value_suffix.contiguous()
    capacity = key_suffix.shape[1]
    anchor = None
    if anchor_mask is not None:
        anchor = anchor_mask if anchor_mask.is_contiguous() else anchor_mask.contiguous()
    output = _buffer(workspace, "output", (heads, group, dim), dev, query.dtype)
    selected = _buffer(workspace, "selected", (heads, summary.num_blocks), dev, torch.uint8)
    lib = _native.load()
    with torch.cuda.device(dev):
        nbytes = lib.rkv_decode_workspace_size(heads, group, summary.num_blocks, dim,
                                               summary.block_size)
        scratch = _scratch(workspace, "rkv_decode_scratch", nbytes, dev)
        _native.check(lib.rkv_decode(
            summary.abi(), q.data_ptr(), _query_code(q), group,
            key_suffix.data_ptr() if capacity else None,
            value_suffix.data_ptr() if capacity else None, capacity,
            key_suffix.stride(0), key_suffix.stride(1),
            value_suffix.stride(0), value_suffix.stride(1),
            suffix_length.data_ptr() if suffix_length is not None else None, capacity,
            anchor.data_ptr() if anchor is not None else None,
            config.eps, _native.GQA_CODES[config.gqa_reduction], output.data_ptr(),
            selected.data_ptr(), scratch.data_ptr(), scratch.numel(), _phases,
            torch.cuda.current_stream(dev).cuda_stream))
    # The reference returns a fresh mask (``mask.bool()``, runtime.py:226); keep that ownership.
    return AttentionResult(output.view(heads, group, 1, dim),
                           selected.view(torch.bool).clone() if return_selected else None)


@torch.no_grad()
def dense_attention(query: torch.Tensor, pages: PageView, key_suffix: torch.Tensor,
                    value_suffix: torch.Tensor, *, workspace: dict | None = None,
                    suffix_length: torch.Tensor | None = None) -> torch.Tensor:
    """Exact attention of ``query`` over every prompt page and the visible suffix.

    The dense decode of the adapter's ``full_attention_layers`` (reference
    ``integrations/transformers.py:510-520``, SDPA over the visible cache)
    on the refinement kernel: no selector, no mask, graph-capturable with a
    device ``suffix_length`` over a fixed-capacity suffix buffer.  Shapes as
    ``sparse_attention``; returns the (kv_heads, group, 1, head_dim) output
    in the query dtype, backed by ``workspace``.
    """
    if query.ndim != 4 or query.shape[2] != 1 or min(query.shape) <= 0:
        raise ValueError("query must have shape (kv_heads, group_size, 1, head_dim)")
    if query.shape[0] != pages.num_heads or query.shape[-1] != pages.keys.shape[-1]:
        raise ValueError("query heads and dimension must match the pages")
    if key_suffix.ndim != 3 or key_suffix.shape != value_suffix.shape:
        raise ValueError("suffix K/V must have matching (kv_heads, tokens, head_dim) shapes")
    if (key_suffix.shape[0], key_suffix.shape[-1]) != (query.shape[0], query.shape[-1]):
        raise ValueError("suffix heads and dimension must match the query")
    _check_backend(query, RefineKVConfig(block_size=pages.block_size))
    if key_suffix.shape[1] and (key_suffix.dtype != torch.bfloat16
                                or value_suffix.dtype != torch.bfloat16):
        raise TypeError("the CUDA backend requires BF16 suffix K/V")
    if suffix_length is not None and (suffix_length.shape != () or
                                      suffix_length.dtype != torch.int32 or
                                      suffix_length.device != query.device):
        raise ValueError("suffix_length must be a scalar int32 tensor on the query device")
    heads, group, _, dim = query.shape
    dev = query.device
    q = query.reshape(heads, group, dim)
    if not q.is_contiguous():
        q = q.contiguous()
    capacity = key_suffix.shape[1]
    output = _buffer(workspace, "dense_output", (heads, group, dim), dev, query.dtype)
    lib = _native.load()
    with torch.cuda.device(dev):
        nbytes = lib.rkv_decode_dense_workspace_size(heads, group, pages.num_blocks, dim,
                                                     pages.block_size)
        scratch = _scratch(workspace, "rkv_dense_scratch", nbytes, dev)
        _native.check(lib.rkv_decode_dense(
            pages.abi(), q.data_ptr(), _query_code(q), group,
            key_suffix.data_ptr() if capacity else None,
            value_suffix.data_ptr() if capacity else None, capacity,
            key_suffix.stride(0), key_suffix.stride(1),
            value_suffix.stride(0), value_suffix.stride(1),
            suffix_length.data_ptr() if suffix_length is not None else None, capacity,
            output.data_ptr(), scratch.data_ptr(), scratch.numel(),
            torch.cuda.current_stream(dev).cuda_stream))
    return output.view(heads, group, 1, dim)

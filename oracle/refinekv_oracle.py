"""CPU oracle for the RefineKV decode path -- TEST INFRASTRUCTURE ONLY.

This module restates, in plain PyTorch on the CPU, the algorithm of the
reference implementation (Kevin-lkw/RefineKV-release v0.1.2, ``src/refinekv``)
for the three parts of the decode hot path:

* the post-prefill block summarizer      (``summary.py:35-113``),
* the per-step block selector            (``reference.py:10-47``),
* the mixed representative/exact softmax (``reference.py:50-73``),

plus the helpers the tests need to judge a CUDA result against it: the
eps-margin classifier, the decode access counters
(``integrations/transformers.py:590-594``) and a direct reading of the split
(m, l, o) partial merge.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
may import this file, and only as the checker or as the timed CPU baseline.
The product package never imports it: there is no CPU fallback.

Pinning: ``tests/golden/make_golden.py`` runs the reference package itself on
seeded inputs and stores its outputs under ``tests/golden/``;
``tests/test_oracle_golden.py`` requires this oracle to reproduce them.
"""

from __future__ import annotations

from dataclasses import dataclass
import math

import torch

_DIRECT_DELTA_MAX = 10.0
_DELTA_INFLATION = 1 + 2**-8  # upward rounding factor, reference.py:16 / summary.py:95


@dataclass
class OracleSummary:
    """Field-for-field twin of ``BlockSummary`` (``summary.py:10-32``)."""

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

    @property
    def num_blocks(self) -> int:
        return self.counts.numel()


def as_cpu_summary(summary) -> OracleSummary:
    """Copy any object with the ``BlockSummary`` fields to an ``OracleSummary`` on the CPU."""
    fields = ("keys", "values", "counts", "key_mean", "value_mean", "ellipsoid",
              "value_norm", "max_value_norm")
    return OracleSummary(
        **{name: getattr(summary, name).detach().cpu() for name in fields},
        prompt_length=int(summary.prompt_length),
        block_size=int(summary.block_size),
    )


# --------------------------------------------------------------------------
# Summarizer
# --------------------------------------------------------------------------

def page_view(tensor: torch.Tensor, block_size: int) -> torch.Tensor:
    """(heads, tokens, dim) -> (heads, pages, block, dim), zero padded to whole pages.

    Follows ``summary.py:35-43``: a copy is made only when the token count is
    not a page multiple or the reshape is not page-contiguous.
    """
    heads, length, dim = tensor.shape
    pad = -length % block_size
    if pad:
        tensor = torch.cat([tensor, torch.zeros(heads, pad, dim, dtype=tensor.dtype)], dim=1)
    paged = tensor.reshape(heads, (length + pad) // block_size, block_size, dim)
    if paged.stride()[1:] != (block_size * dim, dim, 1):
        paged = paged.contiguous()
    return paged


@torch.no_grad()
def build_summary(keys: torch.Tensor, values: torch.Tensor, block_size: int = 32,
                  chunk_blocks: int = 512) -> OracleSummary:
    """Block summaries, following ``summary.py:46-113`` step by step.

    Per (head, block): counts; bf16 means of K and V from FP32 sums
    (``:69-74``); the per-channel half width around the bf16 key mean over the
    real rows only (``:75-79``), squared and stored in bf16 (``:80``); the
    largest normalised centred squared distance of a real row (``:82-93``),
    passed through sqrt/square (``:94``) and folded with the squared width and
    the 1+2^-8 inflation into the bf16 ellipsoid (``:95-97``); the largest
    value row norm (``:98-101``) and its maximum over blocks (``:110``).
    """
    keys, values = keys.detach().cpu(), values.detach().cpu()
    length = keys.shape[1]
    kp, vp = page_view(keys, block_size), page_view(values, block_size)
    nb = kp.shape[1]
    tail = length - (nb - 1) * block_size
    counts = torch.full((nb,), block_size, dtype=torch.int64)
    counts[-1] = tail
    denom = counts.float().view(1, nb, 1)

    key_mean = (kp.sum(2, dtype=torch.float32) / denom).to(torch.bfloat16)
    value_mean = (vp.sum(2, dtype=torch.float32) / denom).to(torch.bfloat16)

    hi, lo = kp.amax(2), kp.amin(2)
    if tail < block_size:
        hi[:, -1] = kp[:, -1, :tail].amax(1)
        lo[:, -1] = kp[:, -1, :tail].amin(1)
    mean_f = key_mean.float()
    half_width = torch.maximum(hi.float() - mean_f, mean_f - lo.float())
    width_sq = half_width.clamp_min(1e-6).square().to(torch.bfloat16)

    ellipsoid = torch.empty_like(width_sq)
    for first in range(0, nb, chunk_blocks):
        last = min(first + chunk_blocks, nb)
        rows = kp[:, first:last].to(dtype=torch.float32, copy=True)
        rows -= mean_f[:, first:last, None]
        rows *= torch.rsqrt(width_sq[:, first:last].float())[:, :, None]
        dist = rows.square().sum(-1)
        if last == nb and tail < block_size:
            dist[:, -1, tail:] = -math.inf
        radius_sq = dist.amax(-1).clamp_min(0).sqrt().square()
        ellipsoid[:, first:last] = (
            radius_sq[..., None] * width_sq[:, first:last].float() * _DELTA_INFLATION
        ).to(torch.bfloat16)

    row_norm = torch.linalg.vector_norm(vp, dim=-1, dtype=torch.float32)
    if tail < block_size:
        row_norm[:, -1, tail:] = -math.inf
    value_norm = row_norm.amax(-1)
    return OracleSummary(kp, vp, counts, key_mean, value_mean, ellipsoid, value_norm,
                         value_norm.amax(-1), length, block_size)


# --------------------------------------------------------------------------
# Selector
# --------------------------------------------------------------------------

def _log_cosh(delta: torch.Tensor) -> torch.Tensor:
    """Two-branch log(cosh(delta)), ``reference.py:19-22``."""
    small = delta.clamp(max=_DIRECT_DELTA_MAX)
    direct = ((small.exp() + (-small).exp()) * 0.5).log()
    large = delta + ((1 + (-2 * delta).exp()) * 0.5).log()
    return torch.where(delta <= _DIRECT_DELTA_MAX, direct, large)


def _scores(query: torch.Tensor, summary):
    """z = q.kbar/sqrt(D) + log count and the inflated bound delta (``reference.py:11-16``)."""
    q = query[:, :, 0].to(torch.bfloat16).float()
    q_sq = q.square().to(torch.bfloat16).float()
    scale = q.shape[-1] ** -0.5
    score = torch.einsum("hgd,hbd->hgb", q, summary.key_mean.float()) * scale
    spread = torch.einsum("hgd,hbd->hgb", q_sq, summary.ellipsoid.float())
    delta = spread.clamp_min(0).sqrt() * scale * _DELTA_INFLATION
    z = score + summary.counts.float().log().view(1, 1, -1)
    return z, delta


@torch.no_grad()
def selection_statistics(query: torch.Tensor, summary):
    """Per (kv head, group row, block): z, risk, log_Z, log_C (``reference.py:10-34``).

    ``query`` is (kv_heads, group, 1, dim) in any float dtype; it is rounded
    to bf16 first, and so is its square (``:11-12``).
    """
    z, delta = _scores(query, summary)
    log_z = torch.logsumexp(z, -1, keepdim=True)
    log_c = torch.logsumexp(z + _log_cosh(delta), -1, keepdim=True)
    return z, _risk(z, delta, log_z, log_c, summary), log_z, log_c


def _risk(z, delta, log_z, log_c, summary):
    """Distortion + importance risk given the row normalisers (``reference.py:24-34``)."""
    small = delta.clamp(max=_DIRECT_DELTA_MAX)
    t = small.exp()
    near = delta <= _DIRECT_DELTA_MAX
    vmax = summary.max_value_norm.view(-1, 1, 1)
    # distortion ("mass") term, direct and large-delta forms (reference.py:25-31)
    mass_direct = 2 * vmax * (z - log_c).exp() * (0.5 * (t + t.reciprocal()) - 1)
    e_neg = (-delta).exp()
    log_cosh_m1 = delta + 2 * (1 - e_neg).clamp_min(1e-30).log() - math.log(2)
    mass_large = 2 * vmax * (z - log_c + log_cosh_m1).exp()
    mass = torch.where(near, mass_direct, mass_large)
    # importance ("value") term (reference.py:32-33)
    tanh_half = torch.where(near, (t - 1) / (t + 1), (1 - e_neg) / (1 + e_neg))
    importance = 2 * summary.value_norm.unsqueeze(1) * (z - log_z).exp() * tanh_half
    return mass + importance


def reduce_group(risk: torch.Tensor, eps: float, reduction: str) -> torch.Tensor:
    """GQA reduction of the (heads, group, blocks) risk, ``reference.py:39-44``."""
    if reduction == "mean":
        return risk.mean(1) > eps
    if reduction == "max":
        return risk.amax(1) > eps
    if reduction == "any":
        return (risk > eps).any(1)
    raise ValueError(reduction)


@torch.no_grad()
def select_blocks(query, summary, eps: float, reduction: str):
    """Mask and representative logits, ``reference.py:37-47``.

    A block is also forced on when any row of its group has a non-finite
    global normaliser or a non-finite risk for it.
    """
    z, risk, log_z, log_c = selection_statistics(query, summary)
    chosen = reduce_group(risk, eps, reduction)
    forced_all = (~torch.isfinite(log_z) | ~torch.isfinite(log_c)).any(1)
    forced_one = (~torch.isfinite(risk)).any(1)
    return chosen | forced_all | forced_one, z


def margin_blocks(query, summary, eps: float, reduction: str, rel: float = 1e-3):
    """Blocks whose decision lies within ``rel`` (relative) of ``eps``.

    For ``mean`` the group mean is tested, for ``max``/``any`` every row's
    risk is: a block is in the margin if a statistic that can decide it lies
    in [eps(1-rel), eps(1+rel)].  The tolerance has an absolute floor of
    1e-30 so that eps == 0 still has a (tiny) margin.
    """
    _, risk, _, _ = selection_statistics(query, summary)
    band = max(rel * eps, 1e-30)
    if reduction == "mean":
        return (risk.mean(1) - eps).abs() <= band
    return ((risk - eps).abs() <= band).any(1)


# --------------------------------------------------------------------------
# Mixed attention
# --------------------------------------------------------------------------

@torch.no_grad()
def mixed_attention(query, summary, key_suffix, value_suffix, selected, z):
    """Softmax over representatives, expanded pages and the suffix for a given mask.

    Follows the per-head loop of ``reference.py:59-72``: unselected blocks
    enter as one representative with logit ``z`` and value ``value_mean``;
    selected blocks with their real rows (``q.k * dim^-1/2``); every suffix
    row is exact.  Returns FP32 (kv_heads, group, 1, dim).
    """
    q = query[:, :, 0].to(torch.bfloat16).float()
    scale = q.shape[-1] ** -0.5
    row_ids = torch.arange(summary.block_size)
    out = []
    for h in range(q.shape[0]):
        live = selected[h, :, None] & (row_ids[None] < summary.counts[:, None])
        k_rows = torch.cat([summary.keys[h][live].to(torch.bfloat16).float(),
                            key_suffix[h].to(torch.bfloat16).float()])
        v_rows = torch.cat([summary.values[h][live].to(torch.bfloat16).float(),
                            value_suffix[h].to(torch.bfloat16).float()])
        logits = torch.cat([z[h][:, ~selected[h]], q[h] @ k_rows.T * scale], -1)
        vals = torch.cat([summary.value_mean[h][~selected[h]].float(), v_rows], 0)
        out.append(logits.softmax(-1) @ vals)
    return torch.stack(out).unsqueeze(2)


@torch.no_grad()
def sparse_attention(query, summary, key_suffix, value_suffix, eps, reduction,
                     anchor_mask=None):
    """Output (in the query dtype) and mask, ``reference.py:50-73``."""
    selected, z = select_blocks(query, summary, eps, reduction)
    if anchor_mask is not None:
        selected = selected | anchor_mask.cpu()
    out = mixed_attention(query, summary, key_suffix, value_suffix, selected, z)
    return out.to(query.dtype), selected


def anchor_union(anchor_queries, summary, eps, reduction):
    """OR of per-anchor masks, ``integrations/transformers.py:543-552``.

    ``anchor_queries`` is (anchors, kv_heads, group, 1, dim).
    """
    mask = None
    for q in anchor_queries:
        sel = select_blocks(q, summary, eps, reduction)[0]
        mask = sel if mask is None else mask | sel
    return mask


def access_counters(selected, counts, group, query_heads, suffix_len, prompt_len):
    """Decode access counters, ``integrations/transformers.py:590-594``."""
    accessed = ((selected * counts).sum() + (~selected).sum()) * group + query_heads * suffix_len
    return int(accessed), int(query_heads * (prompt_len + suffix_len))


def merge_partials(m, l, o):
    """Merge split-softmax partials: m, l (..., S) and o (..., S, D) -> (..., D).

    This is the LSE combine of ``kernels/attention.py:297-329`` written out
    directly; ``o`` holds un-normalised sums relative to ``m``.
    """
    top = m.amax(-1, keepdim=True)
    top = torch.where(torch.isfinite(top), top, torch.zeros_like(top))
    w = torch.where(torch.isfinite(m), (m - top).exp(), torch.zeros_like(m))
    denom = (l * w).sum(-1, keepdim=True).clamp_min(1e-30)
    return (o * w.unsqueeze(-1)).sum(-2) / denom


# --------------------------------------------------------------------------
# Sequence split (prompt blocks spread over ranks)
# --------------------------------------------------------------------------
# The reference has no multi-GPU mode.  These functions write the decode step
# of ``reference.py:10-73`` as per-rank pieces and merges, so that a test can
# run them on separate (CPU, gloo) ranks and compare with the one-piece
# functions above: log Z and log C (``reference.py:15-17``) and the softmax
# denominator are the only sums that cross block ranges.

@torch.no_grad()
def normalizer_partials(query, summary):
    """(heads, group, 4): max and sum of exp(. - max) for z and z + log cosh(delta) over this summary's blocks."""
    z, delta = _scores(query, summary)
    c = z + _log_cosh(delta)
    mz, mc = z.amax(-1, keepdim=True), c.amax(-1, keepdim=True)
    sz, sc = (z - mz).exp().sum(-1, keepdim=True), (c - mc).exp().sum(-1, keepdim=True)
    return torch.cat([mz, sz, mc, sc], -1)


def merge_normalizers(partials):
    """(ranks, heads, group, 4) partials -> log Z, log C of shape (heads, group, 1)."""
    def lse(m, s):
        top = m.amax(0)
        return top + (s * (m - top).exp()).sum(0).log()
    return (lse(partials[..., 0], partials[..., 1]).unsqueeze(-1),
            lse(partials[..., 2], partials[..., 3]).unsqueeze(-1))


@torch.no_grad()
def select_blocks_given(query, summary, log_z, log_c, eps: float, reduction: str):
    """``select_blocks`` with row normalisers computed over the whole prompt elsewhere."""
    z, delta = _scores(query, summary)
    risk = _risk(z, delta, log_z, log_c, summary)
    chosen = reduce_group(risk, eps, reduction)
    forced_all = (~torch.isfinite(log_z) | ~torch.isfinite(log_c)).any(1)
    forced_one = (~torch.isfinite(risk)).any(1)
    return chosen | forced_all | forced_one, z


@torch.no_grad()
def mixed_attention_partial(query, summary, key_suffix, value_suffix, selected, z):
    """This rank's share of ``mixed_attention``: per row (max, sum) and the normalised output.

    Returns m, l of shape (heads, group) and o of shape (heads, group, dim).
    """
    q = query[:, :, 0].to(torch.bfloat16).float()
    scale = q.shape[-1] ** -0.5
    row_ids = torch.arange(summary.block_size)
    ms, ls, os_ = [], [], []
    for h in range(q.shape[0]):
        live = selected[h, :, None] & (row_ids[None] < summary.counts[:, None])
        k_rows = torch.cat([summary.keys[h][live].to(torch.bfloat16).float(),
                            key_suffix[h].to(torch.bfloat16).float()])
        v_rows = torch.cat([summary.values[h][live].to(torch.bfloat16).float(),
                            value_suffix[h].to(torch.bfloat16).float()])
        logits = torch.cat([z[h][:, ~selected[h]], q[h] @ k_rows.T * scale], -1)
        vals = torch.cat([summary.value_mean[h][~selected[h]].float(), v_rows], 0)
        m = logits.amax(-1, keepdim=True)
        p = (logits - m).exp()
        l = p.sum(-1, keepdim=True)
        ms.append(m[:, 0])
        ls.append(l[:, 0])
        os_.append((p @ vals) / l)
    return torch.stack(ms), torch.stack(ls), torch.stack(os_)


def merge_rank_outputs(m, l, o):
    """(ranks, heads, group), (ranks, heads, group), (ranks, heads, group, dim) -> (heads, group, 1, dim)."""
    top = m.amax(0)
    w = l * (m - top).exp()
    return ((w.unsqueeze(-1) * o).sum(0) / w.sum(0).unsqueeze(-1)).unsqueeze(2)

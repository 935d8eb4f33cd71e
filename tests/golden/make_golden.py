"""Generate golden fixtures by running the reference RefineKV package itself.

Run once in a container that has the reference source tree (it is not needed
afterwards; the fixtures are committed):

    REFINEKV_REFERENCE_SRC=<reference>/src python tests/golden/make_golden.py

It imports the reference ``refinekv`` package (v0.1.2) and records, for seeded
inputs, what its PyTorch backend returns:

* ``build_summary`` for every block size, partial and full tails, BF16 and
  FP32 caches and a strided cache prefix (reference ``tests/test_attention.py:19-56``);
* ``selection_statistics`` / ``select_blocks_reference`` / ``sparse_attention``
  on the four GPU-agreement shapes of ``tests/test_attention.py:139-183`` and
  the suffix lengths 0 and 5 with a last-block anchor;
* the known-answer, anchor-only and large-query cases (``:93-128``);
* a scaled-down synthetic workload (8 KV heads, group 4, dim 128, FP32 and
  BF16, 32 anchors, three decode steps) from ``refinekv_b200.synthetic``.

Large inputs are not stored: they are regenerated from their seed in the
tests, and a checksum recorded here proves the regeneration is identical.
"""

from __future__ import annotations

import hashlib
import os
import pathlib
import sys

import torch

HERE = pathlib.Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "refinekv-release_b200"))
if "REFINEKV_REFERENCE_SRC" not in os.environ:
    sys.exit("set REFINEKV_REFERENCE_SRC to the reference source tree's src directory")
sys.path.insert(0, os.environ["REFINEKV_REFERENCE_SRC"])

import refinekv  # noqa: E402  (the reference package)
from refinekv import RefineKVConfig, build_summary, sparse_attention  # noqa: E402
from refinekv.reference import selection_statistics, select_blocks_reference  # noqa: E402
from refinekv_b200 import synthetic  # noqa: E402

assert refinekv.__version__ == "0.1.2", refinekv.__version__
assert "reference" in refinekv.__file__ or "src/refinekv" in refinekv.__file__


def checksum(t: torch.Tensor) -> list:
    f = t.detach().float().reshape(-1)
    idx = torch.linspace(0, f.numel() - 1, steps=min(64, f.numel())).long()
    return [float(f.double().sum()), float(f.double().abs().sum())] + f[idx].tolist()


def digest(t: torch.Tensor) -> dict:
    """Exact fingerprint of a tensor too large to store: dtype, shape, SHA-256 of its bytes."""
    t = t.detach().contiguous().cpu()
    raw = t.view(torch.uint8) if t.dtype != torch.bool else t.to(torch.uint8)
    return dict(dtype=str(t.dtype), shape=tuple(t.shape),
                sha256=hashlib.sha256(raw.numpy().tobytes()).hexdigest(), checksum=checksum(t))


def reference_inputs(length, dim, seed=42):
    """The reference tests' ``_inputs`` draw (tests/test_attention.py:10-16)."""
    gen = torch.Generator().manual_seed(seed)

    def normal(shape):
        return torch.randn(shape, generator=gen, dtype=torch.bfloat16)

    return normal((2, 4, 1, dim)), normal((2, length, dim)), normal((2, length, dim))


def summary_fields(s, exact=True):
    names = ("counts", "key_mean", "value_mean", "ellipsoid", "value_norm", "max_value_norm")
    if exact:
        return {name: getattr(s, name).clone() for name in names}
    return {name: digest(getattr(s, name)) for name in names}


def summary_cases():
    cases = []
    for block in (16, 32, 64):
        for length in (block + 3, 2 * block, 5 * block - 1):
            for dtype in (torch.bfloat16, torch.float32):
                if dtype == torch.float32 and length != block + 3:
                    continue
                gen = torch.Generator().manual_seed(1000 + block + length)
                keys = torch.randn(2, length, 64, generator=gen).to(dtype)
                values = torch.randn(2, length, 64, generator=gen).to(dtype)
                cfg = RefineKVConfig(block_size=block, summary_chunk_blocks=2, backend="torch")
                s = build_summary(keys, values, cfg)
                cases.append(dict(block=block, length=length, dtype=str(dtype), chunk=2,
                                  keys=keys, values=values, out=summary_fields(s),
                                  key_pages=s.keys.clone(), value_pages=s.values.clone()))
    # constant channels (width clamp) and a strided prefix of a larger cache
    q, keys, values = reference_inputs(65, 128)
    keys[..., :3] = torch.tensor([96, 48, -80], dtype=torch.bfloat16)
    cache = torch.cat([keys, torch.zeros_like(keys)], 1)[:, :65]
    s = build_summary(cache, values, RefineKVConfig(summary_chunk_blocks=1, backend="torch"))
    cases.append(dict(block=32, length=65, dtype=str(torch.bfloat16), chunk=1,
                      keys=cache.contiguous(), values=values, out=summary_fields(s),
                      key_pages=s.keys.clone(), value_pages=s.values.clone()))
    return cases


def selection_record(q, summary, cfg, anchor, suffix_keys, suffix_values):
    z, risk, log_z, log_c = selection_statistics(q, summary)
    mask, z2 = select_blocks_reference(q, summary, cfg)
    assert torch.equal(z, z2)
    outs = {}
    for n in sorted({0, 5, suffix_keys.shape[1]}):
        res = sparse_attention(q, summary, suffix_keys[:, :n], suffix_values[:, :n], cfg,
                               anchor_mask=anchor, return_selected=True)
        outs[n] = dict(output=res.output.clone(), selected=res.selected.clone())
    return dict(z=z, risk=risk, log_z=log_z, log_c=log_c, mask=mask, attention=outs)


def agreement_cases():
    """Shapes of the reference's Triton-vs-torch agreement test (test_attention.py:139-183)."""
    cases = []
    for block, reduction, eps, length, dim in [
        (16, "any", 0.0, 71, 64),
        (32, "mean", 0.1, 71, 128),
        (64, "max", 1e6, 71, 64),
        (16, "any", 0.2, 25001, 128),
    ]:
        q, keys, values = reference_inputs(length, dim)
        cfg = RefineKVConfig(block_size=block, eps=eps, gqa_reduction=reduction, backend="torch")
        summary = build_summary(keys, values, cfg)
        anchor = torch.zeros(2, summary.num_blocks, dtype=torch.bool)
        anchor[:, -1] = True
        rec = selection_record(q, summary, cfg, anchor, keys[:, :5], values[:, :5])
        small = length < 1000
        cases.append(dict(
            name=f"agree_b{block}_{reduction}_eps{eps}_n{length}_d{dim}",
            block=block, reduction=reduction, eps=eps, length=length, dim=dim, seed=42,
            q=q, keys=keys if small else None, values=values if small else None,
            input_checksum=[checksum(q), checksum(keys), checksum(values)],
            summary=summary_fields(summary, exact=small), anchor=anchor, suffix_from_prompt=5,
            **rec))
    return cases


def special_cases():
    cases = {}
    # known answer (16 + 9) / 19, test_attention.py:93-103
    cfg = RefineKVConfig(backend="torch", eps=1e6, block_size=16)
    keys = torch.zeros(1, 19, 64, dtype=torch.bfloat16)
    values = torch.zeros_like(keys)
    values[:, :16] = 1
    values[:, 16:] = 3
    s = build_summary(keys, values, cfg)
    q = torch.zeros(1, 2, 1, 64)
    res = sparse_attention(q, s, keys[:, :0], values[:, :0], cfg, return_selected=True)
    cases["known_answer"] = dict(keys=keys, values=values, q=q, block=16, eps=1e6,
                                 reduction="any", output=res.output, selected=res.selected)
    # large finite delta, test_attention.py:119-128
    q, keys, values = reference_inputs(71, 64)
    q = (q.float() * 200).to(torch.bfloat16)
    cfg = RefineKVConfig(backend="torch")
    s = build_summary(keys, values, cfg)
    z, risk, log_z, log_c = selection_statistics(q, s)
    res = sparse_attention(q, s, keys[:, :0], values[:, :0], cfg, return_selected=True)
    cases["large_query"] = dict(keys=keys, values=values, q=q, block=32, eps=0.01,
                                reduction="any", z=z, risk=risk, log_z=log_z, log_c=log_c,
                                output=res.output, selected=res.selected)
    return cases


def synthetic_case(dtype):
    """Scaled-down config-0 workload: 8 KV heads, group 4, dim 128, 4096 prompt tokens."""
    seed, layer, heads, group, dim, tokens, block = 0, 0, 8, 4, 128, 4096, 32
    eps, reduction, anchors, steps = 0.01, "any", 32, 3
    data = synthetic.make_layer(seed, layer, heads, tokens, dim, block, dtype=dtype)
    cfg = RefineKVConfig(block_size=block, eps=eps, gqa_reduction=reduction, backend="torch")
    summary = build_summary(data.keys, data.values, cfg)
    anchor_q = synthetic.make_queries(seed, layer, -1, data.planted_mean, group, anchors, dtype)
    anchor = None
    for a in range(anchors):
        sel = refinekv.select_blocks(anchor_q[a], summary, cfg)
        anchor = sel if anchor is None else anchor | sel
    suffix_k, suffix_v = [], []
    per_step = []
    for step in range(steps):
        k, v = synthetic.make_decode_token(seed, layer, step, heads, dim, tokens + step, dtype)
        suffix_k.append(k)
        suffix_v.append(v)
        q = synthetic.make_queries(seed, layer, step, data.planted_mean, group, 1, dtype)[0]
        ks, vs = torch.cat(suffix_k, 1), torch.cat(suffix_v, 1)
        z, risk, log_z, log_c = selection_statistics(q, summary)
        res = sparse_attention(q, summary, ks, vs, cfg, anchor_mask=anchor, return_selected=True)
        per_step.append(dict(q=q, z=z, risk=risk, log_z=log_z, log_c=log_c,
                             output=res.output, selected=res.selected))
    return dict(seed=seed, layer=layer, heads=heads, group=group, dim=dim, tokens=tokens,
                block=block, eps=eps, reduction=reduction, anchors=anchors, steps=steps,
                dtype=str(dtype), input_checksum=[checksum(data.keys), checksum(data.values)],
                summary=summary_fields(summary, exact=False), anchor_mask=anchor,
                per_step=per_step)


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    fixtures = dict(
        reference_version=refinekv.__version__,
        torch_version=torch.__version__,
        summary_cases=summary_cases(),
        agreement_cases=agreement_cases(),
        special_cases=special_cases(),
        synthetic_cases=[synthetic_case(torch.float32), synthetic_case(torch.bfloat16)],
    )
    path = HERE / "golden_refinekv_v0_1_2.pt"
    torch.save(fixtures, path)
    print(f"wrote {path} ({path.stat().st_size / 1e6:.2f} MB)")


if __name__ == "__main__":
    main()
